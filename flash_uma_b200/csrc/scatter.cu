// Inverse rotation out of the edge frame + envelope + deterministic FP64 segment sum
// over the destination CSR (+ residual), and the initial edge-degree node embedding.
//
// Reference: ops/scatter.py:45-140 (rotate-scatter forward), :146-292 (backward),
//            :360-423 (init scatter forward), :426-481 (init backward).
//
// Per edge e, channel c (C-wide slots):
//   Z_m0 [E,3C] = [l0, l1(m=0), l2(m=0)]; Z_m1 [E,4C] = [R_l1, R_l2, I_l1, I_l2]; Z_m2 [E,2C] = [R_l2, I_l2]
//   edge-frame rows  m1 = (I_l1, l1(m=0), R_l1),  m2 = (I_m2, I_l2, l2(m=0), R_l2, R_m2)
//   message = env_e * [Z_m0[0]; D1^T m1; D2^T m2]
// x_out[j] = x_res[j] + sum_{e in CSR row j} message_e, summed in fp64 in CSR order
// (products in fp32), then rounded to fp32 once. Deterministic run to run.
//
// One warp per destination node and coefficient block; lane l owns channels [4l, 4l+4)
// (+128 per extra group), 16-byte coalesced accesses; the per-edge Wigner values are staged
// in shared memory and broadcast.
#include "common.cuh"
#include "kernels.h"

namespace fuma {

namespace {

constexpr int kFwdWarps = 4;   // rotate-scatter forward: warps per block (static ring below 48 KB)
constexpr int kRing = 4;       // edges staged per warp (rotate-scatter forward, init scatter)

}  // namespace

// Forward, warp per destination atom, one launch per coefficient block (PART 0: rows 0-3, l <= 1,
// Wigner 0-8; PART 1: rows 4-8, l = 2, Wigner 9-33; disjoint rows of x_out). The atom's edges are summed one at a time in CSR
// order into fp64 accumulators; their Z slots, Wigner block and envelope are copied into a
// per-warp ring of kRing shared-memory buffers with cp.async, kRing - 1 edges ahead of the sum,
// so a warp waits for memory about once per kRing - 1 edges instead of once per edge.
template <int PART, bool kH>
__global__ void __launch_bounds__(128, 4) rotate_scatter_fwd_kernel(
    const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col_idx, const float* __restrict__ Z0,
    const float* __restrict__ Z1, const float* __restrict__ Z2, const float* __restrict__ wig,
    const float* __restrict__ env, const float* __restrict__ x_res, float* __restrict__ x_out, int64_t N, int C) {
  constexpr int kRows = PART ? 5 : 4;
  constexpr int kW = PART ? 25 : 9;
  constexpr int kWoff = PART ? 9 : 0;
  constexpr int kRow0 = PART ? 4 : 0;
  constexpr int kS = PART ? 5 : 4;   // Z slots per edge and lane (16-byte copies)
  __shared__ float4 s_stage[kFwdWarps][kRing][kS][32];
  __shared__ float s_w[kFwdWarps][kRing][28];   // Wigner block (0..kW-1) and envelope (27)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C4 = C >> 2;
  // grid-stride over atoms: contiguous even shares (warp_share) measured 4% slower here
  for (int64_t jn = (int64_t)blockIdx.x * kFwdWarps + warp; jn < N; jn += (int64_t)gridDim.x * kFwdWarps) {
    const int kb = row_ptr[jn], ke = row_ptr[jn + 1];
    for (int cb = 0; cb < C4; cb += 32) {
      const int c4 = cb + lane;
      const bool on = c4 < C4;
      const int co = c4 * 4;
      // copies of edge e's Z slots (in the order the sum reads them), Wigner block and envelope
      // into ring buffer b, one commit group per edge
      auto issue = [&](int64_t e, int b) {
        if (on) {
          // element offsets of the edge's rows (fp32, or fp16 with kH)
          const int64_t z0 = e * 3 * (int64_t)C + co, z1 = e * 4 * (int64_t)C + co, z2 = e * 2 * (int64_t)C + co;
          float4* d = &s_stage[warp][b][0][lane];
          if constexpr (PART == 0) {
            cp_act<kH>(d + 0 * 32, Z0, z0);
            cp_act<kH>(d + 1 * 32, Z1, z1 + 2 * C);
            cp_act<kH>(d + 2 * 32, Z0, z0 + C);
            cp_act<kH>(d + 3 * 32, Z1, z1);
          } else {
            cp_act<kH>(d + 0 * 32, Z2, z2 + C);
            cp_act<kH>(d + 1 * 32, Z1, z1 + 3 * C);
            cp_act<kH>(d + 2 * 32, Z0, z0 + 2 * C);
            cp_act<kH>(d + 3 * 32, Z1, z1 + C);
            cp_act<kH>(d + 4 * 32, Z2, z2);
          }
        }
        if (lane < kW) cp_async4(&s_w[warp][b][lane], wig + e * kWig + kWoff + lane);
        if (lane == 31) cp_async4(&s_w[warp][b][27], env + e);
        cp_async_commit();
      };
      // the edge list, 32 entries at a time in a lane register; `ib` is the window's first edge
      int ib = kb;
      int e_l = (kb + lane < ke) ? col_idx[kb + lane] : 0;
      int ki = kb;   // next CSR position to copy
      auto issue_next = [&]() {
        if (ki < ke) {
          if (ki - ib >= 32) {
            ib += 32;
            e_l = (ib + lane < ke) ? col_idx[ib + lane] : 0;
          }
          issue(__shfl_sync(kFull, e_l, ki - ib), (ki - kb) % kRing);
        } else {
          cp_async_commit();   // empty group keeps "groups in flight" counting edges
        }
        ++ki;
      };
#pragma unroll 1
      for (int p = 0; p < kRing - 1; ++p) issue_next();
      d4 acc[kRows];
      if (on) {
        const float* xr = x_res + jn * 9 * (int64_t)C + kRow0 * C + co;
#pragma unroll
        for (int l = 0; l < kRows; ++l) acc[l] = d4_of(ld4(xr + l * C));
      }
#pragma unroll 1
      for (int k = kb; k < ke; ++k) {
        issue_next();   // refills the buffer summed in the previous iteration
        cp_async_wait<kRing - 1>();
        __syncwarp();
        const int b = (k - kb) % kRing;
        const float* D = s_w[warp][b];
        const float ev = D[27];
        const float4* src = &s_stage[warp][b][0][lane];
        if (on) {
          if constexpr (PART == 0) {
            acc[0] += sm_act<kH>(src) * ev;
            const float4 m0 = sm_act<kH>(src + 32), m1 = sm_act<kH>(src + 64), m2 = sm_act<kH>(src + 96);
#pragma unroll
            for (int kk = 0; kk < 3; ++kk) {
              float4 a = D[kk] * m0;
              fma4(a, D[3 + kk], m1);
              fma4(a, D[6 + kk], m2);
              acc[1 + kk] += a * ev;
            }
          } else {
            float4 m[5];
#pragma unroll
            for (int r = 0; r < 5; ++r) m[r] = sm_act<kH>(src + 32 * r);
#pragma unroll
            for (int kk = 0; kk < 5; ++kk) {
              float4 a = D[kk] * m[0];
#pragma unroll
              for (int r = 1; r < 5; ++r) fma4(a, D[r * 5 + kk], m[r]);
              acc[kk] += a * ev;
            }
          }
        }
        __syncwarp();   // buffer b is refilled by the next iteration's copies
      }
      cp_async_wait<0>();   // the trailing (empty) groups
      if (on) {
        float* xo = x_out + jn * 9 * (int64_t)C + kRow0 * C + co;
#pragma unroll
        for (int l = 0; l < kRows; ++l) st4(xo + l * C, f4_of(acc[l]));
      }
    }
  }
}

// Backward, grouped by destination so g_out[j] stays in L1 across the node's edges, one launch
// per coefficient block (PART 0: rows 0-3 / Z slots of l <= 1 / Wigner 0-8; PART 1: rows 4-8 /
// l = 2 slots / Wigner 9-33):
//   g_Z = env * (rows of D applied to g_out[j]); g_wigner[e] = env * sum_c g_out[j] (x) m;
//   g_env[e] = sum_c g_out[j] . (unscaled message): PART 0 writes its share, PART 1 (launched
//   after it on the same stream) adds the rest, so the sum has a fixed order.
// (g_x_res = g_out is returned by the host.)
template <int PART, bool kH>
__global__ void __launch_bounds__(256, 2) rotate_scatter_bwd_kernel(
    const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col_idx, const float* __restrict__ g_out,
    const float* __restrict__ Z0, const float* __restrict__ Z1, const float* __restrict__ Z2,
    const float* __restrict__ wig, const float* __restrict__ env, float* __restrict__ gZ0, float* __restrict__ gZ1,
    float* __restrict__ gZ2, float* __restrict__ g_wig, float* __restrict__ g_env, int64_t N, int C, int split,
    int* err) {
  constexpr int kW = PART ? 25 : 9;
  constexpr int kWoff = PART ? 9 : 0;
  constexpr int kRows = PART ? 5 : 4;
  constexpr int kRow0 = PART ? 4 : 0;
  constexpr int kS = PART ? 5 : 4;     // Z slots per edge and lane (16-byte copies)
  constexpr int NV = PART ? 32 : 16;   // kW Wigner partials (+ g0 . Z0_0 at index 9 in PART 0), padded
  __shared__ float4 s_stage[8][2][kS][32];
  __shared__ float s_w[8][2][28];      // Wigner block (0..kW-1) and envelope (27) of the staged edge
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  const int C4 = C >> 2;
  float amax = 0.f;   // largest magnitude written as a split (range check at the end)
  const Share sh = warp_share(N, (int64_t)blockIdx.x * wpb + warp, (int64_t)gridDim.x * wpb);
  for (int64_t jn = sh.begin; jn < sh.end; ++jn) {
    const int kb = row_ptr[jn], ke = row_ptr[jn + 1];
    for (int cb = 0; cb < C4; cb += 32) {
      const int c4 = cb + lane;
      const bool on = c4 < C4;
      const int co = c4 * 4;
      // copies of edge e's Z slots, Wigner block and envelope into buffer b (one commit group);
      // the next edge's copies are in flight while the current edge is computed
      auto issue = [&](int64_t e, int b) {
        if (on) {
          // element offsets of the edge's rows (fp32, or fp16 with kH)
          const int64_t z0 = e * 3 * (int64_t)C + co, z1 = e * 4 * (int64_t)C + co, z2 = e * 2 * (int64_t)C + co;
          float4* d = &s_stage[warp][b][0][lane];
          if constexpr (PART == 0) {
            cp_act<kH>(d + 0 * 32, Z0, z0);
            cp_act<kH>(d + 1 * 32, Z1, z1 + 2 * C);
            cp_act<kH>(d + 2 * 32, Z0, z0 + C);
            cp_act<kH>(d + 3 * 32, Z1, z1);
          } else {
            cp_act<kH>(d + 0 * 32, Z2, z2 + C);
            cp_act<kH>(d + 1 * 32, Z1, z1 + 3 * C);
            cp_act<kH>(d + 2 * 32, Z0, z0 + 2 * C);
            cp_act<kH>(d + 3 * 32, Z1, z1 + C);
            cp_act<kH>(d + 4 * 32, Z2, z2);
          }
        }
        if (lane < kW) cp_async4(&s_w[warp][b][lane], wig + e * kWig + kWoff + lane);
        if (lane == 31) cp_async4(&s_w[warp][b][27], env + e);
        cp_async_commit();
      };
      // this block's rows of g_out[j], loaded once per node
      float4 g[kRows];
#pragma unroll
      for (int l = 0; l < kRows; ++l) g[l] = on ? ld4_keep(g_out + (jn * 9 + kRow0 + l) * (int64_t)C + co) : f4(0.f);
      int base = kb;
      int e_l = (kb + lane < ke) ? col_idx[kb + lane] : 0;
      int64_t e_cur = __shfl_sync(kFull, e_l, 0);
      if (kb < ke) issue(e_cur, 0);
      for (int k = kb; k < ke; ++k) {
        const int b = (k - kb) & 1;
        int64_t e_next = 0;
        if (k + 1 < ke) {
          if (k + 1 - base >= 32) {
            base += 32;
            e_l = (base + lane < ke) ? col_idx[base + lane] : 0;
          }
          e_next = __shfl_sync(kFull, e_l, k + 1 - base);
          issue(e_next, b ^ 1);
        } else {
          cp_async_commit();   // empty group: "all but the newest group" is then edge k
        }
        cp_async_wait1();
        __syncwarp();
        const int64_t e = e_cur;
        const float* sw = s_w[warp][b];
        const float ev = sw[27];
        const float4* src = &s_stage[warp][b][0][lane];
        const float4 zz = f4(0.f);
        float* q0 = gZ0 + e * 3 * (int64_t)C;   // gradient rows; columns slot * C + co
        float* q1 = gZ1 + e * 4 * (int64_t)C;
        float* q2 = gZ2 + e * 2 * (int64_t)C;
        float part[NV];
#pragma unroll
        for (int m = 0; m < NV; ++m) part[m] = 0.f;
        if constexpr (PART == 0) {
          const float4 zl0 = on ? sm_act<kH>(src) : zz;
          const float4 m1[3] = {on ? sm_act<kH>(src + 32) : zz, on ? sm_act<kH>(src + 64) : zz,
                                on ? sm_act<kH>(src + 96) : zz};
          float4 t1[3];
#pragma unroll
          for (int r = 0; r < 3; ++r) {
            float4 a = sw[r * 3] * g[1];
            fma4(a, sw[r * 3 + 1], g[2]);
            fma4(a, sw[r * 3 + 2], g[3]);
            t1[r] = a * ev;
          }
          if (on) {
            st_out4(q0, 3 * C, co, g[0] * ev, split, amax);
            st_out4(q0, 3 * C, C + co, t1[1], split, amax);
            st_out4(q1, 4 * C, co, t1[2], split, amax);
            st_out4(q1, 4 * C, 2 * C + co, t1[0], split, amax);
          }
#pragma unroll
          for (int r = 0; r < 3; ++r)
#pragma unroll
            for (int kk = 0; kk < 3; ++kk) part[r * 3 + kk] = dot4(g[1 + kk], m1[r]);
          part[9] = dot4(g[0], zl0);
        } else {
          const float4 m2[5] = {on ? sm_act<kH>(src) : zz, on ? sm_act<kH>(src + 32) : zz,
                                on ? sm_act<kH>(src + 64) : zz, on ? sm_act<kH>(src + 96) : zz,
                                on ? sm_act<kH>(src + 128) : zz};
          float4 t2[5];
#pragma unroll
          for (int r = 0; r < 5; ++r) {
            float4 a = sw[r * 5] * g[0];
#pragma unroll
            for (int kk = 1; kk < 5; ++kk) fma4(a, sw[r * 5 + kk], g[kk]);
            t2[r] = a * ev;
          }
          if (on) {
            st_out4(q0, 3 * C, 2 * C + co, t2[2], split, amax);
            st_out4(q1, 4 * C, C + co, t2[3], split, amax);
            st_out4(q1, 4 * C, 3 * C + co, t2[1], split, amax);
            st_out4(q2, 2 * C, co, t2[4], split, amax);
            st_out4(q2, 2 * C, C + co, t2[0], split, amax);
          }
#pragma unroll
          for (int r = 0; r < 5; ++r)
#pragma unroll
            for (int kk = 0; kk < 5; ++kk) part[r * 5 + kk] = dot4(g[kk], m2[r]);
        }
        // lane l < kW: the channel sum of Wigner partial l (lane 9: g0 . Z0_0 in PART 0)
        const float tot = warp_transpose_sum<NV>(part, lane);
        // g_env share: sum_{r,k} D[r][k] raw[r][k] (+ g0 . Z0_0 in PART 0)
        float genv = warp_sum(lane < kW ? sw[lane] * tot : 0.f);
        if (PART == 0) genv += __shfl_sync(kFull, tot, 9);
        if (lane < kW) {
          float* dst = g_wig + e * kWig + kWoff + lane;
          *dst = cb == 0 ? tot * ev : *dst + tot * ev;
        }
        if (lane == 0) g_env[e] = (PART == 0 && cb == 0) ? genv : g_env[e] + genv;
        __syncwarp();   // buffer b is refilled by the next iteration's copies
        e_cur = e_next;
      }
    }
  }
  report_split_range(amax, err);
}

// Initial embedding scatter (the reference's init_node_scatter forward, ops/scatter.py:382-423),
// warp per destination atom: x[n] = W_sphere[Z_n] + csd[batch_n] on l = 0, plus over the atom's
// edges in CSR order env * [r0; D1 row 1 r1; D2 row 2 r2] / 5 in fp64 accumulators. Each edge's
// radial row, Wigner entries and envelope are copied into a per-warp cp.async ring kRing - 1
// edges ahead of the sum (the per-edge arithmetic and its order are unchanged).
template <int WARPS>
__global__ void __launch_bounds__(WARPS * 32) init_scatter_fwd_kernel(
    const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col_idx, const float* __restrict__ rad,
    const float* __restrict__ wig, const float* __restrict__ env, const int64_t* __restrict__ Z,
    const int64_t* __restrict__ batch, const float* __restrict__ W_sphere, const float* __restrict__ csd,
    float* __restrict__ x_out, int64_t N, int C) {
  __shared__ float4 s_stage[WARPS][kRing][3][32];   // radial slots 0-2 of the staged edges
  __shared__ float s_w[WARPS][kRing][12];          // D1 row 1 (0-2), D2 row 2 (3-7), envelope (8)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C4 = C >> 2;
  const Share sh = warp_share(N, (int64_t)blockIdx.x * WARPS + warp, (int64_t)gridDim.x * WARPS);
  for (int64_t jn = sh.begin; jn < sh.end; ++jn) {
    const int kb = row_ptr[jn], ke = row_ptr[jn + 1];
    const int64_t z = Z[jn], b = batch[jn];
    for (int c0 = 0; c0 < C4; c0 += 32) {
      const int c4 = c0 + lane;
      const bool act = c4 < C4;
      const int co = c4 * 4;
      auto issue = [&](int64_t e, int bf) {
        if (act) {
          const float* rr = rad + e * 3 * (int64_t)C + co;
          float4* d = &s_stage[warp][bf][0][lane];
          cp_async16(d, rr);
          cp_async16(d + 32, rr + C);
          cp_async16(d + 64, rr + 2 * C);
        }
        if (lane < 3) cp_async4(&s_w[warp][bf][lane], wig + e * kWig + 3 + lane);
        else if (lane < 8) cp_async4(&s_w[warp][bf][lane], wig + e * kWig + 19 + (lane - 3));
        else if (lane == 8) cp_async4(&s_w[warp][bf][8], env + e);
        cp_async_commit();
      };
      int ib = kb;
      int e_l = (kb + lane < ke) ? col_idx[kb + lane] : 0;
      int ki = kb;
      auto issue_next = [&]() {
        if (ki < ke) {
          if (ki - ib >= 32) {
            ib += 32;
            e_l = (ib + lane < ke) ? col_idx[ib + lane] : 0;
          }
          issue(__shfl_sync(kFull, e_l, ki - ib), (ki - kb) % kRing);
        } else {
          cp_async_commit();
        }
        ++ki;
      };
#pragma unroll 1
      for (int p = 0; p < kRing - 1; ++p) issue_next();
      d4 acc[9];
      if (act) {
        acc[0] = d4_of(ld4_keep(W_sphere + z * C + co) + ld4_keep(csd + b * C + co));
#pragma unroll
        for (int l = 1; l < 9; ++l) acc[l] = d4{0.0, 0.0, 0.0, 0.0};
      }
#pragma unroll 1
      for (int k = kb; k < ke; ++k) {
        issue_next();
        cp_async_wait<kRing - 1>();
        __syncwarp();
        const int bf = (k - kb) % kRing;
        const float* sw = s_w[warp][bf];
        if (act) {
          const float ev = sw[8];
          const float4* src = &s_stage[warp][bf][0][lane];
          const float4 r0 = src[0], r1 = src[32], r2 = src[64];
          acc[0] += div4(r0 * ev, 5.f);
#pragma unroll
          for (int kk = 0; kk < 3; ++kk) acc[1 + kk] += div4((r1 * sw[kk]) * ev, 5.f);
#pragma unroll
          for (int kk = 0; kk < 5; ++kk) acc[4 + kk] += div4((r2 * sw[3 + kk]) * ev, 5.f);
        }
        __syncwarp();   // buffer bf is refilled by the next iteration's copies
      }
      cp_async_wait<0>();
      if (act) {
        float* xo = x_out + jn * 9 * (int64_t)C + co;
#pragma unroll
        for (int l = 0; l < 9; ++l) st4(xo + l * C, f4_of(acc[l]));
      }
    }
  }
}

// Backward of the initial embedding scatter, warp per destination atom over its CSR edges:
//   g_rad = env * [g0, D1 row 1 . g1, D2 row 2 . g2] / 5, and per edge the Wigner entries of
//   D1 row 1 / D2 row 2 and the envelope gradient (channel sums).
// The atom's gradient rows (divided by 5) stay in registers across its edges; each edge's
// radial row, Wigner entries and envelope are copied into a per-warp cp.async ring kRing - 1
// edges ahead; the nine channel sums of an edge use the transpose reduction.
template <int WARPS>
__global__ void __launch_bounds__(WARPS * 32) init_scatter_bwd_kernel(
    const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col_idx, const float* __restrict__ g_out,
    const float* __restrict__ rad, const float* __restrict__ wig, const float* __restrict__ env,
    float* __restrict__ g_rad, float* __restrict__ g_wig, float* __restrict__ g_env, int64_t N, int C, int split,
    int* err) {
  __shared__ float4 s_stage[WARPS][kRing][3][32];   // radial slots 0-2 of the staged edges
  __shared__ float s_w[WARPS][kRing][12];          // D1 row 1 (0-2), D2 row 2 (3-7), envelope (8)
  float amax = 0.f;   // largest magnitude written as a split (range check at the end)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C4 = C >> 2;
  const Share sh = warp_share(N, (int64_t)blockIdx.x * WARPS + warp, (int64_t)gridDim.x * WARPS);
  for (int64_t jn = sh.begin; jn < sh.end; ++jn) {
    const int kb = row_ptr[jn], ke = row_ptr[jn + 1];
    for (int cb = 0; cb < C4; cb += 32) {
      const int c4 = cb + lane;
      const bool on = c4 < C4;
      const int co = c4 * 4;
      auto issue = [&](int64_t e, int b) {
        if (on) {
          const float* rr = rad + e * 3 * (int64_t)C + co;
          float4* d = &s_stage[warp][b][0][lane];
          cp_async16(d, rr);
          cp_async16(d + 32, rr + C);
          cp_async16(d + 64, rr + 2 * C);
        }
        if (lane < 3) cp_async4(&s_w[warp][b][lane], wig + e * kWig + 3 + lane);
        else if (lane < 8) cp_async4(&s_w[warp][b][lane], wig + e * kWig + 19 + (lane - 3));
        else if (lane == 8) cp_async4(&s_w[warp][b][8], env + e);
        cp_async_commit();
      };
      int ib = kb;
      int e_l = (kb + lane < ke) ? col_idx[kb + lane] : 0;
      int ki = kb;
      auto issue_next = [&]() {
        if (ki < ke) {
          if (ki - ib >= 32) {
            ib += 32;
            e_l = (ib + lane < ke) ? col_idx[ib + lane] : 0;
          }
          issue(__shfl_sync(kFull, e_l, ki - ib), (ki - kb) % kRing);
        } else {
          cp_async_commit();
        }
        ++ki;
      };
#pragma unroll 1
      for (int p = 0; p < kRing - 1; ++p) issue_next();
      // this atom's gradient rows / 5, kept for all its edges
      float4 g[9];
#pragma unroll
      for (int l = 0; l < 9; ++l) g[l] = on ? div4(ld4_keep(g_out + (jn * 9 + l) * (int64_t)C + co), 5.f) : f4(0.f);
      int base_c = kb, e_lc = e_l;   // edge ids for the sum side (its own 32-wide window)
#pragma unroll 1
      for (int k = kb; k < ke; ++k) {
        issue_next();
        cp_async_wait<kRing - 1>();
        __syncwarp();
        if (k - base_c >= 32) {
          base_c += 32;
          e_lc = (base_c + lane < ke) ? col_idx[base_c + lane] : 0;
        }
        const int64_t e = __shfl_sync(kFull, e_lc, k - base_c);
        const int b = (k - kb) % kRing;
        const float* sw = s_w[warp][b];
        const float ev = sw[8];
        const float4* src = &s_stage[warp][b][0][lane];
        const float4 r0 = on ? src[0] : f4(0.f), r1 = on ? src[32] : f4(0.f), r2 = on ? src[64] : f4(0.f);
        float4 s1 = g[1] * sw[0];
        fma4(s1, sw[1], g[2]);
        fma4(s1, sw[2], g[3]);
        float4 s2 = g[4] * sw[3];
#pragma unroll
        for (int kk = 1; kk < 5; ++kk) fma4(s2, sw[3 + kk], g[4 + kk]);
        if (on) {
          float* gr = g_rad + e * 3 * (int64_t)C;
          st_out4(gr, 3 * C, co, g[0] * ev, split, amax);
          st_out4(gr, 3 * C, C + co, s1 * ev, split, amax);
          st_out4(gr, 3 * C, 2 * C + co, s2 * ev, split, amax);
        }
        float part[16];
#pragma unroll
        for (int kk = 0; kk < 3; ++kk) part[kk] = dot4(g[1 + kk], r1);
#pragma unroll
        for (int kk = 0; kk < 5; ++kk) part[3 + kk] = dot4(g[4 + kk], r2);
        part[8] = dot4(g[0], r0) + dot4(s1, r1) + dot4(s2, r2);
#pragma unroll
        for (int m = 9; m < 16; ++m) part[m] = 0.f;
        const float tot = warp_transpose_sum<16>(part, lane);   // lane m < 9: channel sum of partial m
        // full 34-wide row: D1 row 1 -> entries 3..5, D2 row 2 -> entries 19..23, zeros elsewhere
        const float t3 = __shfl_sync(kFull, tot, (lane - 3) & 31), t19 = __shfl_sync(kFull, tot, (lane - 16) & 31);
        float v = 0.f;
        if (lane >= 3 && lane < 6) v = t3 * ev;
        if (lane >= 19 && lane < 24) v = t19 * ev;
        float* gw = g_wig + e * kWig;
        gw[lane] = cb == 0 ? v : gw[lane] + v;
        if (lane < 2) gw[32 + lane] = 0.f;
        const float t8 = __shfl_sync(kFull, tot, 8);
        if (lane == 0) g_env[e] = cb == 0 ? t8 : g_env[e] + t8;
        __syncwarp();   // buffer b is refilled by the next iteration's copies
      }
      cp_async_wait<0>();
    }
  }
  report_split_range(amax, err);
}

template <bool kH>
void rs_fwd_launch(const int32_t* row_ptr, const int32_t* col_idx, const float* Z0, const float* Z1, const float* Z2,
                   const float* wig, const float* env, const float* x_res, float* x_out, int64_t N, int C,
                   cudaStream_t s) {
  const int t = kFwdWarps * 32;
  rotate_scatter_fwd_kernel<0, kH><<<grid_resident(rotate_scatter_fwd_kernel<0, kH>, t, N, kFwdWarps), t, 0, s>>>(
      row_ptr, col_idx, Z0, Z1, Z2, wig, env, x_res, x_out, N, C);
  rotate_scatter_fwd_kernel<1, kH><<<grid_resident(rotate_scatter_fwd_kernel<1, kH>, t, N, kFwdWarps), t, 0, s>>>(
      row_ptr, col_idx, Z0, Z1, Z2, wig, env, x_res, x_out, N, C);
}

void launch_rotate_scatter_fwd(const int32_t* row_ptr, const int32_t* col_idx, const float* Z0, const float* Z1,
                               const float* Z2, const float* wig, const float* env, const float* x_res, float* x_out,
                               int64_t N, int C, cudaStream_t s, bool act_half) {
  if (act_half)
    rs_fwd_launch<true>(row_ptr, col_idx, Z0, Z1, Z2, wig, env, x_res, x_out, N, C, s);
  else
    rs_fwd_launch<false>(row_ptr, col_idx, Z0, Z1, Z2, wig, env, x_res, x_out, N, C, s);
}

void launch_rotate_scatter_bwd(const int32_t* row_ptr, const int32_t* col_idx, const float* g_out, const float* Z0,
                               const float* Z1, const float* Z2, const float* wig, const float* env, float* gZ0,
                               float* gZ1, float* gZ2, float* g_wig, float* g_env, int64_t N, int C, int split,
                               int* err, cudaStream_t s, bool act_half) {
  const unsigned g = grid_for(N, 8, 2);
  if (act_half) {
    rotate_scatter_bwd_kernel<0, true><<<g, 256, 0, s>>>(row_ptr, col_idx, g_out, Z0, Z1, Z2, wig, env, gZ0, gZ1, gZ2,
                                                         g_wig, g_env, N, C, split, err);
    rotate_scatter_bwd_kernel<1, true><<<g, 256, 0, s>>>(row_ptr, col_idx, g_out, Z0, Z1, Z2, wig, env, gZ0, gZ1, gZ2,
                                                         g_wig, g_env, N, C, split, err);
  } else {
    rotate_scatter_bwd_kernel<0, false><<<g, 256, 0, s>>>(row_ptr, col_idx, g_out, Z0, Z1, Z2, wig, env, gZ0, gZ1,
                                                          gZ2, g_wig, g_env, N, C, split, err);
    rotate_scatter_bwd_kernel<1, false><<<g, 256, 0, s>>>(row_ptr, col_idx, g_out, Z0, Z1, Z2, wig, env, gZ0, gZ1,
                                                          gZ2, g_wig, g_env, N, C, split, err);
  }
}

void launch_init_scatter_fwd(const int32_t* row_ptr, const int32_t* col_idx, const float* rad, const float* wig,
                             const float* env, const int64_t* Z, const int64_t* batch, const float* W_sphere,
                             const float* csd, float* x_out, int64_t N, int C, cudaStream_t s) {
  init_scatter_fwd_kernel<4><<<grid_resident(init_scatter_fwd_kernel<4>, 128, N, 4), 128, 0, s>>>(row_ptr, col_idx, rad, wig, env, Z, batch, W_sphere,
                                                               csd, x_out, N, C);
}

void launch_init_scatter_bwd(const int32_t* row_ptr, const int32_t* col_idx, const float* g_out, const float* rad,
                             const float* wig, const float* env, float* g_rad, float* g_wig, float* g_env, int64_t N,
                             int C, int split, int* err, cudaStream_t s) {
  init_scatter_bwd_kernel<4><<<grid_resident(init_scatter_bwd_kernel<4>, 128, N, 4), 128, 0, s>>>(row_ptr, col_idx, g_out, rad, wig, env, g_rad, g_wig,
                                                                 g_env, N, C, split, err);
}

}  // namespace fuma
