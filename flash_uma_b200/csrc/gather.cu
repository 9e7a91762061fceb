// Gather of source/target node embeddings, rotation into the edge frame and radial
// modulation, split into the three SO(2) m-blocks (forward), and its adjoint.
//
// Reference: ops/gather.py:34-154 (forward), :160-405 (backward, fp32 atomics).
//
// Layouts (fp32, C channels per slot, c fastest):
//   x [N, 9, C]; rad [E, 12C]; wigner [E, 34]; csd [nsys, C]; batch [N] int64
//   X_m0 [E, 6C] = [v_i0 r0, v_j0 r1, (D1v_i)_1 r2, (D1v_j)_1 r3, (D2v_i)_2 r4, (D2v_j)_2 r5]
//   X_m1 [E, 8C] = [(D1v_i)_2 r6, (D1v_j)_2 r7, (D2v_i)_3 r8, (D2v_j)_3 r9,
//                   (D1v_i)_0 r6, (D1v_j)_0 r7, (D2v_i)_1 r8, (D2v_j)_1 r9]
//   X_m2 [E, 4C] = [(D2v_i)_4 r10, (D2v_j)_4 r11, (D2v_i)_0 r10, (D2v_j)_0 r11]
// where v_i0 / v_j0 include csd[batch[node]] (the system embedding).
// The source side s=0 of an edge uses the even radial slots, the target side s=1 the odd ones.
//
// Work decomposition: one warp per edge (forward) or per destination node
// (backward); lane l owns channels [4l, 4l+4) (+128 per extra iteration), so every
// global access is a coalesced 16-byte vector access. Each side / degree block is
// processed on its own to keep the live register set small (these kernels are
// bandwidth-bound and need occupancy, not ILP from a 200-register body).
//
// Backward without atomics, in two passes over the edges, one per side of every edge. The
// target pass walks the destination CSR (warp per node j, edges in CSR order): the target
// side of each edge gives the odd radial-slot gradients, its share of the Wigner gradient
// and a contribution to the gradient of x[j], summed in registers and written at the end of
// the segment. The source pass walks the source CSR (warp per node i) and does the same for
// the source side, adding to what the target pass wrote (g_x, g_wigner). Fixed orders
// everywhere, so g_x and g_wigner are run-to-run deterministic; each pass reads only its
// half of every edge's gradient and radial rows. Each pass runs in two launches, l <= 1 and
// l = 2 coefficient blocks, to keep the live register set small.
#include "common.cuh"
#include "kernels.h"

namespace fuma {

namespace {

// out[r] = sum_k D[r*n + k] v[k]
template <int n>
__device__ __forceinline__ void rot(const float* D, const float4* v, float4* out) {
#pragma unroll
  for (int r = 0; r < n; ++r) {
    float4 a = D[r * n] * v[0];
#pragma unroll
    for (int k = 1; k < n; ++k) fma4(a, D[r * n + k], v[k]);
    out[r] = a;
  }
}

// sum_k D[r*n + k] v[k] (row r of rot<n>, same operation order)
template <int n>
__device__ __forceinline__ float4 rot_row(const float* D, int r, const float4* v) {
  float4 a = D[r * n] * v[0];
#pragma unroll
  for (int k = 1; k < n; ++k) fma4(a, D[r * n + k], v[k]);
  return a;
}

// out[k] = sum_r D[r*n + k] g[r]
template <int n>
__device__ __forceinline__ void rotT(const float* D, const float4* g, float4* out) {
#pragma unroll
  for (int k = 0; k < n; ++k) {
    float4 a = D[k] * g[0];
#pragma unroll
    for (int r = 1; r < n; ++r) fma4(a, D[r * n + k], g[r]);
    out[k] = a;
  }
}

constexpr int kFwdWarps = 8;
constexpr int kBwdWarps = 8;

}  // namespace

// Warp per edge, one launch per coefficient block: PART 0 writes the l <= 1 slots (radial slots
// 0-3, 6-7; node rows 0-3; D1), PART 1 the l = 2 slots (radial slots 4-5, 8-11; node rows 4-8;
// D2). The two read disjoint parts of every radial and node row, so splitting costs only the
// second read of the indices and Wigner rows, and lowers the live registers of a launch: at 64
// registers (4 blocks of 8 warps per SM) the pair measured 350 us against 375 us for one
// 80-register kernel at 3 blocks (E = 120,000, B200). With the chunked loop below both parts
// still run at 64 registers (4 blocks per SM), PART 1 with a few spilled registers: at 80
// registers (3 blocks) the pair measured 10% slower at E = 120,000; an L2 evict-last hint on the
// node-row loads measured 3% slower, and is not used.
// A warp takes chunks of 32 consecutive edges: the lanes load the chunk's edge indices (and, for
// PART 0, the atoms' system ids) in one coalesced step and the chunk's Wigner blocks into shared
// memory, so each edge then waits only for its own node and radial rows, not for a chain of
// index -> system id -> row loads.
template <int PART, bool kH>
__global__ void __launch_bounds__(kFwdWarps * 32, 4) gather_fwd_kernel(
    const float* __restrict__ x, const int64_t* __restrict__ idx_i, const int64_t* __restrict__ idx_j,
    const float* __restrict__ wig, const float* __restrict__ rad, const float* __restrict__ csd,
    const int64_t* __restrict__ batch, float* __restrict__ X0, float* __restrict__ X1, float* __restrict__ X2,
    int64_t E, int C, int split, int* err) {
  constexpr int nw = PART ? 25 : 9;     // Wigner values of this block per edge
  constexpr int woff = PART ? 9 : 0;
  __shared__ float s_w[kFwdWarps][32 * nw];
  float amax = 0.f;   // largest magnitude written as a split (range check at the end)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C4 = C >> 2;
  float* swc = s_w[warp];
  const int64_t nchunks = (E + 31) >> 5;
  for (int64_t ch = (int64_t)blockIdx.x * kFwdWarps + warp; ch < nchunks; ch += (int64_t)gridDim.x * kFwdWarps) {
    const int64_t e0 = ch << 5;
    const int ne = (int)min((int64_t)32, E - e0);
    int li = 0, lj = 0, lbi = 0, lbj = 0;   // this lane's edge of the chunk: atoms (and systems)
    if (lane < ne) {
      li = (int)idx_i[e0 + lane];
      lj = (int)idx_j[e0 + lane];
      if (PART == 0) {
        lbi = (int)batch[li];
        lbj = (int)batch[lj];
      }
    }
    for (int t = lane; t < ne * nw; t += 32) {
      const int r = t / nw;
      swc[t] = __ldg(wig + (e0 + r) * kWig + woff + (t - r * nw));
    }
    __syncwarp();
#pragma unroll 1
    for (int k = 0; k < ne; ++k) {
      const int64_t e = e0 + k;
      const int64_t ni = __shfl_sync(kFull, li, k), nj = __shfl_sync(kFull, lj, k);
      int64_t bi = 0, bj = 0;
      if (PART == 0) {
        bi = __shfl_sync(kFull, lbi, k);
        bj = __shfl_sync(kFull, lbj, k);
      }
      const float* sw = swc + k * nw;
      for (int c4 = lane; c4 < C4; c4 += 32) {
        const int co = c4 * 4;
        const int64_t rr = e * 12 * (int64_t)C + co;   // element offset of the radial row (fp32 or fp16 rad)
        float* x0 = X0 + e * 6 * (int64_t)C;   // output rows; columns are co + slot * C
        float* x1 = X1 + e * 8 * (int64_t)C;
        float* x2 = X2 + e * 4 * (int64_t)C;
#pragma unroll 1
        for (int s = 0; s < 2; ++s) {
          const int64_t node = s ? nj : ni;
          const float* xr = x + node * 9 * (int64_t)C + co;
          if constexpr (PART == 0) {
            const int64_t bsys = s ? bj : bi;
            const float4 c0 = ld4_keep(xr), cs = ld4_keep(csd + bsys * C + co), r0 = ld4_act<kH>(rad, rr + s * C);
            float4 v[3];
#pragma unroll
            for (int m = 0; m < 3; ++m) v[m] = ld4_keep(xr + (1 + m) * C);
            const float4 r2 = ld4_act<kH>(rad, rr + (2 + s) * C), r6 = ld4_act<kH>(rad, rr + (6 + s) * C);
            st_out4(x0, 6 * C, s * C + co, (c0 + cs) * r0, split, amax);
            st_out4(x1, 8 * C, (4 + s) * C + co, rot_row<3>(sw, 0, v) * r6, split, amax);
            st_out4(x0, 6 * C, (2 + s) * C + co, rot_row<3>(sw, 1, v) * r2, split, amax);
            st_out4(x1, 8 * C, (0 + s) * C + co, rot_row<3>(sw, 2, v) * r6, split, amax);
          } else {
            float4 v[5];
#pragma unroll
            for (int m = 0; m < 5; ++m) v[m] = ld4_keep(xr + (4 + m) * C);
            const float4 r4 = ld4_act<kH>(rad, rr + (4 + s) * C), r8 = ld4_act<kH>(rad, rr + (8 + s) * C),
                         r10 = ld4_act<kH>(rad, rr + (10 + s) * C);
            st_out4(x2, 4 * C, (2 + s) * C + co, rot_row<5>(sw, 0, v) * r10, split, amax);
            st_out4(x1, 8 * C, (6 + s) * C + co, rot_row<5>(sw, 1, v) * r8, split, amax);
            st_out4(x0, 6 * C, (4 + s) * C + co, rot_row<5>(sw, 2, v) * r4, split, amax);
            st_out4(x1, 8 * C, (2 + s) * C + co, rot_row<5>(sw, 3, v) * r8, split, amax);
            st_out4(x2, 4 * C, (0 + s) * C + co, rot_row<5>(sw, 4, v) * r10, split, amax);
          }
        }
      }
    }
    __syncwarp();   // the chunk's Wigner blocks are replaced by the next chunk's
  }
  report_split_range(amax, err);
}

template <int PART>
struct BwdSlots {
  static constexpr int n = PART ? 8 : 7;   // 16-byte loads per lane and edge: gX and rad slots of one side
};

// One side (SIDE 1: target pass over the destination CSR, SIDE 0: source pass over the source
// CSR) and one coefficient block (PART 0: rows 0-3, radial slots 0-3 and 6-7, D1; PART 1:
// rows 4-8, radial slots 4-5 and 8-11, D2) of the gather backward. Warp per node n, lane =
// 4 channels (channel chunks of 128 in an outer loop); the node's rows stay in registers
// and are rotated into every edge's frame. The next edge's gradient and radial slots and
// Wigner block are copied into shared memory (cp.async, double-buffered per warp) while the
// current edge is computed, so two edges' loads are in flight per warp.
// Dynamic shared memory: kBwdWarps * 2 * BwdSlots<PART>::n * 512 bytes.
template <int SIDE, int PART, bool kH>
__global__ void __launch_bounds__(kBwdWarps * 32, 2) gather_bwd_side_kernel(
    const float* __restrict__ gX0, const float* __restrict__ gX1, const float* __restrict__ gX2,
    const float* __restrict__ x, const float* __restrict__ wig, const float* __restrict__ rad,
    const float* __restrict__ csd, const int64_t* __restrict__ batch, const int32_t* __restrict__ row_ptr,
    const int32_t* __restrict__ col_idx, float* __restrict__ g_x, float* __restrict__ g_wig,
    float* __restrict__ g_rad, int64_t N, int C, int split, int* err) {
  constexpr int s = SIDE;
  constexpr int nrows = PART ? 5 : 4;
  constexpr int nw = PART ? 25 : 9;
  constexpr int woff = PART ? 9 : 0;
  constexpr int row0 = PART ? 4 : 0;
  constexpr int NV = PART ? 32 : 16;
  constexpr int kS = BwdSlots<PART>::n;
  extern __shared__ float4 s_stage[];
  __shared__ float s_w[kBwdWarps][2][28];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C4 = C >> 2;
  const int W = 12 * C;   // g_rad / rad row width
  float4* stage = s_stage + (size_t)warp * 2 * kS * 32;   // [buffer][slot][lane]
  float amax = 0.f;   // largest magnitude written as a split (range check at the end)
  const Share sh = warp_share(N, (int64_t)blockIdx.x * kBwdWarps + warp, (int64_t)gridDim.x * kBwdWarps);
  for (int64_t n = sh.begin; n < sh.end; ++n) {
    const int kb = row_ptr[n], ke = row_ptr[n + 1];
    const int64_t bn = batch[n];
    for (int cb = 0; cb < C4; cb += 32) {
      const int c4 = cb + lane;
      const bool on = c4 < C4;
      const int co = c4 * 4;
      // copies of edge e's slots (this side) and Wigner block into buffer b; one commit group
      auto issue = [&](int64_t e, int b) {
        float4* dst = stage + b * kS * 32 + lane;
        if (on) {
          // element offsets of the edge's gradient and radial rows (fp32, or fp16 with kH)
          const int64_t g0 = e * 6 * (int64_t)C + co, g1 = e * 8 * (int64_t)C + co, g2 = e * 4 * (int64_t)C + co;
          const int64_t rr = e * (int64_t)W + co;
          if constexpr (PART == 0) {
            cp_act<kH>(dst + 0 * 32, gX0, g0 + s * C);
            cp_act<kH>(dst + 1 * 32, gX0, g0 + (2 + s) * C);
            cp_act<kH>(dst + 2 * 32, gX1, g1 + s * C);
            cp_act<kH>(dst + 3 * 32, gX1, g1 + (4 + s) * C);
            cp_act<kH>(dst + 4 * 32, rad, rr + s * C);
            cp_act<kH>(dst + 5 * 32, rad, rr + (2 + s) * C);
            cp_act<kH>(dst + 6 * 32, rad, rr + (6 + s) * C);
          } else {
            cp_act<kH>(dst + 0 * 32, gX0, g0 + (4 + s) * C);
            cp_act<kH>(dst + 1 * 32, gX1, g1 + (2 + s) * C);
            cp_act<kH>(dst + 2 * 32, gX1, g1 + (6 + s) * C);
            cp_act<kH>(dst + 3 * 32, gX2, g2 + s * C);
            cp_act<kH>(dst + 4 * 32, gX2, g2 + (2 + s) * C);
            cp_act<kH>(dst + 5 * 32, rad, rr + (4 + s) * C);
            cp_act<kH>(dst + 6 * 32, rad, rr + (8 + s) * C);
            cp_act<kH>(dst + 7 * 32, rad, rr + (10 + s) * C);
          }
        }
        if (lane < nw) cp_async4(&s_w[warp][b][lane], wig + e * kWig + woff + lane);
        cp_async_commit();
      };
      // the node's rows of this block (l = 0 with the system embedding added)
      float4 v[nrows], acc[nrows];
#pragma unroll
      for (int r = 0; r < nrows; ++r) {
        v[r] = on ? ld4_keep(x + (n * 9 + row0 + r) * (int64_t)C + co) : f4(0.f);
        acc[r] = f4(0.f);
      }
      if (PART == 0 && on) v[0] = v[0] + ld4_keep(csd + bn * C + co);
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
          cp_async_commit();   // empty group: keeps "all but the newest group" = edge k
        }
        cp_async_wait1();
        __syncwarp();   // edge k's Wigner block, copied by lanes < nw, is visible to the warp
        const int64_t e = e_cur;
        const float4* src = stage + b * kS * 32 + lane;
        const float* sw = s_w[warp][b];
        float* grow = g_rad + e * (int64_t)W;
        float gw[NV];
#pragma unroll
        for (int m = 0; m < NV; ++m) gw[m] = 0.f;
        if constexpr (PART == 0) {
          const float4 z = f4(0.f);
          const float4 a0 = on ? sm_act<kH>(src) : z, a2 = on ? sm_act<kH>(src + 32) : z,
                       b0 = on ? sm_act<kH>(src + 64) : z, b4 = on ? sm_act<kH>(src + 96) : z;
          const float4 r0 = on ? sm_act<kH>(src + 128) : z, r2 = on ? sm_act<kH>(src + 160) : z,
                       r6 = on ? sm_act<kH>(src + 192) : z;
          const float* D1 = sw;
          float4 r1[3];
          rot<3>(D1, v + 1, r1);
          if (on) {
            st_out4(grow, W, s * C + co, a0 * v[0], split, amax);
            st_out4(grow, W, (2 + s) * C + co, a2 * r1[1], split, amax);
            st_out4(grow, W, (6 + s) * C + co, b0 * r1[2] + b4 * r1[0], split, amax);
          }
          acc[0] += a0 * r0;
          const float4 gi[3] = {b4 * r6, a2 * r2, b0 * r6};
          float4 t[3];
          rotT<3>(D1, gi, t);
#pragma unroll
          for (int m = 0; m < 3; ++m) acc[1 + m] += t[m];
#pragma unroll
          for (int r = 0; r < 3; ++r)
#pragma unroll
            for (int m = 0; m < 3; ++m) gw[r * 3 + m] = dot4(gi[r], v[1 + m]);
        } else {
          const float4 z = f4(0.f);
          const float4 a4 = on ? sm_act<kH>(src) : z, b2 = on ? sm_act<kH>(src + 32) : z,
                       b6 = on ? sm_act<kH>(src + 64) : z;
          const float4 c0 = on ? sm_act<kH>(src + 96) : z, c2 = on ? sm_act<kH>(src + 128) : z;
          const float4 r4 = on ? sm_act<kH>(src + 160) : z, r8 = on ? sm_act<kH>(src + 192) : z,
                       r10 = on ? sm_act<kH>(src + 224) : z;
          const float* D2 = sw;
          float4 rv[5];
          rot<5>(D2, v, rv);
          if (on) {
            st_out4(grow, W, (4 + s) * C + co, a4 * rv[2], split, amax);
            st_out4(grow, W, (8 + s) * C + co, b2 * rv[3] + b6 * rv[1], split, amax);
            st_out4(grow, W, (10 + s) * C + co, c0 * rv[4] + c2 * rv[0], split, amax);
          }
          const float4 g[5] = {c2 * r10, b6 * r8, a4 * r4, b2 * r8, c0 * r10};
          float4 t[5];
          rotT<5>(D2, g, t);
#pragma unroll
          for (int m = 0; m < 5; ++m) acc[m] += t[m];
#pragma unroll
          for (int r = 0; r < 5; ++r)
#pragma unroll
            for (int m = 0; m < 5; ++m) gw[r * 5 + m] = dot4(g[r], v[m]);
        }
        const float tot = warp_transpose_sum<NV>(gw, lane);
        if (lane < nw) {
          float* dst = g_wig + e * kWig + woff + lane;
          *dst = (SIDE == 1 && cb == 0) ? tot : *dst + tot;
        }
        __syncwarp();   // buffer b is refilled by the next iteration's copies
        e_cur = e_next;
      }
      if (on) {
        float* gx = g_x + (n * 9 + row0) * (int64_t)C + co;
#pragma unroll
        for (int r = 0; r < nrows; ++r) st4(gx + r * C, SIDE == 1 ? acc[r] : ld4(gx + r * C) + acc[r]);
      }
    }
  }
  report_split_range(amax, err);
}

template <bool kH>
void gather_fwd_launch(const float* x, const int64_t* idx_i, const int64_t* idx_j, const float* wig, const float* rad,
                       const float* csd, const int64_t* batch, float* X0, float* X1, float* X2, int64_t E, int C,
                       int split, int* err, cudaStream_t s) {
  const int t = kFwdWarps * 32;
  const int64_t chunks = (E + 31) / 32;   // a warp's unit of work: 32 consecutive edges
  gather_fwd_kernel<0, kH><<<grid_resident(gather_fwd_kernel<0, kH>, t, chunks, kFwdWarps), t, 0, s>>>(
      x, idx_i, idx_j, wig, rad, csd, batch, X0, X1, X2, E, C, split, err);
  gather_fwd_kernel<1, kH><<<grid_resident(gather_fwd_kernel<1, kH>, t, chunks, kFwdWarps), t, 0, s>>>(
      x, idx_i, idx_j, wig, rad, csd, batch, X0, X1, X2, E, C, split, err);
}

void launch_gather_fwd(const float* x, const int64_t* idx_i, const int64_t* idx_j, const float* wig, const float* rad,
                       const float* csd, const int64_t* batch, float* X0, float* X1, float* X2, int64_t E, int C,
                       int split, int* err, cudaStream_t s, bool act_half) {
  if (act_half)
    gather_fwd_launch<true>(x, idx_i, idx_j, wig, rad, csd, batch, X0, X1, X2, E, C, split, err, s);
  else
    gather_fwd_launch<false>(x, idx_i, idx_j, wig, rad, csd, batch, X0, X1, X2, E, C, split, err, s);
}

template <bool kH>
void gather_bwd_launch(const float* gX0, const float* gX1, const float* gX2, const float* x, const float* wig,
                       const float* rad, const float* csd, const int64_t* batch, const int32_t* dst_ptr,
                       const int32_t* dst_col, const int32_t* src_ptr, const int32_t* src_col, float* g_x,
                       float* g_wig, float* g_rad, int64_t N, int C, int split, int* err, cudaStream_t s) {
  const unsigned g = grid_for(N, kBwdWarps, 2);
  const int b = kBwdWarps * 32;
  const size_t sm0 = (size_t)kBwdWarps * 2 * BwdSlots<0>::n * 32 * sizeof(float4);
  const size_t sm1 = (size_t)kBwdWarps * 2 * BwdSlots<1>::n * 32 * sizeof(float4);
  static thread_local uint64_t configured = 0;   // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured >> (dev & 63) & 1)) {
    cudaFuncSetAttribute(gather_bwd_side_kernel<1, 0, kH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm0);
    cudaFuncSetAttribute(gather_bwd_side_kernel<1, 1, kH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm1);
    cudaFuncSetAttribute(gather_bwd_side_kernel<0, 0, kH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm0);
    cudaFuncSetAttribute(gather_bwd_side_kernel<0, 1, kH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm1);
    configured |= uint64_t(1) << (dev & 63);
  }
  // target pass (writes g_x, g_wigner), then source pass (adds to them)
  gather_bwd_side_kernel<1, 0, kH><<<g, b, sm0, s>>>(gX0, gX1, gX2, x, wig, rad, csd, batch, dst_ptr, dst_col, g_x,
                                                     g_wig, g_rad, N, C, split, err);
  gather_bwd_side_kernel<1, 1, kH><<<g, b, sm1, s>>>(gX0, gX1, gX2, x, wig, rad, csd, batch, dst_ptr, dst_col, g_x,
                                                     g_wig, g_rad, N, C, split, err);
  gather_bwd_side_kernel<0, 0, kH><<<g, b, sm0, s>>>(gX0, gX1, gX2, x, wig, rad, csd, batch, src_ptr, src_col, g_x,
                                                     g_wig, g_rad, N, C, split, err);
  gather_bwd_side_kernel<0, 1, kH><<<g, b, sm1, s>>>(gX0, gX1, gX2, x, wig, rad, csd, batch, src_ptr, src_col, g_x,
                                                     g_wig, g_rad, N, C, split, err);
}

void launch_gather_bwd(const float* gX0, const float* gX1, const float* gX2, const float* x, const int64_t* idx_i,
                       const float* wig, const float* rad, const float* csd, const int64_t* batch,
                       const int32_t* dst_ptr, const int32_t* dst_col, const int32_t* src_ptr, const int32_t* src_col,
                       float* g_x, float* g_wig, float* g_rad, float* scratch, int64_t N, int C, int split, int* err,
                       cudaStream_t s, bool act_half) {
  (void)idx_i;
  (void)scratch;   // the two-pass backward needs no scratch rows
  if (act_half)
    gather_bwd_launch<true>(gX0, gX1, gX2, x, wig, rad, csd, batch, dst_ptr, dst_col, src_ptr, src_col, g_x, g_wig,
                            g_rad, N, C, split, err, s);
  else
    gather_bwd_launch<false>(gX0, gX1, gX2, x, wig, rad, csd, batch, dst_ptr, dst_col, src_ptr, src_col, g_x, g_wig,
                             g_rad, N, C, split, err, s);
}

}  // namespace fuma
