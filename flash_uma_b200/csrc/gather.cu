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
// Backward without atomics: pass A walks the destination CSR, two warps per
// destination node j (l <= 1 and l = 2 coefficient blocks); it writes g_rad[e] and
// g_wigner[e], accumulates the target-side gradient of x[j] in shared memory and writes
// the source-side contribution of every edge to a scratch row [9C]. Pass B walks the
// source CSR and adds those rows to g_x[i] in a fixed order: run-to-run deterministic g_x.
#include "common.cuh"
#include "kernels.h"

namespace fuma {

namespace {

// Load the 34 Wigner values of edge e into smem.
__device__ __forceinline__ void stage_wigner(float* sw, const float* __restrict__ wig, int64_t e, int lane) {
  sw[lane] = __ldg(wig + e * kWig + lane);
  if (lane < 2) sw[32 + lane] = __ldg(wig + e * kWig + 32 + lane);
}

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

__global__ void __launch_bounds__(kFwdWarps * 32, 3) gather_fwd_kernel(
    const float* __restrict__ x, const int64_t* __restrict__ idx_i, const int64_t* __restrict__ idx_j,
    const float* __restrict__ wig, const float* __restrict__ rad, const float* __restrict__ csd,
    const int64_t* __restrict__ batch, float* __restrict__ X0, float* __restrict__ X1, float* __restrict__ X2,
    int64_t E, int C, bool split, int* err) {
  __shared__ float s_w[kFwdWarps][36];
  bool bad = false;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C4 = C >> 2;
  float* sw = s_w[warp];
  const float* D1 = sw;
  const float* D2 = sw + 9;
  for (int64_t e = (int64_t)blockIdx.x * kFwdWarps + warp; e < E; e += (int64_t)gridDim.x * kFwdWarps) {
    stage_wigner(sw, wig, e, lane);
    const int64_t ni = idx_i[e], nj = idx_j[e];
    const int64_t bi = batch[ni], bj = batch[nj];
    __syncwarp();
    for (int c4 = lane; c4 < C4; c4 += 32) {
      const int co = c4 * 4;
      const float* rr = rad + e * 12 * (int64_t)C + co;
      float* x0 = X0 + e * 6 * (int64_t)C;   // output rows; columns are co + slot * C
      float* x1 = X1 + e * 8 * (int64_t)C;
      float* x2 = X2 + e * 4 * (int64_t)C;
#pragma unroll 1
      for (int s = 0; s < 2; ++s) {
        const int64_t node = s ? nj : ni;
        const int64_t bsys = s ? bj : bi;
        const float* xr = x + node * 9 * (int64_t)C + co;
        // l = 0
        st_out4(x0, 6 * C, s * C + co, (ld4_keep(xr) + ld4_keep(csd + bsys * C + co)) * ld4_stream(rr + s * C), split,
                bad);
        // l = 1
        {
          float4 v[3], r1[3];
#pragma unroll
          for (int m = 0; m < 3; ++m) v[m] = ld4_keep(xr + (1 + m) * C);
          rot<3>(D1, v, r1);
          const float4 r6 = ld4_stream(rr + (6 + s) * C);
          st_out4(x0, 6 * C, (2 + s) * C + co, r1[1] * ld4_stream(rr + (2 + s) * C), split, bad);
          st_out4(x1, 8 * C, (0 + s) * C + co, r1[2] * r6, split, bad);
          st_out4(x1, 8 * C, (4 + s) * C + co, r1[0] * r6, split, bad);
        }
        // l = 2
        {
          float4 v[5], r2[5];
#pragma unroll
          for (int m = 0; m < 5; ++m) v[m] = ld4_keep(xr + (4 + m) * C);
          rot<5>(D2, v, r2);
          const float4 r8 = ld4_stream(rr + (8 + s) * C), r10 = ld4_stream(rr + (10 + s) * C);
          st_out4(x0, 6 * C, (4 + s) * C + co, r2[2] * ld4_stream(rr + (4 + s) * C), split, bad);
          st_out4(x1, 8 * C, (2 + s) * C + co, r2[3] * r8, split, bad);
          st_out4(x1, 8 * C, (6 + s) * C + co, r2[1] * r8, split, bad);
          st_out4(x2, 4 * C, (0 + s) * C + co, r2[4] * r10, split, bad);
          st_out4(x2, 4 * C, (2 + s) * C + co, r2[0] * r10, split, bad);
        }
      }
    }
    __syncwarp();
  }
  report_split_range(bad, err);
}

// Pass A of the backward (see file comment), one launch per coefficient block: PART 0 handles
// the l <= 1 coefficients (rows 0-3, radial slots 0-3 and 6-7, Wigner D1), PART 1 the l = 2
// coefficients (rows 4-8, radial slots 4-5 and 8-11, Wigner D2). Their outputs are disjoint.
// The destination's CSR chunk (edge id, source atom, source system) is loaded once into the
// lanes and broadcast with shuffles, so an edge iteration issues only independent loads.
// Dynamic shared memory: kBwdWarps * 5 * C floats (target-side accumulator of this warp's rows).
template <int PART>
__global__ void __launch_bounds__(kBwdWarps * 32, 2) gather_bwd_dst_kernel(
    const float* __restrict__ gX0, const float* __restrict__ gX1, const float* __restrict__ gX2,
    const float* __restrict__ x, const int64_t* __restrict__ idx_i, const float* __restrict__ wig,
    const float* __restrict__ rad, const float* __restrict__ csd, const int64_t* __restrict__ batch,
    const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col_idx, float* __restrict__ g_x,
    float* __restrict__ g_wig, float* __restrict__ g_rad, float* __restrict__ g_src_rows, int64_t N, int C,
    bool split, int* err) {
  extern __shared__ float4 s_acc4[];
  bool bad = false;
  __shared__ float s_w[kBwdWarps][28];
  __shared__ float s_red[kBwdWarps][28];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C4 = C >> 2;
  float* sw = s_w[warp];
  float4* acc = s_acc4 + (size_t)warp * 5 * C4;
  constexpr int part = PART;
  for (int64_t jn = (int64_t)blockIdx.x * kBwdWarps + warp; jn < N; jn += (int64_t)gridDim.x * kBwdWarps) {
    constexpr int nrows = part ? 5 : 4;       // target-side accumulator rows (l=0..1 -> 4, l=2 -> 5)
    constexpr int nw = part ? 25 : 9;         // Wigner entries of this part
    constexpr int woff = part ? 9 : 0;
    for (int t = lane; t < nrows * C4; t += 32) acc[t] = f4(0.f);
    const int kb = row_ptr[jn], ke = row_ptr[jn + 1];
    const int64_t bj = batch[jn];
    const float* xj_base = x + jn * 9 * (int64_t)C;
    for (int k0 = kb; k0 < ke; k0 += 32) {
      // CSR chunk prefetch: lane l holds edge k0+l, its source atom and the source's system
      int64_t e_l = 0, in_l = 0, bi_l = 0;
      if (k0 + lane < ke) {
        e_l = col_idx[k0 + lane];
        in_l = idx_i[e_l];
        bi_l = batch[in_l];
      }
      const int cnt = (ke - k0) < 32 ? (ke - k0) : 32;
      for (int q = 0; q < cnt; ++q) {
        const int64_t e = __shfl_sync(kFull, e_l, q);
        const int64_t in = __shfl_sync(kFull, in_l, q);
        const int64_t bi = __shfl_sync(kFull, bi_l, q);
        if (lane < nw) sw[lane] = __ldg(wig + e * kWig + woff + lane);
        __syncwarp();
        const float* xi_base = x + in * 9 * (int64_t)C;
        const float* g0b = gX0 + e * 6 * (int64_t)C;
        const float* g1b = gX1 + e * 8 * (int64_t)C;
        const float* g2b = gX2 + e * 4 * (int64_t)C;
        const float* rrb = rad + e * 12 * (int64_t)C;
        float* grb = g_rad + e * 12 * (int64_t)C;   // g_rad row (12C wide), columns slot * C + co
        float* gsb = g_src_rows + e * 9 * (int64_t)C;
        float gw[nw];
#pragma unroll
        for (int m = 0; m < nw; ++m) gw[m] = 0.f;
        if constexpr (part == 0) {
          const float* D1 = sw;
          for (int c4 = lane; c4 < C4; c4 += 32) {
            const int co = c4 * 4;
            const float* rr = rrb + co; const float* g0 = g0b + co; const float* g1 = g1b + co;
            const float* xi = xi_base + co; const float* xj = xj_base + co;
            float* gsrc = gsb + co;
            const int W = 12 * C;
            {
              const float4 a0 = ld4_stream(g0), a1 = ld4_stream(g0 + C);
              st_out4(grb, W, co, a0 * (ld4_keep(xi) + ld4_keep(csd + bi * C + co)), split, bad);
              st_out4(grb, W, C + co, a1 * (ld4_keep(xj) + ld4_keep(csd + bj * C + co)), split, bad);
              st4(gsrc, a0 * ld4_stream(rr));
              acc[c4] += a1 * ld4_stream(rr + C);
            }
            float4 vi[3], vj[3], ri[3], rj[3];
#pragma unroll
            for (int m = 0; m < 3; ++m) { vi[m] = ld4_keep(xi + (1 + m) * C); vj[m] = ld4_keep(xj + (1 + m) * C); }
            rot<3>(D1, vi, ri);
            rot<3>(D1, vj, rj);
            const float4 r2 = ld4_stream(rr + 2 * C), r3 = ld4_stream(rr + 3 * C);
            const float4 r6 = ld4_stream(rr + 6 * C), r7 = ld4_stream(rr + 7 * C);
            const float4 a2 = ld4_stream(g0 + 2 * C), a3 = ld4_stream(g0 + 3 * C);
            const float4 b0 = ld4_stream(g1), b1 = ld4_stream(g1 + C);
            const float4 b4 = ld4_stream(g1 + 4 * C), b5 = ld4_stream(g1 + 5 * C);
            st_out4(grb, W, 2 * C + co, a2 * ri[1], split, bad);
            st_out4(grb, W, 3 * C + co, a3 * rj[1], split, bad);
            st_out4(grb, W, 6 * C + co, b0 * ri[2] + b4 * ri[0], split, bad);
            st_out4(grb, W, 7 * C + co, b1 * rj[2] + b5 * rj[0], split, bad);
            const float4 gi[3] = {b4 * r6, a2 * r2, b0 * r6};
            const float4 gj[3] = {b5 * r7, a3 * r3, b1 * r7};
            float4 t[3];
            rotT<3>(D1, gi, t);
#pragma unroll
            for (int m = 0; m < 3; ++m) st4(gsrc + (1 + m) * C, t[m]);
            rotT<3>(D1, gj, t);
#pragma unroll
            for (int m = 0; m < 3; ++m) acc[(1 + m) * C4 + c4] += t[m];
#pragma unroll
            for (int r = 0; r < 3; ++r)
#pragma unroll
              for (int m = 0; m < 3; ++m) gw[r * 3 + m] += dot4(gi[r], vi[m]) + dot4(gj[r], vj[m]);
          }
        } else {
          const float* D2 = sw;
          for (int c4 = lane; c4 < C4; c4 += 32) {
            const int co = c4 * 4;
            const float* rr = rrb + co; const float* g0 = g0b + co; const float* g1 = g1b + co;
            const float* g2 = g2b + co;
            const float* xi = xi_base + co; const float* xj = xj_base + co;
            float* gsrc = gsb + co;
            const int W = 12 * C;
#pragma unroll 1
            for (int s = 0; s < 2; ++s) {   // s = 0: source side (even slots), s = 1: target side (odd slots)
              const float* xs = s ? xj : xi;
              float4 v[5], r[5];
#pragma unroll
              for (int m = 0; m < 5; ++m) v[m] = ld4_keep(xs + (4 + m) * C);
              rot<5>(D2, v, r);
              const float4 a4 = ld4_stream(g0 + (4 + s) * C);
              const float4 b2 = ld4_stream(g1 + (2 + s) * C), b6 = ld4_stream(g1 + (6 + s) * C);
              const float4 c0 = ld4_stream(g2 + s * C), c2 = ld4_stream(g2 + (2 + s) * C);
              const float4 r4 = ld4_stream(rr + (4 + s) * C), r8 = ld4_stream(rr + (8 + s) * C);
              const float4 r10 = ld4_stream(rr + (10 + s) * C);
              st_out4(grb, W, (4 + s) * C + co, a4 * r[2], split, bad);
              st_out4(grb, W, (8 + s) * C + co, b2 * r[3] + b6 * r[1], split, bad);
              st_out4(grb, W, (10 + s) * C + co, c0 * r[4] + c2 * r[0], split, bad);
              const float4 g[5] = {c2 * r10, b6 * r8, a4 * r4, b2 * r8, c0 * r10};
              float4 t[5];
              rotT<5>(D2, g, t);
              if (s == 0) {
#pragma unroll
                for (int m = 0; m < 5; ++m) st4(gsrc + (4 + m) * C, t[m]);
              } else {
#pragma unroll
                for (int m = 0; m < 5; ++m) acc[m * C4 + c4] += t[m];
              }
#pragma unroll
              for (int rr2 = 0; rr2 < 5; ++rr2)
#pragma unroll
                for (int m = 0; m < 5; ++m) gw[rr2 * 5 + m] += dot4(g[rr2], v[m]);
            }
          }
        }
        // reduce this part's Wigner-gradient partials across the warp
#pragma unroll
        for (int m = 0; m < nw; ++m) {
          const float tsum = warp_sum(gw[m]);
          if (lane == 0) s_red[warp][m] = tsum;
        }
        __syncwarp();
        if (lane < nw) g_wig[e * kWig + woff + lane] = s_red[warp][lane];
        __syncwarp();
      }
    }
    // target-side gradient of x[jn] for this part's rows
    float* gx = g_x + jn * 9 * (int64_t)C + (part ? 4 : 0) * C;
    for (int t = lane; t < nrows * C4; t += 32) {
      const int l = t / C4, c4 = t - l * C4;
      st4(gx + l * C + c4 * 4, acc[t]);
    }
    __syncwarp();
  }
  report_split_range(bad, err);
}

// Pass B: g_x[n] += sum over edges with source n (source CSR order) of the scratch rows.
__global__ void __launch_bounds__(256) gather_bwd_src_kernel(const int32_t* __restrict__ src_ptr,
                                                             const int32_t* __restrict__ src_col,
                                                             const float* __restrict__ g_src_rows,
                                                             float* __restrict__ g_x, int64_t N, int C) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  const int C4 = C >> 2;
  for (int64_t n = (int64_t)blockIdx.x * wpb + warp; n < N; n += (int64_t)gridDim.x * wpb) {
    const int kb = src_ptr[n], ke = src_ptr[n + 1];
    for (int l = 0; l < 9; ++l) {
      for (int c4 = lane; c4 < C4; c4 += 32) {
        float* gx = g_x + n * 9 * (int64_t)C + l * C + c4 * 4;
        float4 a = ld4(gx);
        for (int k = kb; k < ke; ++k) a += ld4_stream(g_src_rows + (int64_t)src_col[k] * 9 * C + l * C + c4 * 4);
        st4(gx, a);
      }
    }
  }
}

void launch_gather_fwd(const float* x, const int64_t* idx_i, const int64_t* idx_j, const float* wig, const float* rad,
                       const float* csd, const int64_t* batch, float* X0, float* X1, float* X2, int64_t E, int C,
                       bool split, int* err, cudaStream_t s) {
  gather_fwd_kernel<<<grid_for(E, kFwdWarps, 3), kFwdWarps * 32, 0, s>>>(x, idx_i, idx_j, wig, rad, csd, batch, X0,
                                                                         X1, X2, E, C, split, err);
}

void launch_gather_bwd(const float* gX0, const float* gX1, const float* gX2, const float* x, const int64_t* idx_i,
                       const float* wig, const float* rad, const float* csd, const int64_t* batch,
                       const int32_t* dst_ptr, const int32_t* dst_col, const int32_t* src_ptr, const int32_t* src_col,
                       float* g_x, float* g_wig, float* g_rad, float* scratch, int64_t N, int C, bool split, int* err,
                       cudaStream_t s) {
  const size_t smem = (size_t)kBwdWarps * 5 * C * sizeof(float);
  if (smem > 48 * 1024) {
    cudaFuncSetAttribute(gather_bwd_dst_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaFuncSetAttribute(gather_bwd_dst_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  }
  gather_bwd_dst_kernel<0><<<grid_for(N, kBwdWarps, 2), kBwdWarps * 32, smem, s>>>(
      gX0, gX1, gX2, x, idx_i, wig, rad, csd, batch, dst_ptr, dst_col, g_x, g_wig, g_rad, scratch, N, C, split, err);
  gather_bwd_dst_kernel<1><<<grid_for(N, kBwdWarps, 2), kBwdWarps * 32, smem, s>>>(
      gX0, gX1, gX2, x, idx_i, wig, rad, csd, batch, dst_ptr, dst_col, g_x, g_wig, g_rad, scratch, N, C, split, err);
  gather_bwd_src_kernel<<<grid_for(N, 8, 8), 256, 0, s>>>(src_ptr, src_col, scratch, g_x, N, C);
}

}  // namespace fuma
