// Streaming kernels: split gating (forward/backward) and fused LayerNorm + SiLU.
//
// Gating reference: ops/gating.py:32-103 (forward), :109-185 (backward).
//   g0 = sigmoid(Y0[0]), g1 = sigmoid(Y0[1])
//   Z_m0 = [silu(Y0[2]), Y0[3] g0, Y0[4] g1]; Z_m1 = [Y1[0] g0, Y1[1] g1, Y1[2] g0, Y1[3] g1];
//   Z_m2 = [Y2[0] g1, Y2[1] g1]                        (C-wide slots, per edge)
// LayerNorm + SiLU reference: ops/ln_silu.py:29-72 (forward), :77-123 (backward, dx only):
//   y = (x - mean) * rstd * gamma + beta, rstd = 1/sqrt(var + eps) (biased variance), out = y sigmoid(y)
#include "common.cuh"
#include "kernels.h"

namespace fuma {

namespace {
__device__ __forceinline__ float4 sig4(float4 a) {
  return make_float4(sigmoidf_(a.x), sigmoidf_(a.y), sigmoidf_(a.z), sigmoidf_(a.w));
}
}  // namespace

// One thread per (edge, 4 channels). kH: Y is stored as fp16 (the single-product mode).
template <bool kH>
__global__ void __launch_bounds__(256) gating_fwd_kernel(const float* __restrict__ Y0, const float* __restrict__ Y1,
                                                         const float* __restrict__ Y2, float* __restrict__ Z0,
                                                         float* __restrict__ Z1, float* __restrict__ Z2, int64_t E,
                                                         int C, int split, int* err) {
  const int C4 = C >> 2;
  float amax = 0.f;   // largest magnitude written as a split (range check at the end)
  const int64_t total = E * C4;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = t / C4;
    const int co = (int)(t - e * C4) * 4;
    const int64_t y0 = e * 5 * (int64_t)C + co, y1 = e * 4 * (int64_t)C + co, y2 = e * 2 * (int64_t)C + co;
    // every load of the row first (11 x 16 bytes in flight per thread), then the arithmetic
    const float4 p0 = ld4_act<kH>(Y0, y0), p1 = ld4_act<kH>(Y0, y0 + C), a = ld4_act<kH>(Y0, y0 + 2 * C);
    const float4 y3 = ld4_act<kH>(Y0, y0 + 3 * C), y4 = ld4_act<kH>(Y0, y0 + 4 * C);
    const float4 u0 = ld4_act<kH>(Y1, y1), u1 = ld4_act<kH>(Y1, y1 + C), u2 = ld4_act<kH>(Y1, y1 + 2 * C),
                 u3 = ld4_act<kH>(Y1, y1 + 3 * C);
    const float4 w0 = ld4_act<kH>(Y2, y2), w1 = ld4_act<kH>(Y2, y2 + C);
    const float4 g0 = sig4(p0), g1 = sig4(p1);
    float* z0 = Z0 + e * 3 * (int64_t)C;
    float* z1 = Z1 + e * 4 * (int64_t)C;
    float* z2 = Z2 + e * 2 * (int64_t)C;
    st_out4(z0, 3 * C, co, a * sig4(a), split, amax);
    st_out4(z0, 3 * C, C + co, y3 * g0, split, amax);
    st_out4(z0, 3 * C, 2 * C + co, y4 * g1, split, amax);
    st_out4(z1, 4 * C, co, u0 * g0, split, amax);
    st_out4(z1, 4 * C, C + co, u1 * g1, split, amax);
    st_out4(z1, 4 * C, 2 * C + co, u2 * g0, split, amax);
    st_out4(z1, 4 * C, 3 * C + co, u3 * g1, split, amax);
    st_out4(z2, 2 * C, co, w0 * g1, split, amax);
    st_out4(z2, 2 * C, C + co, w1 * g1, split, amax);
  }
  report_split_range(amax, err);
}

template <bool kH>
__global__ void __launch_bounds__(256) gating_bwd_kernel(
    const float* __restrict__ gZ0, const float* __restrict__ gZ1, const float* __restrict__ gZ2,
    const float* __restrict__ Y0, const float* __restrict__ Y1, const float* __restrict__ Y2,
    float* __restrict__ gY0, float* __restrict__ gY1, float* __restrict__ gY2, int64_t E, int C, int split,
    int* err) {
  const int C4 = C >> 2;
  float amax = 0.f;   // largest magnitude written as a split (range check at the end)
  const int64_t total = E * C4;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = t / C4;
    const int co = (int)(t - e * C4) * 4;
    const int64_t y0 = e * 5 * (int64_t)C + co, y1 = e * 4 * (int64_t)C + co, y2 = e * 2 * (int64_t)C + co;
    const int64_t q0 = e * 3 * (int64_t)C + co, q1 = e * 4 * (int64_t)C + co, q2 = e * 2 * (int64_t)C + co;
    const float4 g0 = sig4(ld4_act<kH>(Y0, y0)), g1 = sig4(ld4_act<kH>(Y0, y0 + C));
    const float4 a = ld4_act<kH>(Y0, y0 + 2 * C), sa = sig4(a);
    const float4 y3 = ld4_act<kH>(Y0, y0 + 3 * C), y4 = ld4_act<kH>(Y0, y0 + 4 * C);
    const float4 u0 = ld4_act<kH>(Y1, y1), u1 = ld4_act<kH>(Y1, y1 + C), u2 = ld4_act<kH>(Y1, y1 + 2 * C),
                 u3 = ld4_act<kH>(Y1, y1 + 3 * C);
    const float4 w0 = ld4_act<kH>(Y2, y2), w1 = ld4_act<kH>(Y2, y2 + C);
    const float4 ga = ld4_act<kH>(gZ0, q0), g3 = ld4_act<kH>(gZ0, q0 + C), g4 = ld4_act<kH>(gZ0, q0 + 2 * C);
    const float4 h0 = ld4_act<kH>(gZ1, q1), h1 = ld4_act<kH>(gZ1, q1 + C), h2 = ld4_act<kH>(gZ1, q1 + 2 * C),
                 h3 = ld4_act<kH>(gZ1, q1 + 3 * C);
    const float4 k0 = ld4_act<kH>(gZ2, q2), k1 = ld4_act<kH>(gZ2, q2 + C);
    const float4 one = f4(1.f);
    const float4 dg0 = g0 * (one - g0), dg1 = g1 * (one - g1);
    float* p0 = gY0 + e * 5 * (int64_t)C;
    float* p1 = gY1 + e * 4 * (int64_t)C;
    float* p2 = gY2 + e * 2 * (int64_t)C;
    st_out4(p0, 5 * C, co, dg0 * (g3 * y3 + h0 * u0 + h2 * u2), split, amax);
    st_out4(p0, 5 * C, C + co, dg1 * (g4 * y4 + h1 * u1 + h3 * u3 + k0 * w0 + k1 * w1), split, amax);
    st_out4(p0, 5 * C, 2 * C + co, ga * (sa + a * (sa * (one - sa))), split, amax);
    st_out4(p0, 5 * C, 3 * C + co, g3 * g0, split, amax);
    st_out4(p0, 5 * C, 4 * C + co, g4 * g1, split, amax);
    st_out4(p1, 4 * C, co, h0 * g0, split, amax);
    st_out4(p1, 4 * C, C + co, h1 * g1, split, amax);
    st_out4(p1, 4 * C, 2 * C + co, h2 * g0, split, amax);
    st_out4(p1, 4 * C, 3 * C + co, h3 * g1, split, amax);
    st_out4(p2, 2 * C, co, k0 * g1, split, amax);
    st_out4(p2, 2 * C, C + co, k1 * g1, split, amax);
  }
  report_split_range(amax, err);
}

// One warp per group of ROWS rows (their loads in flight together); VPL float4 per lane
// (D <= 128 * VPL), rows kept in registers.
template <int VPL, int ROWS>
__global__ void __launch_bounds__(256) ln_silu_fwd_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                                                          const float* __restrict__ beta, float* __restrict__ out,
                                                          float* __restrict__ mean_out, float* __restrict__ rstd_out,
                                                          int64_t M, int D, float eps, int split, int* err) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  const int D4 = D >> 2;
  float amax = 0.f;   // largest magnitude written as a split (range check at the end)
  for (int64_t r0 = ((int64_t)blockIdx.x * wpb + warp) * ROWS; r0 < M; r0 += (int64_t)gridDim.x * wpb * ROWS) {
    float4 v[ROWS][VPL];
    float s[ROWS];
#pragma unroll
    for (int i = 0; i < ROWS; ++i) {
      s[i] = 0.f;
      const bool row_ok = r0 + i < M;
#pragma unroll
      for (int q = 0; q < VPL; ++q) {
        const int d4 = lane + 32 * q;
        v[i][q] = (row_ok && d4 < D4) ? ld4_stream(x + (r0 + i) * D + d4 * 4) : f4(0.f);
        s[i] += (v[i][q].x + v[i][q].y) + (v[i][q].z + v[i][q].w);
      }
    }
    float mean[ROWS], rstd[ROWS];
#pragma unroll
    for (int i = 0; i < ROWS; ++i) mean[i] = warp_sum(s[i]) / (float)D;
#pragma unroll
    for (int i = 0; i < ROWS; ++i) {
      float ss = 0.f;
#pragma unroll
      for (int q = 0; q < VPL; ++q) {
        const int d4 = lane + 32 * q;
        if (d4 < D4) {
          const float4 c = v[i][q] - f4(mean[i]);
          ss += dot4(c, c);
        }
      }
      s[i] = ss;
    }
#pragma unroll
    for (int i = 0; i < ROWS; ++i) rstd[i] = 1.0f / sqrtf(warp_sum(s[i]) / (float)D + eps);
#pragma unroll
    for (int i = 0; i < ROWS; ++i) {
      const int64_t r = r0 + i;
      if (r >= M) break;
      if (lane == 0) { mean_out[r] = mean[i]; rstd_out[r] = rstd[i]; }
      float* orow = out + r * D;
#pragma unroll
      for (int q = 0; q < VPL; ++q) {
        const int d4 = lane + 32 * q;
        if (d4 < D4) {
          const float4 y = (v[i][q] - f4(mean[i])) * rstd[i] * ld4_keep(gamma + d4 * 4) + ld4_keep(beta + d4 * 4);
          st_out4(orow, D, d4 * 4, y * sig4(y), split, amax);
        }
      }
    }
  }
  report_split_range(amax, err);
}

template <int VPL, int ROWS>
__global__ void __launch_bounds__(256) ln_silu_bwd_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                                                          const float* __restrict__ beta, const float* __restrict__ mean,
                                                          const float* __restrict__ rstd, const float* __restrict__ g_out,
                                                          float* __restrict__ g_x, int64_t M, int D, int split,
                                                          int* err) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  const int D4 = D >> 2;
  float amax = 0.f;   // largest magnitude written as a split (range check at the end)
  for (int64_t r0 = ((int64_t)blockIdx.x * wpb + warp) * ROWS; r0 < M; r0 += (int64_t)gridDim.x * wpb * ROWS) {
    float4 xh[ROWS][VPL], gxh[ROWS][VPL];
    float s1[ROWS], s2[ROWS], rs[ROWS];
#pragma unroll
    for (int i = 0; i < ROWS; ++i) {
      const int64_t r = r0 + i;
      const bool row_ok = r < M;
      const float mu = row_ok ? mean[r] : 0.f;
      rs[i] = row_ok ? rstd[r] : 0.f;
      s1[i] = 0.f;
      s2[i] = 0.f;
#pragma unroll
      for (int q = 0; q < VPL; ++q) {
        const int d4 = lane + 32 * q;
        if (row_ok && d4 < D4) {
          xh[i][q] = (ld4_stream(x + r * D + d4 * 4) - f4(mu)) * rs[i];
          const float4 gm = ld4_keep(gamma + d4 * 4);
          const float4 y = xh[i][q] * gm + ld4_keep(beta + d4 * 4);
          const float4 sg = sig4(y);
          const float4 ds = sg + y * (sg * (f4(1.f) - sg));
          gxh[i][q] = ld4_stream(g_out + r * D + d4 * 4) * ds * gm;
          s1[i] += (gxh[i][q].x + gxh[i][q].y) + (gxh[i][q].z + gxh[i][q].w);
          s2[i] += dot4(gxh[i][q], xh[i][q]);
        } else {
          xh[i][q] = f4(0.f);
          gxh[i][q] = f4(0.f);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < ROWS; ++i) {
      s1[i] = warp_sum(s1[i]);
      s2[i] = warp_sum(s2[i]);
    }
    const float invD = 1.0f / (float)D;
#pragma unroll
    for (int i = 0; i < ROWS; ++i) {
      const int64_t r = r0 + i;
      if (r >= M) break;
#pragma unroll
      for (int q = 0; q < VPL; ++q) {
        const int d4 = lane + 32 * q;
        if (d4 < D4)
          st_out4(g_x + r * D, D, d4 * 4, (gxh[i][q] - (f4(s1[i]) + xh[i][q] * s2[i]) * invD) * rs[i], split, amax);
      }
    }
  }
  report_split_range(amax, err);
}

// Backward of rows of at most 128 values, one row per warp per iteration with the next row's
// loads (x, dL/dh, mean, 1/std) issued before the current row is reduced, so two rows' loads
// are in flight per warp; 64 registers, 4 blocks per SM. Same arithmetic as
// ln_silu_bwd_kernel<1, 1>; 47 -> 37 us at E = 120,000 (B200).
__global__ void __launch_bounds__(256, 4) ln_silu_bwd_row_kernel(const float* __restrict__ x,
                                                              const float* __restrict__ gamma,
                                                              const float* __restrict__ beta,
                                                              const float* __restrict__ mean,
                                                              const float* __restrict__ rstd,
                                                              const float* __restrict__ g_out,
                                                              float* __restrict__ g_x, int64_t M, int D, int split,
                                                              int* err) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t stride = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int D4 = D >> 2;
  const bool act = lane < D4;
  const float invD = 1.0f / (float)D;
  const float4 gm = act ? ld4_keep(gamma + lane * 4) : f4(0.f), bt = act ? ld4_keep(beta + lane * 4) : f4(0.f);
  float amax = 0.f;   // largest magnitude written as a split (range check at the end)
  int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
  float4 nx = f4(0.f), ng = f4(0.f);
  float nmu = 0.f, nrs = 0.f;
  if (r < M) {
    if (act) {
      nx = ld4_stream(x + r * D + lane * 4);
      ng = ld4_stream(g_out + r * D + lane * 4);
    }
    nmu = mean[r];
    nrs = rstd[r];
  }
  for (; r < M; r += stride) {
    const float4 xv = nx, gv = ng;
    const float mu = nmu, rs = nrs;
    const int64_t rn = r + stride;
    if (rn < M) {
      if (act) {
        nx = ld4_stream(x + rn * D + lane * 4);
        ng = ld4_stream(g_out + rn * D + lane * 4);
      }
      nmu = mean[rn];
      nrs = rstd[rn];
    }
    float4 xh = f4(0.f), gxh = f4(0.f);
    if (act) {
      xh = (xv - f4(mu)) * rs;
      const float4 y = xh * gm + bt;
      const float4 sg = sig4(y);
      const float4 ds = sg + y * (sg * (f4(1.f) - sg));
      gxh = gv * ds * gm;
    }
    const float s1 = warp_sum((gxh.x + gxh.y) + (gxh.z + gxh.w));
    const float s2 = warp_sum(dot4(gxh, xh));
    if (act) st_out4(g_x + r * D, D, lane * 4, (gxh - (f4(s1) + xh * s2) * invD) * rs, split, amax);
  }
  report_split_range(amax, err);
}

// (A one-row-per-warp forward with the next row's load in flight, the scheme of
// ln_silu_bwd_row_kernel, measured slower here: 35.3 vs 31.0 us at E = 120,000.)
// Forward LayerNorm + SiLU of rows of at most 128 values: 8 lanes per row, 4 rows per warp
// (lane = 4 float4 of its row; reductions over the 8 lanes of a row), so four rows' loads are in
// flight per warp, for the radial MLP's E x 128 LayerNorms (0.46 -> 0.40 ms per step measured).
__device__ __forceinline__ float sum8(float v) {
  v += __shfl_xor_sync(kFull, v, 1);
  v += __shfl_xor_sync(kFull, v, 2);
  v += __shfl_xor_sync(kFull, v, 4);
  return v;
}

__global__ void __launch_bounds__(256) ln_silu_fwd_short_kernel(const float* __restrict__ x,
                                                                const float* __restrict__ gamma,
                                                                const float* __restrict__ beta, float* __restrict__ out,
                                                                float* __restrict__ mean_out,
                                                                float* __restrict__ rstd_out, int64_t M, int D,
                                                                float eps, int split, int* err) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  const int sub = lane >> 3, l8 = lane & 7;
  const int D4 = D >> 2;
  float amax = 0.f;   // largest magnitude written as a split (range check at the end)
  for (int64_t r0 = ((int64_t)blockIdx.x * wpb + warp) * 4; r0 < M; r0 += (int64_t)gridDim.x * wpb * 4) {
    const int64_t r = r0 + sub;
    const bool ok = r < M;
    float4 v[4];
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int d4 = l8 + 8 * q;
      v[q] = (ok && d4 < D4) ? ld4_stream(x + r * D + d4 * 4) : f4(0.f);
      s += (v[q].x + v[q].y) + (v[q].z + v[q].w);
    }
    const float mean = sum8(s) / (float)D;
    float ss = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (l8 + 8 * q < D4) {
        const float4 c = v[q] - f4(mean);
        ss += dot4(c, c);
      }
    }
    const float rstd = 1.0f / sqrtf(sum8(ss) / (float)D + eps);
    if (ok) {
      if (l8 == 0) {
        mean_out[r] = mean;
        rstd_out[r] = rstd;
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int d4 = l8 + 8 * q;
        if (d4 < D4) {
          const float4 y = (v[q] - f4(mean)) * rstd * ld4_keep(gamma + d4 * 4) + ld4_keep(beta + d4 * 4);
          st_out4(out + r * D, D, d4 * 4, y * sig4(y), split, amax);
        }
      }
    }
  }
  report_split_range(amax, err);
}

void launch_gating_fwd(const float* Y0, const float* Y1, const float* Y2, float* Z0, float* Z1, float* Z2, int64_t E,
                       int C, int split, int* err, cudaStream_t s, bool act_half) {
  if (act_half)
    gating_fwd_kernel<true><<<grid_resident(gating_fwd_kernel<true>, 256, E * (C / 4), 256), 256, 0, s>>>(
        Y0, Y1, Y2, Z0, Z1, Z2, E, C, split, err);
  else
    gating_fwd_kernel<false><<<grid_resident(gating_fwd_kernel<false>, 256, E * (C / 4), 256), 256, 0, s>>>(
        Y0, Y1, Y2, Z0, Z1, Z2, E, C, split, err);
}

void launch_gating_bwd(const float* gZ0, const float* gZ1, const float* gZ2, const float* Y0, const float* Y1,
                       const float* Y2, float* gY0, float* gY1, float* gY2, int64_t E, int C, int split, int* err,
                       cudaStream_t s, bool act_half) {
  if (act_half)
    gating_bwd_kernel<true><<<grid_resident(gating_bwd_kernel<true>, 256, E * (C / 4), 256), 256, 0, s>>>(
        gZ0, gZ1, gZ2, Y0, Y1, Y2, gY0, gY1, gY2, E, C, split, err);
  else
    gating_bwd_kernel<false><<<grid_resident(gating_bwd_kernel<false>, 256, E * (C / 4), 256), 256, 0, s>>>(
        gZ0, gZ1, gZ2, Y0, Y1, Y2, gY0, gY1, gY2, E, C, split, err);
}

void launch_ln_silu_fwd(const float* x, const float* gamma, const float* beta, float* out, float* mean, float* rstd,
                        int64_t M, int D, float eps, int split, int* err, cudaStream_t s) {
  const int d4 = D / 4;
  // rows of <= 128 values: 8 lanes per row; longer rows: one row per warp (several rows per
  // warp at 32 lanes each raised the register count and measured slower on B200)
#define FWD(V, R) \
  ln_silu_fwd_kernel<V, R><<<grid_resident(ln_silu_fwd_kernel<V, R>, 256, (M + R - 1) / R, 8), 256, 0, s>>>(x, gamma, beta, out, mean, rstd, M, D, eps, \
                                                                           split, err)
  if (d4 <= 32) {
    ln_silu_fwd_short_kernel<<<grid_resident(ln_silu_fwd_short_kernel, 256, (M + 3) / 4, 8), 256, 0, s>>>(x, gamma, beta, out, mean, rstd, M, D, eps,
                                                                         split, err);
  } else if (d4 <= 64) FWD(2, 1);
  else if (d4 <= 128) FWD(4, 1);
  else if (d4 <= 256) FWD(8, 1);
  else FWD(16, 1);
#undef FWD
}

void launch_ln_silu_bwd(const float* x, const float* gamma, const float* beta, const float* mean, const float* rstd,
                        const float* g_out, float* g_x, int64_t M, int D, int split, int* err, cudaStream_t s) {
  const int d4 = D / 4;
#define BWD(V, R)                                                                                                      \
  ln_silu_bwd_kernel<V, R><<<grid_resident(ln_silu_bwd_kernel<V, R>, 256, (M + R - 1) / R, 8), 256, 0, s>>>(x, gamma, beta, mean, rstd, g_out, g_x, M, \
                                                                           D, split, err)
  if (d4 <= 32) {   // (an 8-lanes-per-row variant measured slower: 0.68 vs 0.53 ms / step)
    ln_silu_bwd_row_kernel<<<grid_resident(ln_silu_bwd_row_kernel, 256, M, 8), 256, 0, s>>>(
        x, gamma, beta, mean, rstd, g_out, g_x, M, D, split, err);
  }
  else if (d4 <= 64) BWD(2, 1);
  else if (d4 <= 128) BWD(4, 1);
  else if (d4 <= 256) BWD(8, 1);
  else BWD(16, 1);
#undef BWD
}

}  // namespace fuma
