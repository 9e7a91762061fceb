// Node-wise equivariant RMS norm over the 9 real-SH coefficients of every atom, forward and
// backward, one warp per atom.
//
// The module is the stand-in for FAIRChem's rms_norm_sh that the layers call as norm_1 / norm_2
// and the model as final_norm (the reference's model.py:145,157,218); its definition, shared
// with the CPU oracle, is flash_uma_b200/nodewise.py::EquivariantRMSNormSH. Per atom, with x_k
// the C channels of coefficient k and l(k) its degree (0, 1,1,1, 2,2,2,2,2):
//   f_0 = x_0 - mean_c x_0,   f_k = x_k (k >= 1)
//   S = (1/C) sum_c sum_k w_k f_k[c]^2,   w_k = 1 / ((2 l(k) + 1)(lmax + 1))
//   s = 1 / sqrt(S + eps)
//   out_k = f_k s W[l(k)] (+ b on k = 0)
// Backward (input gradient; the affine parameters are frozen), with G_k = dL/dout_k:
//   P = sum_c sum_k G_k W[l(k)] f_k
//   dL/df_k = s G_k W[l(k)] - (s^3 / C) w_k f_k P
//   dL/dx_0 = dL/df_0 - mean_c dL/df_0,   dL/dx_k = dL/df_k (k >= 1)
// Lane l holds channels 4l.. of all 9 rows (VPL float4 per row for C up to 128 VPL), so each
// direction is one read of the atom's rows plus two (forward) or three (backward) warp sums.
#include "common.cuh"
#include "kernels.h"

namespace fuma {

namespace {

constexpr int kNodeWarps = 4;

}  // namespace

template <int VPL>
__global__ void __launch_bounds__(kNodeWarps * 32) rmsnorm_sh_fwd_kernel(
    const float* __restrict__ x, const float* __restrict__ aw, const float* __restrict__ ab,
    const float* __restrict__ bal, float eps, int64_t N, int C, float* __restrict__ out, float* __restrict__ rstd) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C4 = C >> 2;
  const float invC = 1.0f / (float)C;
  for (int64_t n = (int64_t)blockIdx.x * kNodeWarps + warp; n < N; n += (int64_t)gridDim.x * kNodeWarps) {
    const float* xr = x + n * 9 * (int64_t)C;
    float4 v[9][VPL];
#pragma unroll
    for (int k = 0; k < 9; ++k)
#pragma unroll
      for (int q = 0; q < VPL; ++q) {
        const int c4 = lane + 32 * q;
        v[k][q] = c4 < C4 ? ld4(xr + k * C + c4 * 4) : f4(0.f);
      }
    float s0 = 0.f;
#pragma unroll
    for (int q = 0; q < VPL; ++q) s0 += (v[0][q].x + v[0][q].y) + (v[0][q].z + v[0][q].w);
    const float m = warp_sum(s0) * invC;
#pragma unroll
    for (int q = 0; q < VPL; ++q)
      if (lane + 32 * q < C4) v[0][q] = v[0][q] - f4(m);
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < 9; ++k) {
      float sk = 0.f;
#pragma unroll
      for (int q = 0; q < VPL; ++q) sk += dot4(v[k][q], v[k][q]);
      ss = fmaf(__ldg(bal + k), sk, ss);
    }
    const float s = rsqrtf(warp_sum(ss) * invC + eps);
    if (lane == 0) rstd[n] = s;
    float* orow = out + n * 9 * (int64_t)C;
#pragma unroll
    for (int q = 0; q < VPL; ++q) {
      const int c4 = lane + 32 * q;
      if (c4 >= C4) continue;
      const float4 w0 = ld4_keep(aw + c4 * 4), w1 = ld4_keep(aw + C + c4 * 4), w2 = ld4_keep(aw + 2 * C + c4 * 4);
#pragma unroll
      for (int k = 0; k < 9; ++k) {
        const float4 w = k == 0 ? w0 : (k < 4 ? w1 : w2);
        float4 o = (v[k][q] * s) * w;
        if (k == 0) o = o + ld4_keep(ab + c4 * 4);
        st4(orow + k * C + c4 * 4, o);
      }
    }
  }
}

template <int VPL>
__global__ void __launch_bounds__(kNodeWarps * 32) rmsnorm_sh_bwd_kernel(
    const float* __restrict__ x, const float* __restrict__ aw, const float* __restrict__ bal,
    const float* __restrict__ rstd, const float* __restrict__ g_out, int64_t N, int C, float* __restrict__ g_x) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C4 = C >> 2;
  const float invC = 1.0f / (float)C;
  for (int64_t n = (int64_t)blockIdx.x * kNodeWarps + warp; n < N; n += (int64_t)gridDim.x * kNodeWarps) {
    const float* xr = x + n * 9 * (int64_t)C;
    const float* gr = g_out + n * 9 * (int64_t)C;
    float4 f[9][VPL], gw[9][VPL];
    float s0 = 0.f, p = 0.f;
#pragma unroll
    for (int q = 0; q < VPL; ++q) {
      const int c4 = lane + 32 * q;
      const bool on = c4 < C4;
      const float4 w0 = on ? ld4_keep(aw + c4 * 4) : f4(0.f), w1 = on ? ld4_keep(aw + C + c4 * 4) : f4(0.f),
                   w2 = on ? ld4_keep(aw + 2 * C + c4 * 4) : f4(0.f);
#pragma unroll
      for (int k = 0; k < 9; ++k) {
        f[k][q] = on ? ld4(xr + k * C + c4 * 4) : f4(0.f);
        gw[k][q] = on ? ld4(gr + k * C + c4 * 4) * (k == 0 ? w0 : (k < 4 ? w1 : w2)) : f4(0.f);
      }
      s0 += (f[0][q].x + f[0][q].y) + (f[0][q].z + f[0][q].w);
    }
    const float m = warp_sum(s0) * invC;
#pragma unroll
    for (int q = 0; q < VPL; ++q)
      if (lane + 32 * q < C4) f[0][q] = f[0][q] - f4(m);
#pragma unroll
    for (int k = 0; k < 9; ++k)
#pragma unroll
      for (int q = 0; q < VPL; ++q) p += dot4(gw[k][q], f[k][q]);
    const float s = rstd[n];
    const float coef = warp_sum(p) * s * s * s * invC;
    // dL/df_k = s gw_k - coef w_k f_k; the l = 0 row then loses its channel mean
    float g0 = 0.f;
#pragma unroll
    for (int k = 0; k < 9; ++k) {
      const float ck = coef * __ldg(bal + k);
#pragma unroll
      for (int q = 0; q < VPL; ++q) {
        gw[k][q] = gw[k][q] * s - f[k][q] * ck;
        if (k == 0) g0 += (gw[0][q].x + gw[0][q].y) + (gw[0][q].z + gw[0][q].w);
      }
    }
    const float gm = warp_sum(g0) * invC;
    float* orow = g_x + n * 9 * (int64_t)C;
#pragma unroll
    for (int q = 0; q < VPL; ++q) {
      const int c4 = lane + 32 * q;
      if (c4 >= C4) continue;
#pragma unroll
      for (int k = 0; k < 9; ++k) st4(orow + k * C + c4 * 4, k == 0 ? gw[0][q] - f4(gm) : gw[k][q]);
    }
  }
}

void launch_rmsnorm_sh_fwd(const float* x, const float* aw, const float* ab, const float* bal, float eps, int64_t N,
                           int C, float* out, float* rstd, cudaStream_t s) {
  const int t = kNodeWarps * 32;
  if (C <= 128)
    rmsnorm_sh_fwd_kernel<1><<<grid_resident(rmsnorm_sh_fwd_kernel<1>, t, N, kNodeWarps), t, 0, s>>>(
        x, aw, ab, bal, eps, N, C, out, rstd);
  else
    rmsnorm_sh_fwd_kernel<2><<<grid_resident(rmsnorm_sh_fwd_kernel<2>, t, N, kNodeWarps), t, 0, s>>>(
        x, aw, ab, bal, eps, N, C, out, rstd);
}

void launch_rmsnorm_sh_bwd(const float* x, const float* aw, const float* bal, const float* rstd, const float* g_out,
                           int64_t N, int C, float* g_x, cudaStream_t s) {
  const int t = kNodeWarps * 32;
  if (C <= 128)
    rmsnorm_sh_bwd_kernel<1><<<grid_resident(rmsnorm_sh_bwd_kernel<1>, t, N, kNodeWarps), t, 0, s>>>(
        x, aw, bal, rstd, g_out, N, C, g_x);
  else
    rmsnorm_sh_bwd_kernel<2><<<grid_resident(rmsnorm_sh_bwd_kernel<2>, t, N, kNodeWarps), t, 0, s>>>(
        x, aw, bal, rstd, g_out, N, C, g_x);
}

}  // namespace fuma
