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
  const Share sh = warp_share(N, (int64_t)blockIdx.x * kNodeWarps + warp, (int64_t)gridDim.x * kNodeWarps);
  for (int64_t n = sh.begin; n < sh.end; ++n) {
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
  const Share sh = warp_share(N, (int64_t)blockIdx.x * kNodeWarps + warp, (int64_t)gridDim.x * kNodeWarps);
  for (int64_t n = sh.begin; n < sh.end; ++n) {
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

// ---- gated atom-wise block (the stand-in SpectralAtomwise, flash_uma_b200/nodewise.py; the
// atom_wise module of the reference's layers, model.py:157) --------------------------------------
// With h [9, N, H] the per-coefficient output of the first per-degree linear map (no bias) and
// u [N, 2H] the scalar MLP pre-activation (bias included):
//   z_0 = SiLU(h_0 + b1),  z_k = h_k * sigmoid(SiLU(u))[l(k) - 1 block]  (k >= 1)
// Thread per (atom, 4 channels); h and z are coefficient-major (row k * N + n), the layout in
// which each degree's map is one GEMM over rows of the same degree.
namespace {

__device__ __forceinline__ float4 silu4(float4 a) {
  return make_float4(a.x * sigmoidf_(a.x), a.y * sigmoidf_(a.y), a.z * sigmoidf_(a.z), a.w * sigmoidf_(a.w));
}
__device__ __forceinline__ float dsilu(float a) {   // d/da a sigmoid(a)
  const float s = sigmoidf_(a);
  return s * (1.0f + a * (1.0f - s));
}
__device__ __forceinline__ float4 dsilu4(float4 a) { return make_float4(dsilu(a.x), dsilu(a.y), dsilu(a.z), dsilu(a.w)); }
__device__ __forceinline__ float4 sig4n(float4 a) {
  return make_float4(sigmoidf_(a.x), sigmoidf_(a.y), sigmoidf_(a.z), sigmoidf_(a.w));
}

}  // namespace

// Coefficient rows of the atom-wise block: row k * N + n of a coefficient-major array holds
// coefficient k of atom n. The per-degree maps run as one GEMM against the three degree weights
// stacked ([W_0; W_1; W_2]), whose output is "degree-blocked": row k * N + n, column block
// deg(k) * width holds the product with the weight of coefficient k's own degree (the other two
// blocks are not read). Plain layouts: ld = width, block offset 0.
__device__ __forceinline__ int coef_degree(int k) { return k == 0 ? 0 : (k < 4 ? 1 : 2); }

// z = [silu(h_0 + b1), h_1..3 * sigmoid(silu(u_1)), h_4..8 * sigmoid(silu(u_2))] on coefficient
// rows (h: row stride ldh, column block deg(k) * H when blocked; u [N, 2H]). z [9N, H] fp32
// (split 0) or its row-packed split (split 1, 2).
__global__ void __launch_bounds__(256) atomwise_gate_fwd_kernel(const float* __restrict__ h, int64_t ldh,
                                                                 int blocked, const float* __restrict__ u,
                                                                 const float* __restrict__ b1, int64_t N, int H,
                                                                 float* __restrict__ z, int split, int* err) {
  const int H4 = H >> 2;
  float amax = 0.f;   // largest magnitude written as a split (range check at the end)
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < N * H4; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = t / H4;
    const int c = (int)(t - n * H4) * 4;
    const float4 g1 = sig4n(silu4(ld4(u + n * 2 * H + c))), g2 = sig4n(silu4(ld4(u + n * 2 * H + H + c)));
    st_out4(z + n * H, H, c, silu4(ld4(h + n * ldh + c) + ld4_keep(b1 + c)), split, amax);
#pragma unroll
    for (int k = 1; k < 9; ++k) {
      const int64_t r = k * N + n;
      const float4 v = ld4(h + r * ldh + (blocked ? coef_degree(k) * H : 0) + c);
      st_out4(z + r * H, H, c, v * (k < 4 ? g1 : g2), split, amax);
    }
  }
  report_split_range(amax, err);
}

// Backward of the gating, given gz = dL/dz on coefficient rows (same layout as h): gh = dL/dh
// [9N, H] and gu = dL/du [N, 2H], fp32 (split 0) or row-packed splits (split 1, 2).
__global__ void __launch_bounds__(256) atomwise_gate_bwd_kernel(const float* __restrict__ gz,
                                                                 const float* __restrict__ h, int64_t ldh,
                                                                 int blocked, const float* __restrict__ u,
                                                                 const float* __restrict__ b1, int64_t N, int H,
                                                                 float* __restrict__ gh, float* __restrict__ gu,
                                                                 int split, int* err) {
  const int H4 = H >> 2;
  float amax = 0.f;   // largest magnitude written as a split (range check at the end)
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < N * H4; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = t / H4;
    const int c = (int)(t - n * H4) * 4;
    const float4 u1 = ld4(u + n * 2 * H + c), u2 = ld4(u + n * 2 * H + H + c);
    const float4 a1 = silu4(u1), a2 = silu4(u2);
    const float4 g1 = sig4n(a1), g2 = sig4n(a2);
    st_out4(gh + n * H, H, c, ld4(gz + n * ldh + c) * dsilu4(ld4(h + n * ldh + c) + ld4_keep(b1 + c)), split, amax);
    float4 s1 = f4(0.f), s2 = f4(0.f);
#pragma unroll
    for (int k = 1; k < 9; ++k) {
      const int64_t r = k * N + n;
      const int64_t o = r * ldh + (blocked ? coef_degree(k) * H : 0) + c;
      const float4 g = ld4(gz + o);
      st_out4(gh + r * H, H, c, g * (k < 4 ? g1 : g2), split, amax);
      if (k < 4)
        s1 += g * ld4(h + o);
      else
        s2 += g * ld4(h + o);
    }
    const float4 one = f4(1.f);
    st_out4(gu + n * 2 * H, 2 * H, c, s1 * (g1 * (one - g1)) * dsilu4(u1), split, amax);
    st_out4(gu + n * 2 * H, 2 * H, H + c, s2 * (g2 * (one - g2)) * dsilu4(u2), split, amax);
  }
  report_split_range(amax, err);
}

// out[n, k, :] = src[k * N + n, block(k) :] (+ add[n, k, :]) (+ row0[n or 0, :] on k = 0):
// coefficient rows (row stride lds, column block deg(k) * W when blocked) back to the node-major
// [N, 9, W] layout, with the residual and the l = 0 bias (forward) or the scalar-MLP input
// gradient (backward) folded in.
__global__ void __launch_bounds__(256) coef_to_node_kernel(const float* __restrict__ src, int64_t lds, int blocked,
                                                           const float* __restrict__ add,
                                                           const float* __restrict__ row0, int row0_per_node,
                                                           int64_t N, int W, float* __restrict__ out) {
  const int W4 = W >> 2;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < N * 9 * W4;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t nk = t / W4;
    const int c = (int)(t - nk * W4) * 4;
    const int64_t n = nk / 9;
    const int k = (int)(nk - n * 9);
    float4 v = ld4(src + (k * N + n) * lds + (blocked ? coef_degree(k) * W : 0) + c);
    if (add) v = v + ld4(add + nk * W + c);
    if (k == 0 && row0) v = v + ld4(row0 + (row0_per_node ? n * W : 0) + c);
    st4(out + nk * W + c, v);
  }
}

// The node-major [N, 9, W] array x as coefficient rows (row k * N + n = x[n, k, :]): the
// row-packed split (split 1, 2) that the tensor-core GEMMs of the atom-wise block read.
__global__ void __launch_bounds__(256) node_to_coef_kernel(const float* __restrict__ x, int64_t N, int W,
                                                           float* __restrict__ out, int split, int* err) {
  const int W4 = W >> 2;
  float amax = 0.f;   // largest magnitude written as a split (range check at the end)
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < N * 9 * W4;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t nk = t / W4;
    const int c = (int)(t - nk * W4) * 4;
    const int64_t n = nk / 9;
    const int k = (int)(nk - n * 9);
    st_out4(out + (k * N + n) * W, W, c, ld4_stream(x + nk * W + c), split, amax);
  }
  report_split_range(amax, err);
}

void launch_atomwise_gate_fwd(const float* h, int64_t ldh, bool blocked, const float* u, const float* b1, int64_t N,
                              int H, float* z, int split, int* err, cudaStream_t s) {
  atomwise_gate_fwd_kernel<<<grid_resident(atomwise_gate_fwd_kernel, 256, N * (H / 4), 256), 256, 0, s>>>(
      h, ldh, blocked ? 1 : 0, u, b1, N, H, z, split, err);
}

void launch_atomwise_gate_bwd(const float* gz, const float* h, int64_t ldh, bool blocked, const float* u,
                              const float* b1, int64_t N, int H, float* gh, float* gu, int split, int* err,
                              cudaStream_t s) {
  atomwise_gate_bwd_kernel<<<grid_resident(atomwise_gate_bwd_kernel, 256, N * (H / 4), 256), 256, 0, s>>>(
      gz, h, ldh, blocked ? 1 : 0, u, b1, N, H, gh, gu, split, err);
}

void launch_coef_to_node(const float* src, int64_t lds, bool blocked, const float* add, const float* row0,
                         int row0_per_node, int64_t N, int W, float* out, cudaStream_t s) {
  coef_to_node_kernel<<<grid_resident(coef_to_node_kernel, 256, N * 9 * (W / 4), 256), 256, 0, s>>>(
      src, lds, blocked ? 1 : 0, add, row0, row0_per_node, N, W, out);
}

void launch_node_to_coef(const float* x, int64_t N, int W, float* out, int split, int* err, cudaStream_t s) {
  node_to_coef_kernel<<<grid_resident(node_to_coef_kernel, 256, N * 9 * (W / 4), 256), 256, 0, s>>>(x, N, W, out,
                                                                                                   split, err);
}

}  // namespace fuma
