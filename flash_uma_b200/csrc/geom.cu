// Edge geometry: distances, envelope, Gaussian basis, element embeddings and the
// l<=2 Wigner blocks of the edge frame (forward), and the analytic gradient with
// respect to the edge vector (backward).
//
// Reference: ops/geom.py:36-214 (forward), :220-493 (backward).
//
// Forward, per edge e = (i -> j):  d = pos_i - pos_j + shift_e,
//   env = 1 - 21u^5 + 35u^6 - 15u^7 (u = |d|/cutoff < 1, else 0),
//   x_edge_raw[e] = [exp(coeff (|d| - mu_b)^2) for b < B, W_src[Z_i], W_tgt[Z_j]],
//   q = blended two-chart quaternion that rotates d/|d| onto +y,
//   D1 = R(q) (3x3), D2 = l=2 representation of R in the real basis
//   (xz, xy, (2y^2-x^2-z^2)/sqrt3 /2..., yz, z^2-x^2) written as quadratic forms of
//   R's rows a, b, c:
//     D2 rows = [P(a,c), P(a,b), (2P(b,b) - P(a,a) - P(c,c)) / (2 sqrt3), P(b,c), (P(c,c) - P(a,a)) / 2]
//   with P(u,v) = [u0v2+u2v0, u0v1+u1v0, (2u1v1-u0v0-u2v2)/sqrt3, u1v2+u2v1, u2v2-u0v0].
//
// Backward: per edge the gradient with respect to d (this is g_shifts[e]); the
// per-atom sums g_pos[n] = sum_{e: i=n} g_e - sum_{e: j=n} g_e are done by
// node_vec3_segment_kernel in a fixed order (no atomics, run-to-run deterministic).
#include "common.cuh"
#include "kernels.h"

namespace fuma {

namespace {

constexpr float kEps = 1e-7f;
constexpr float kInvSqrt3 = 0.57735026918962576f;

struct Frame {
  float ex, ey, ez, dist, dist_safe;
  // chart quaternions (w, x, z) for chart 1 (y = 0) and (w, x, y) for chart 2 (z = 0)
  float q1w, q1x, q1z, n1, q2w, q2x, q2y, n2;
  float t, s, sign1;
  float quw, qux, quy, quz, ne;   // unnormalised blend and its norm
  float qw, qx, qy, qz;           // normalised quaternion
};

__device__ __forceinline__ void edge_frame(float dx, float dy, float dz, Frame& f) {
  f.dist = sqrtf(dx * dx + dy * dy + dz * dz);
  f.dist_safe = fmaxf(f.dist, kEps);
  f.ex = dx / f.dist_safe; f.ey = dy / f.dist_safe; f.ez = dz / f.dist_safe;
  const float ex = f.ex, ey = f.ey, ez = f.ez;
  f.n1 = sqrtf((1.f + ey) * (1.f + ey) + ez * ez + ex * ex + kEps);
  f.q1w = (1.f + ey) / f.n1; f.q1x = -ez / f.n1; f.q1z = ex / f.n1;
  f.n2 = sqrtf(ez * ez + (1.f - ey) * (1.f - ey) + ex * ex + kEps);
  f.q2w = -ez / f.n2; f.q2x = (1.f - ey) / f.n2; f.q2y = ex / f.n2;
  f.t = fminf(fmaxf((ey + 0.9f) / 1.8f, 0.f), 1.f);
  const float num = 2.f * f.t - 1.f;
  const float den = fmaxf(f.t * (1.f - f.t), kEps);
  float s = 1.f / (1.f + expf(-(num / den)));
  if (f.t < kEps) s = 0.f;
  if (f.t > 1.f - kEps) s = 1.f;
  f.s = s;
  f.sign1 = (f.q1w * f.q2w + f.q1x * f.q2x) < 0.f ? -1.f : 1.f;
  const float a1w = f.sign1 * f.q1w, a1x = f.sign1 * f.q1x, a1z = f.sign1 * f.q1z;
  f.quw = (1.f - s) * f.q2w + s * a1w;
  f.qux = (1.f - s) * f.q2x + s * a1x;
  f.quy = (1.f - s) * f.q2y;
  f.quz = s * a1z;
  f.ne = sqrtf(f.quw * f.quw + f.qux * f.qux + f.quy * f.quy + f.quz * f.quz + kEps);
  f.qw = f.quw / f.ne; f.qx = f.qux / f.ne; f.qy = f.quy / f.ne; f.qz = f.quz / f.ne;
}

__device__ __forceinline__ void rotation(const Frame& f, float R[9]) {
  const float w = f.qw, x = f.qx, y = f.qy, z = f.qz;
  R[0] = 1.f - 2.f * (y * y + z * z); R[1] = 2.f * (x * y - w * z);       R[2] = 2.f * (x * z + w * y);
  R[3] = 2.f * (x * y + w * z);       R[4] = 1.f - 2.f * (x * x + z * z); R[5] = 2.f * (y * z - w * x);
  R[6] = 2.f * (x * z - w * y);       R[7] = 2.f * (y * z + w * x);       R[8] = 1.f - 2.f * (x * x + y * y);
}

__device__ __forceinline__ void Pform(const float* u, const float* v, float out[5]) {
  out[0] = u[0] * v[2] + u[2] * v[0];
  out[1] = u[0] * v[1] + u[1] * v[0];
  out[2] = (2.f * u[1] * v[1] - u[0] * v[0] - u[2] * v[2]) * kInvSqrt3;
  out[3] = u[1] * v[2] + u[2] * v[1];
  out[4] = u[2] * v[2] - u[0] * v[0];
}

__device__ __forceinline__ void wigner_l2(const float R[9], float D2[25]) {
  const float* a = R; const float* b = R + 3; const float* c = R + 6;
  float paa[5], pbb[5], pcc[5];
  Pform(a, c, D2 + 0);
  Pform(a, b, D2 + 5);
  Pform(a, a, paa); Pform(b, b, pbb); Pform(c, c, pcc);
  const float k = 0.5f * kInvSqrt3;
#pragma unroll
  for (int m = 0; m < 5; ++m) {
    D2[10 + m] = (2.f * pbb[m] - paa[m] - pcc[m]) * k;
    D2[20 + m] = 0.5f * (pcc[m] - paa[m]);
  }
  Pform(b, c, D2 + 15);
}

// g_u += K(G) v, the adjoint of P(u, v) with respect to u (P is symmetric in u, v).
__device__ __forceinline__ void Padj(const float G[5], const float* v, float s, float* gu) {
  const float g2 = G[2] * kInvSqrt3;
  gu[0] += s * ((-g2 - G[4]) * v[0] + G[1] * v[1] + G[0] * v[2]);
  gu[1] += s * (G[1] * v[0] + 2.f * g2 * v[1] + G[3] * v[2]);
  gu[2] += s * (G[0] * v[0] + G[3] * v[1] + (-g2 + G[4]) * v[2]);
}

}  // namespace

// One warp per tile of 32 edges: lane-per-edge for the scalar geometry, then the
// warp writes the 34 Wigner values (staged in shared memory) and the B + 2C wide
// x_edge_raw rows cooperatively so that every store is coalesced.
__global__ void __launch_bounds__(128) geom_fwd_kernel(
    const float* __restrict__ pos, const int64_t* __restrict__ Z, const int64_t* __restrict__ idx_i,
    const int64_t* __restrict__ idx_j, const float* __restrict__ shifts, const float* __restrict__ W_src,
    const float* __restrict__ W_tgt, const float* __restrict__ offset_g, float* __restrict__ x_edge,
    float* __restrict__ wig, float* __restrict__ env_out, int64_t E, int B, int C, float cutoff, float coeff) {
  __shared__ float s_w[4][32 * 35];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t ntiles = (E + 31) / 32;
  const int row = B + 2 * C;
  const bool vec = ((B & 3) == 0) && ((C & 3) == 0);
  for (int64_t tile = (int64_t)blockIdx.x * 4 + warp; tile < ntiles; tile += (int64_t)gridDim.x * 4) {
    const int64_t e0 = tile * 32;
    const int nvalid = (E - e0) < 32 ? (int)(E - e0) : 32;
    const int64_t e = e0 + lane;
    float dist = 0.f;
    int zi = 0, zj = 0;
    if (lane < nvalid) {
      const int64_t i = idx_i[e], j = idx_j[e];
      zi = (int)Z[i]; zj = (int)Z[j];
      const float dx = pos[i * 3 + 0] - pos[j * 3 + 0] + shifts[e * 3 + 0];
      const float dy = pos[i * 3 + 1] - pos[j * 3 + 1] + shifts[e * 3 + 1];
      const float dz = pos[i * 3 + 2] - pos[j * 3 + 2] + shifts[e * 3 + 2];
      Frame f;
      edge_frame(dx, dy, dz, f);
      dist = f.dist;
      const float u = f.dist / cutoff;
      const float u5 = (u * u) * (u * u) * u;
      const float ev = u < 1.f ? 1.f + u5 * (-21.f + u * (35.f - 15.f * u)) : 0.f;
      env_out[e] = ev;
      float R[9], D2[25];
      rotation(f, R);
      wigner_l2(R, D2);
      float* sw = s_w[warp] + lane * 35;
#pragma unroll
      for (int k = 0; k < 9; ++k) sw[k] = R[k];
#pragma unroll
      for (int k = 0; k < 25; ++k) sw[9 + k] = D2[k];
    }
    __syncwarp();
    // coalesced Wigner write-out: element m of the tile's [nvalid, 34] block
    for (int m = lane; m < nvalid * kWig; m += 32) {
      const int r = m / kWig, k = m - r * kWig;
      wig[e0 * kWig + m] = s_w[warp][r * 35 + k];
    }
    // x_edge_raw rows, one per edge of the tile
    for (int r = 0; r < nvalid; ++r) {
      const float dr = __shfl_sync(kFull, dist, r);
      const int zir = __shfl_sync(kFull, zi, r), zjr = __shfl_sync(kFull, zj, r);
      float* out = x_edge + (e0 + r) * (int64_t)row;
      for (int b = lane; b < B; b += 32) {
        const float diff = dr - offset_g[b];
        out[b] = expf(coeff * diff * diff);
      }
      const float* ws = W_src + (int64_t)zir * C;
      const float* wt = W_tgt + (int64_t)zjr * C;
      if (vec) {
        for (int c4 = lane; c4 < (C >> 2); c4 += 32) {
          st4(out + B + c4 * 4, ld4_keep(ws + c4 * 4));
          st4(out + B + C + c4 * 4, ld4_keep(wt + c4 * 4));
        }
      } else {
        for (int c = lane; c < C; c += 32) {
          out[B + c] = ws[c];
          out[B + C + c] = wt[c];
        }
      }
    }
    __syncwarp();
  }
}

// Thread per edge. g_vec[e] = dL/dd for d = pos_i - pos_j + shift_e.
__global__ void __launch_bounds__(128) geom_bwd_kernel(
    const float* __restrict__ pos, const int64_t* __restrict__ idx_i, const int64_t* __restrict__ idx_j,
    const float* __restrict__ shifts, const float* __restrict__ offset_g, const float* __restrict__ g_xe,
    int64_t xe_stride, const float* __restrict__ g_wig, const float* __restrict__ g_env, float* __restrict__ g_vec,
    int64_t E, int B, float cutoff, float coeff) {
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < E; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = idx_i[e], j = idx_j[e];
    const float dx = pos[i * 3 + 0] - pos[j * 3 + 0] + shifts[e * 3 + 0];
    const float dy = pos[i * 3 + 1] - pos[j * 3 + 1] + shifts[e * 3 + 1];
    const float dz = pos[i * 3 + 2] - pos[j * 3 + 2] + shifts[e * 3 + 2];
    Frame f;
    edge_frame(dx, dy, dz, f);
    float R[9];
    rotation(f, R);
    // ---- dL/dR from the D1 block (direct) and the D2 block (quadratic forms)
    const float* gw = g_wig + e * kWig;
    float gR[9];
#pragma unroll
    for (int k = 0; k < 9; ++k) gR[k] = gw[k];
    float G[5][5];
#pragma unroll
    for (int r = 0; r < 5; ++r)
#pragma unroll
      for (int m = 0; m < 5; ++m) G[r][m] = gw[9 + r * 5 + m];
    const float* a = R; const float* b = R + 3; const float* c = R + 6;
    float* ga = gR; float* gb = gR + 3; float* gc = gR + 6;
    Padj(G[0], c, 1.f, ga); Padj(G[0], a, 1.f, gc);             // row 0: P(a, c)
    Padj(G[1], b, 1.f, ga); Padj(G[1], a, 1.f, gb);             // row 1: P(a, b)
    Padj(G[2], b, 2.f * kInvSqrt3, gb);                         // row 2: (2P(b,b)-P(a,a)-P(c,c))/(2 sqrt3)
    Padj(G[2], a, -kInvSqrt3, ga);
    Padj(G[2], c, -kInvSqrt3, gc);
    Padj(G[3], c, 1.f, gb); Padj(G[3], b, 1.f, gc);             // row 3: P(b, c)
    Padj(G[4], c, 1.f, gc); Padj(G[4], a, -1.f, ga);            // row 4: (P(c,c)-P(a,a))/2
    // ---- dL/dq through R(q)
    const float w = f.qw, x = f.qx, y = f.qy, z = f.qz;
    const float gqw = 2.f * (z * (gR[3] - gR[1]) + y * (gR[2] - gR[6]) + x * (gR[7] - gR[5]));
    const float gqx = 2.f * (y * (gR[1] + gR[3]) + z * (gR[2] + gR[6]) + w * (gR[7] - gR[5])) - 4.f * x * (gR[4] + gR[8]);
    const float gqy = 2.f * (x * (gR[1] + gR[3]) + z * (gR[5] + gR[7]) + w * (gR[2] - gR[6])) - 4.f * y * (gR[0] + gR[8]);
    const float gqz = 2.f * (x * (gR[2] + gR[6]) + y * (gR[5] + gR[7]) + w * (gR[3] - gR[1])) - 4.f * z * (gR[0] + gR[4]);
    // ---- normalisation q = qu / sqrt(|qu|^2 + eps)
    const float proj = gqw * w + gqx * x + gqy * y + gqz * z;
    const float guw = (gqw - w * proj) / f.ne, gux = (gqx - x * proj) / f.ne;
    const float guy = (gqy - y * proj) / f.ne, guz = (gqz - z * proj) / f.ne;
    // ---- blend qu = (1-s) q2 + s sign1 q1
    const float s = f.s;
    const float a1w = f.sign1 * f.q1w, a1x = f.sign1 * f.q1x, a1z = f.sign1 * f.q1z;
    const float gs = guw * (a1w - f.q2w) + gux * (a1x - f.q2x) + guy * (0.f - f.q2y) + guz * a1z;
    const float g1w = f.sign1 * s * guw, g1x = f.sign1 * s * gux, g1z = f.sign1 * s * guz;
    const float g2w = (1.f - s) * guw, g2x = (1.f - s) * gux, g2y = (1.f - s) * guy;
    float gex = 0.f, gey = 0.f, gez = 0.f;
    // chart 1: q1 = (1+ey, -ez, ex) / n1
    {
      const float p = g1w * f.q1w + g1x * f.q1x + g1z * f.q1z;
      const float hw = (g1w - f.q1w * p) / f.n1, hx = (g1x - f.q1x * p) / f.n1, hz = (g1z - f.q1z * p) / f.n1;
      gey += hw; gez -= hx; gex += hz;
    }
    // chart 2: q2 = (-ez, 1-ey, ex) / n2
    {
      const float p = g2w * f.q2w + g2x * f.q2x + g2y * f.q2y;
      const float hw = (g2w - f.q2w * p) / f.n2, hx = (g2x - f.q2x * p) / f.n2, hy = (g2y - f.q2y * p) / f.n2;
      gez -= hw; gey -= hx; gex += hy;
    }
    // blend weight s(t(ey)), only inside the open interval where it is not clamped
    if (f.t > kEps && f.t < 1.f - kEps) {
      const float num = 2.f * f.t - 1.f;
      const float tt = f.t * (1.f - f.t);
      const float den = fmaxf(tt, kEps);
      const float dden = tt > kEps ? 1.f - 2.f * f.t : 0.f;
      const float darg = (2.f * den - num * dden) / (den * den);
      gey += gs * s * (1.f - s) * darg * (1.f / 1.8f);
    }
    // ---- radial terms: envelope and Gaussians depend on |d|
    const float u = f.dist / cutoff;
    float gdist = 0.f;
    if (u < 1.f) {
      const float u4 = (u * u) * (u * u);
      gdist += g_env[e] * u4 * (-105.f + u * (210.f - 105.f * u)) / cutoff;
    }
    const float* gx = g_xe + e * xe_stride;
    for (int bb = 0; bb < B; ++bb) {
      const float diff = f.dist - offset_g[bb];
      const float gauss = expf(coeff * diff * diff);
      gdist += gx[bb] * 2.f * coeff * diff * gauss;
    }
    // ---- unit vector e = d / max(|d|, eps)
    const float pe = gex * f.ex + gey * f.ey + gez * f.ez;
    g_vec[e * 3 + 0] = (gex - f.ex * pe) / f.dist_safe + gdist * f.ex;
    g_vec[e * 3 + 1] = (gey - f.ey * pe) / f.dist_safe + gdist * f.ey;
    g_vec[e * 3 + 2] = (gez - f.ez * pe) / f.dist_safe + gdist * f.ez;
  }
}

// g_pos[n] = sum_{e in src segment of n} g_vec[e] - sum_{e in dst segment of n} g_vec[e],
// accumulated in fp64 in CSR order (deterministic).
__global__ void node_vec3_segment_kernel(const int32_t* __restrict__ src_ptr, const int32_t* __restrict__ src_col,
                                         const int32_t* __restrict__ dst_ptr, const int32_t* __restrict__ dst_col,
                                         const float* __restrict__ g_vec, float* __restrict__ g_pos, int64_t N) {
  for (int64_t n = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; n < N; n += (int64_t)gridDim.x * blockDim.x) {
    double ax = 0.0, ay = 0.0, az = 0.0;
    for (int k = src_ptr[n]; k < src_ptr[n + 1]; ++k) {
      const int64_t e = src_col[k];
      ax += g_vec[e * 3 + 0]; ay += g_vec[e * 3 + 1]; az += g_vec[e * 3 + 2];
    }
    for (int k = dst_ptr[n]; k < dst_ptr[n + 1]; ++k) {
      const int64_t e = dst_col[k];
      ax -= g_vec[e * 3 + 0]; ay -= g_vec[e * 3 + 1]; az -= g_vec[e * 3 + 2];
    }
    g_pos[n * 3 + 0] = (float)ax; g_pos[n * 3 + 1] = (float)ay; g_pos[n * 3 + 2] = (float)az;
  }
}

void launch_geom_fwd(const float* pos, const int64_t* Z, const int64_t* idx_i, const int64_t* idx_j,
                     const float* shifts, const float* W_src, const float* W_tgt, const float* offset_g,
                     float* x_edge, float* wig, float* env_out, int64_t E, int B, int C, float cutoff, float coeff,
                     cudaStream_t s) {
  const int64_t tiles = (E + 31) / 32;
  geom_fwd_kernel<<<grid_for(tiles, 4, 8), 128, 0, s>>>(pos, Z, idx_i, idx_j, shifts, W_src, W_tgt, offset_g, x_edge,
                                                        wig, env_out, E, B, C, cutoff, coeff);
}

void launch_geom_bwd(const float* pos, const int64_t* idx_i, const int64_t* idx_j, const float* shifts,
                     const float* offset_g, const float* g_xe, int64_t xe_stride, const float* g_wig,
                     const float* g_env, float* g_vec, int64_t E, int B, float cutoff, float coeff, cudaStream_t s) {
  geom_bwd_kernel<<<grid_for(E, 128, 8), 128, 0, s>>>(pos, idx_i, idx_j, shifts, offset_g, g_xe, xe_stride, g_wig,
                                                      g_env, g_vec, E, B, cutoff, coeff);
}

void launch_node_vec3_segment(const int32_t* src_ptr, const int32_t* src_col, const int32_t* dst_ptr,
                              const int32_t* dst_col, const float* g_vec, float* g_pos, int64_t N, cudaStream_t s) {
  node_vec3_segment_kernel<<<grid_for(N, 128, 8), 128, 0, s>>>(src_ptr, src_col, dst_ptr, dst_col, g_vec, g_pos, N);
}

}  // namespace fuma
