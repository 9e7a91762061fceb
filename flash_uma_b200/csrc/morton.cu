// Morton order of the atoms and the renumbered graph (the reference's reorder_graph_morton,
// model.py:47-74, run at the start of every forward, model.py:189).
//
// The reference quantises every position to 10 bits per axis over the global bounding box,
//   q = int32((pos - pos_min) * (1023 / max(pos_max - pos_min, 1e-5)))   (per axis, fp32)
// interleaves the bits into a 30-bit code (x in bit 0, y in bit 1, z in bit 2 of every triple),
// sorts the atoms stably by key = code | (system << 32), and renumbers the edges. Here, for up to
// kMortonMaxAtoms atoms, one block of 1024 threads does the bounding box, the codes and the sort in
// shared memory: a bitonic sort of (key, atom index) pairs, which orders ties by index, i.e. the
// stable order. The fp32 operations are the reference's (subtract, then multiply by the per-axis
// scale, truncating conversion), so the order is identical. A second grid-stride kernel gathers
// positions, species and system ids and renumbers both edge index rows.
#include "common.cuh"
#include "kernels.h"

namespace fuma {

namespace {

constexpr int kSortThreads = 1024;

__device__ __forceinline__ uint32_t expand_bits10(uint32_t v) {   // 10 bits -> every third bit
  v = (v | (v << 16)) & 0x030000FFu;
  v = (v | (v << 8)) & 0x0300F00Fu;
  v = (v | (v << 4)) & 0x030C30C3u;
  v = (v | (v << 2)) & 0x09249249u;
  return v;
}

}  // namespace

__global__ void __launch_bounds__(kSortThreads) morton_sort_kernel(const float* __restrict__ pos,
                                                                   const int64_t* __restrict__ batch, int N, int P,
                                                                   int64_t* __restrict__ perm,
                                                                   int64_t* __restrict__ inv_perm) {
  extern __shared__ uint64_t s_key[];                        // [P]
  int32_t* s_idx = reinterpret_cast<int32_t*>(s_key + P);    // [P]
  __shared__ float s_red[6][kSortThreads / 32];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  // bounding box
  float mn[3] = {3.402823466e38f, 3.402823466e38f, 3.402823466e38f};
  float mx[3] = {-3.402823466e38f, -3.402823466e38f, -3.402823466e38f};
  for (int a = t; a < N; a += kSortThreads)
#pragma unroll
    for (int d = 0; d < 3; ++d) {
      const float v = pos[a * 3 + d];
      mn[d] = fminf(mn[d], v);
      mx[d] = fmaxf(mx[d], v);
    }
#pragma unroll
  for (int d = 0; d < 3; ++d)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mn[d] = fminf(mn[d], __shfl_xor_sync(kFull, mn[d], o));
      mx[d] = fmaxf(mx[d], __shfl_xor_sync(kFull, mx[d], o));
    }
  if (lane == 0)
#pragma unroll
    for (int d = 0; d < 3; ++d) {
      s_red[d][warp] = mn[d];
      s_red[3 + d][warp] = mx[d];
    }
  __syncthreads();
  float lo[3], sc[3];
#pragma unroll
  for (int d = 0; d < 3; ++d) {
    float a = s_red[d][0], b = s_red[3 + d][0];
    for (int w = 1; w < kSortThreads / 32; ++w) {
      a = fminf(a, s_red[d][w]);
      b = fmaxf(b, s_red[3 + d][w]);
    }
    lo[d] = a;
    sc[d] = 1023.0f / fmaxf(b - a, 1e-5f);
  }
  // keys; padding sorts last
  for (int a = t; a < P; a += kSortThreads) {
    uint64_t key = ~uint64_t(0);
    if (a < N) {
      uint32_t code = 0;
#pragma unroll
      for (int d = 0; d < 3; ++d) {
        const int32_t q = (int32_t)((pos[a * 3 + d] - lo[d]) * sc[d]);
        code |= expand_bits10((uint32_t)q) << d;
      }
      key = (uint64_t)code | ((uint64_t)batch[a] << 32);
    }
    s_key[a] = key;
    s_idx[a] = a;
  }
  __syncthreads();
  // bitonic sort of (key, index), ascending
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = t; i < P; i += kSortThreads) {
        const int p = i ^ j;
        if (p > i) {
          const uint64_t ki = s_key[i], kp = s_key[p];
          const int32_t ii = s_idx[i], ip = s_idx[p];
          const bool gt = ki > kp || (ki == kp && ii > ip);   // (i) after (p)
          const bool up = (i & k) == 0;
          if (gt == up) {
            s_key[i] = kp;
            s_key[p] = ki;
            s_idx[i] = ip;
            s_idx[p] = ii;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int a = t; a < N; a += kSortThreads) {
    const int32_t o = s_idx[a];
    perm[a] = o;
    inv_perm[o] = a;
  }
}

__global__ void __launch_bounds__(256) morton_apply_kernel(const float* __restrict__ pos,
                                                           const int64_t* __restrict__ Z,
                                                           const int64_t* __restrict__ batch,
                                                           const int64_t* __restrict__ idx_i,
                                                           const int64_t* __restrict__ idx_j,
                                                           const int64_t* __restrict__ perm,
                                                           const int64_t* __restrict__ inv_perm, int64_t N, int64_t E,
                                                           float* __restrict__ pos_s, int64_t* __restrict__ Z_s,
                                                           int64_t* __restrict__ batch_s, int64_t* __restrict__ ii,
                                                           int64_t* __restrict__ jj) {
  const int64_t n = N > E ? N : E;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
    if (t < N) {
      const int64_t o = perm[t];
      if (pos_s) {
        pos_s[t * 3] = pos[o * 3];
        pos_s[t * 3 + 1] = pos[o * 3 + 1];
        pos_s[t * 3 + 2] = pos[o * 3 + 2];
      }
      Z_s[t] = Z[o];
      batch_s[t] = batch[o];
    }
    if (t < E) {
      ii[t] = inv_perm[idx_i[t]];
      jj[t] = inv_perm[idx_j[t]];
    }
  }
}

cudaError_t launch_morton_reorder(const float* pos, const int64_t* Z, const int64_t* batch, const int64_t* idx_i,
                                  const int64_t* idx_j, int64_t N, int64_t E, int64_t* perm, int64_t* inv_perm,
                                  float* pos_s, int64_t* Z_s, int64_t* batch_s, int64_t* ii, int64_t* jj,
                                  cudaStream_t s) {
  int P = 1;
  while (P < N) P <<= 1;
  if (P < 2) P = 2;
  const size_t smem = (size_t)P * (sizeof(uint64_t) + sizeof(int32_t));
  static thread_local uint64_t configured = 0;   // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured >> (dev & 63) & 1)) {
    const size_t mx = (size_t)kMortonMaxAtoms * (sizeof(uint64_t) + sizeof(int32_t));
    const cudaError_t st = cudaFuncSetAttribute(morton_sort_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mx);
    if (st != cudaSuccess) return st;
    configured |= uint64_t(1) << (dev & 63);
  }
  if (N > 0) morton_sort_kernel<<<1, kSortThreads, smem, s>>>(pos, batch, (int)N, P, perm, inv_perm);
  const int64_t n = N > E ? N : E;
  if (n > 0)
    morton_apply_kernel<<<grid_resident(morton_apply_kernel, 256, n, 256), 256, 0, s>>>(
        pos, Z, batch, idx_i, idx_j, perm, inv_perm, N, E, pos_s, Z_s, batch_s, ii, jj);
  return cudaGetLastError();
}

}  // namespace fuma
