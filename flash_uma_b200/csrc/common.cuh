// Shared device helpers for the flash_uma_b200 kernels (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace fuma {

constexpr int kWarp = 32;
constexpr unsigned kFull = 0xffffffffu;
constexpr int kWig = 34;  // packed Wigner row: D1 3x3 (0..8) + D2 5x5 (9..33)

// ---- float4 arithmetic -------------------------------------------------------------------
__device__ __forceinline__ float4 f4(float v) { return make_float4(v, v, v, v); }
__device__ __forceinline__ float4 operator+(float4 a, float4 b) { return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w); }
__device__ __forceinline__ float4 operator-(float4 a, float4 b) { return make_float4(a.x - b.x, a.y - b.y, a.z - b.z, a.w - b.w); }
__device__ __forceinline__ float4 operator*(float4 a, float4 b) { return make_float4(a.x * b.x, a.y * b.y, a.z * b.z, a.w * b.w); }
__device__ __forceinline__ float4 operator*(float s, float4 a) { return make_float4(s * a.x, s * a.y, s * a.z, s * a.w); }
__device__ __forceinline__ float4 operator*(float4 a, float s) { return make_float4(s * a.x, s * a.y, s * a.z, s * a.w); }
__device__ __forceinline__ void operator+=(float4& a, float4 b) { a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w; }
// a += s * b  (fused)
__device__ __forceinline__ void fma4(float4& a, float s, float4 b) {
  a.x = fmaf(s, b.x, a.x); a.y = fmaf(s, b.y, a.y); a.z = fmaf(s, b.z, a.z); a.w = fmaf(s, b.w, a.w);
}
__device__ __forceinline__ float4 div4(float4 a, float d) { return make_float4(a.x / d, a.y / d, a.z / d, a.w / d); }
__device__ __forceinline__ float dot4(float4 a, float4 b) { return a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w; }

// ---- global memory with cache hints --------------------------------------------------------
// Streaming (read-once / write-once) traffic uses the evict-first hints so that the
// node tensors, which are gathered many times, stay resident in L2.
__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 ld4_stream(const float* p) { return __ldcs(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ float4 ld4_keep(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ void st4_stream(float* p, float4 v) { __stcs(reinterpret_cast<float4*>(p), v); }

// ---- fp64 float4 accumulators --------------------------------------------------------------
struct d4 { double x, y, z, w; };
__device__ __forceinline__ d4 d4_of(float4 a) { return {(double)a.x, (double)a.y, (double)a.z, (double)a.w}; }
__device__ __forceinline__ void operator+=(d4& a, float4 b) { a.x += (double)b.x; a.y += (double)b.y; a.z += (double)b.z; a.w += (double)b.w; }
__device__ __forceinline__ float4 f4_of(d4 a) { return make_float4((float)a.x, (float)a.y, (float)a.z, (float)a.w); }

// ---- warp reductions ----------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

// ---- host-side launch helpers ------------------------------------------------------------
inline int sm_count() {
  static thread_local int cached_dev = -1, cached_n = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cached_n;
  if (dev != cached_dev) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0) cached_n = n;
    cached_dev = dev;
  }
  return cached_n;
}

// grid for a grid-stride kernel over `items` with `per_block` items per block, capped at
// `blocks_per_sm` resident blocks on every SM
inline unsigned grid_for(int64_t items, int per_block, int blocks_per_sm) {
  const int64_t need = (items + per_block - 1) / per_block;
  const int64_t cap = (int64_t)sm_count() * blocks_per_sm;
  const int64_t g = need < cap ? need : cap;
  return (unsigned)(g > 0 ? g : 1);
}

}  // namespace fuma
