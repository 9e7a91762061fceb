// Shared device helpers for the flash_uma_b200 kernels (sm_100a).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

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

// Logistic sigmoid of the LN-SiLU and gating kernels through CUDA's fast intrinsics (__expf:
// ex2-based exponential, __fdividef: approximate quotient); a few ulp per value, as the
// reference's Triton tl.sigmoid. For -x beyond the fp32 range __expf gives inf and the
// quotient 0, the limit. 8-21% faster LN-SiLU / gating kernels than expf and an IEEE divide.
__device__ __forceinline__ float sigmoidf_(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }

// One round of the recursive-halving warp reduction: lanes with bit OFF clear keep entries
// [0, OFF), the others [OFF, 2 OFF) (moved down to [0, OFF)), each adding its partner's copy.
template <int OFF, int NV>
__device__ __forceinline__ void halve(float (&v)[NV], int lane) {
  const bool upper = (lane & OFF) != 0;
#pragma unroll
  for (int k = 0; k < OFF; ++k) {
    const float send = upper ? v[k] : v[k + OFF];
    const float keep = upper ? v[k + OFF] : v[k];
    v[k] = keep + __shfl_xor_sync(kFull, send, OFF);
  }
}

// Warp reduction of NV per-lane partial sums (NV = 16 or 32): lane l receives the warp total
// of v[l % NV], in NV - 1 (+1) shuffles instead of 5 per value.
template <int NV>
__device__ __forceinline__ float warp_transpose_sum(float (&v)[NV], int lane) {
  if constexpr (NV == 32) halve<16>(v, lane);
  halve<8>(v, lane);
  halve<4>(v, lane);
  halve<2>(v, lane);
  halve<1>(v, lane);
  float r = v[0];
  if constexpr (NV == 16) r += __shfl_xor_sync(kFull, r, 16);
  return r;
}

// Contiguous, even share [begin, end) of n_units work units for warp w of n_warps: the shares
// differ by at most one unit, so every SM ends up with the same work to within one unit per
// warp (a grid-stride loop gives some warps one more round than others: with 4,000 atoms over
// 2,368 resident warps, SMs of 32 atoms against a mean of 27).
struct Share {
  int64_t begin, end;
};
__device__ __forceinline__ Share warp_share(int64_t n_units, int64_t w, int64_t n_warps) {
  const int64_t q = n_units / n_warps, r = n_units % n_warps;
  const int64_t b = w * q + (w < r ? w : r);
  return {b, b + q + (w < r ? 1 : 0)};
}

// ---- cp.async (global -> shared, per-thread groups) ------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
// wait until at most N of this thread's cp.async groups are still in flight
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// ---- f16x3 split operands -------------------------------------------------------------------
// The fp16 tensor-core GEMM takes each fp32 operand value x as hi + lo * 2^-11 with
// hi = fp16_rn(x) and lo = fp16_rn((x - hi) * 2^11) (the residual, scaled so it stays a normal
// fp16 number). Producers of GEMM inputs can write that split directly, "row-packed": an fp32
// [rows, W] output keeps its 4W bytes per row, the fp16 hi values of the row in its first 2W
// bytes and the fp16 lo values in the next 2W bytes (row slices stay valid).
constexpr float kSplitLoScale = 2048.0f;
constexpr int kErrSplitRange = 16;   // error code: a finite value at or beyond the fp16 limit

__device__ __forceinline__ uint32_t h2_bits(__half2 h) {
  uint32_t u;
  memcpy(&u, &h, 4);
  return u;
}

// Split 4 values; `bad` is set if one of them is finite but rounds beyond the fp16 range.
__device__ __forceinline__ void split_f16x4(float4 v, uint2& hi, uint2& lo, bool& bad) {
  const __half2 h01 = __float22half2_rn(make_float2(v.x, v.y));
  const __half2 h23 = __float22half2_rn(make_float2(v.z, v.w));
  const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
  const __half2 l01 =
      __float22half2_rn(make_float2((v.x - f01.x) * kSplitLoScale, (v.y - f01.y) * kSplitLoScale));
  const __half2 l23 =
      __float22half2_rn(make_float2((v.z - f23.x) * kSplitLoScale, (v.w - f23.y) * kSplitLoScale));
  hi = make_uint2(h2_bits(h01), h2_bits(h23));
  lo = make_uint2(h2_bits(l01), h2_bits(l23));
  const float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
  bad |= (m >= 65520.0f) & (m <= 3.402823466e38f);
}

// Store 4 consecutive values at column `col` of the [*, W] output row starting at `row`:
// split = 0: plain fp32 (streaming); 2: the row-packed split (hi and lo halves); 1: only the
// hi halves of the row-packed split (the operand of the single-product GEMM, which reads
// nothing else; the lo half of the row is left as it is, and no lo value is computed).
// `amax` keeps the largest magnitude stored as a split; report_split_range checks it once at the
// end of the kernel (NaN is ignored by fmaxf; an infinity in the data also hides a finite
// overflow of the same thread, which is then already visible in the results).
__device__ __forceinline__ void st_out4(float* row, int W, int col, float4 v, int split, float& amax) {
  if (!split) {
    st4_stream(row + col, v);
    return;
  }
  const __half2 h01 = __float22half2_rn(make_float2(v.x, v.y));
  const __half2 h23 = __float22half2_rn(make_float2(v.z, v.w));
  uint8_t* rb = reinterpret_cast<uint8_t*>(row);
  __stcs(reinterpret_cast<uint2*>(rb + 2 * col), make_uint2(h2_bits(h01), h2_bits(h23)));
  if (split == 2) {
    const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
    const __half2 l01 =
        __float22half2_rn(make_float2((v.x - f01.x) * kSplitLoScale, (v.y - f01.y) * kSplitLoScale));
    const __half2 l23 =
        __float22half2_rn(make_float2((v.z - f23.x) * kSplitLoScale, (v.w - f23.y) * kSplitLoScale));
    __stcs(reinterpret_cast<uint2*>(rb + 2 * (W + col)), make_uint2(h2_bits(l01), h2_bits(l23)));
  }
  amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
}

// ---- 16-bit activation storage (the single-product mode) ------------------------------------
// The single-product GEMMs can write their results as fp16 (radial output, conv1 Y, conv2
// output); the kernels that read them take the pointer as float* and, with kHalf, treat it as
// __half* with the same element offsets.
__device__ __forceinline__ float4 h4_to_f4(uint2 u) {
  __half2 a, b;
  memcpy(&a, &u.x, 4);
  memcpy(&b, &u.y, 4);
  const float2 fa = __half22float2(a), fb = __half22float2(b);
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}
template <bool kHalf>
__device__ __forceinline__ float4 ld4_act(const float* base, int64_t idx) {
  if constexpr (kHalf) {
    return h4_to_f4(__ldcs(reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(base) + idx)));
  } else {
    return ld4_stream(base + idx);
  }
}
__device__ __forceinline__ void cp_async8(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_addr(smem)), "l"(gmem) : "memory");
}
// copy 4 activation values into a 16-byte shared-memory slot (fp16: its first 8 bytes)
template <bool kHalf>
__device__ __forceinline__ void cp_act(float4* slot, const float* base, int64_t idx) {
  if constexpr (kHalf) {
    cp_async8(slot, reinterpret_cast<const __half*>(base) + idx);
  } else {
    cp_async16(slot, base + idx);
  }
}
template <bool kHalf>
__device__ __forceinline__ float4 sm_act(const float4* slot) {
  if constexpr (kHalf) {
    return h4_to_f4(*reinterpret_cast<const uint2*>(slot));
  } else {
    return *slot;
  }
}

__device__ __forceinline__ void report_split_range(bool bad, int* err) {
  if (bad && err) atomicCAS(err, 0, kErrSplitRange);
}
__device__ __forceinline__ void report_split_range(float amax, int* err) {
  if (amax >= 65520.0f && amax <= 3.402823466e38f && err) atomicCAS(err, 0, kErrSplitRange);
}

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

// Blocks of `fn` (at `threads` threads per block) that fit on one SM at once, from the
// compiled register and shared-memory use; queried once per kernel, block size and device.
inline int resident_blocks(const void* fn, int threads) {
  struct Entry {
    const void* fn;
    int dev, threads, n;
  };
  static thread_local Entry cache[48];
  static thread_local int used = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  for (int i = 0; i < used; ++i)
    if (cache[i].fn == fn && cache[i].dev == dev && cache[i].threads == threads) return cache[i].n;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, threads, 0) != cudaSuccess || n < 1) {
    (void)cudaGetLastError();
    n = 1;
  }
  if (used < 48) cache[used++] = Entry{fn, dev, threads, n};
  return n;
}

// Grid of a grid-stride kernel: one wave of resident blocks (or fewer blocks if the work is
// smaller), so no block waits for an SM while others run their last iterations.
template <typename Kernel>
inline unsigned grid_resident(Kernel* fn, int threads, int64_t items, int per_block) {
  return grid_for(items, per_block, resident_blocks(reinterpret_cast<const void*>(fn), threads));
}

}  // namespace fuma
