// Dense contraction C[M,N] = A[M,K] . W[N,K]^T (+ bias[N]) on the 5th-generation tensor
// cores (tcgen05, kind::tf32) with fp32-level accuracy (3xTF32 split).
//
// This replaces the cuBLAS F.linear calls of the reference's radial MLP and SO(2)
// convolutions (model.py:147-154, weights packed at :101-141) and their input-gradient
// GEMMs in the backward pass.
//
// Precision: every fp32 operand x is split into hi and lo parts. Weights (prepared once):
// hi = rn_tf32(x), lo = rn_tf32(x - hi). Activations: hi = the raw fp32 value, which the
// tensor core reads as TF32 by truncation, and lo = rn_tf32(x - trunc_tf32(x)), written by
// the kernel into shared memory. Three MMAs per K step, hi.hi + hi.lo + lo.hi,
// accumulate in fp32 in tensor memory; the dropped lo.lo term and the rounding of lo are
// ~2^-22 relative and unbiased (a truncating split biases every product the same way
// and the error then grows like sqrt(K)), i.e. fp32-level results. The weight
// halves are prepared once on the host side (weights are frozen); the activation
// halves are produced in shared memory by the kernel itself. kSplit=false gives the
// plain single-pass TF32 product (hi and lo not used).
//
// Structure (persistent, one CTA per SM, 320 threads, 128 x BN output tiles):
//   warp 0      TMA producer: A tile [128 x 32] and W tiles [BN x 32] (128-byte
//               swizzle, K-major) into a STAGES-deep ring, mbarrier complete_tx.
//   warp 1      allocates 2 x BN TMEM columns (two accumulators); lane 0 issues
//               tcgen05.mma (M=128, N=BN, K=8 per instruction), tcgen05.commit releases
//               ring slots and hands a finished accumulator to the epilogue.
//   warps 2-5   write A_lo next to the A tile (fence.proxy.async so the tensor core
//               sees the generic-proxy writes).
//   warps 6-9   drain the other accumulator with tcgen05.ld (each warp owns TMEM lanes
//               32*(warp%4)..+32), add the bias and store, while the next tile's K loop
//               runs.
// Every mbarrier wait is bounded; on timeout the kernel records a code in *err, waits
// (bounded) for its own in-flight copies and MMAs, releases TMEM and returns.
#include <cstdio>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace fuma {

namespace {

constexpr int kBM = 128;          // rows per tile (one tcgen05 M=128 MMA, cta_group::1)
constexpr int kBK = 32;           // fp32 elements per K step = one 128-byte swizzle row
constexpr int kThreads = 320;  // producer, MMA, 4 split warps, 4 epilogue warps

// Instruction descriptor: kind::tf32, fp32 accumulator, both operands K-major, M=128.
template <int BN>
__device__ __forceinline__ constexpr uint32_t instr_desc_tf32() {
  return (1u << 4)               // D format F32
         | (2u << 7)             // A format TF32
         | (2u << 10)            // B format TF32
         | ((uint32_t)(BN >> 3) << 17)
         | ((uint32_t)(kBM >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// Round-to-nearest TF32 split of one fp32 value: hi = rn_tf32(x), lo = rn_tf32(x - hi). Rounding
// (not truncation) keeps the residual errors unbiased, so they do not grow linearly with K.
__device__ __forceinline__ uint32_t rn_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ void split_rn(uint32_t xbits, uint32_t& hi, uint32_t& lo) {
  const float x = __uint_as_float(xbits);
  hi = rn_tf32(x);
  lo = rn_tf32(x - __uint_as_float(hi));
}

// Low part of the 3xTF32 split for an operand the tensor core truncates to TF32 itself:
// rn_tf32(x - trunc_tf32(x)) (exact difference, rounded to nearest so the residual is unbiased).
__device__ __forceinline__ uint32_t lo_part(uint32_t xbits) {
  const float x = __uint_as_float(xbits);
  const float t = __uint_as_float(xbits & 0xFFFFE000u);
  return rn_tf32(x - t);
}


template <int BN, int STAGES, bool kSplit>
struct GemmSmem {
  static constexpr int kA = kBM * kBK * 4;                          // 16 KB
  static constexpr int kB = BN * kBK * 4;
  static constexpr int kStage = kSplit ? 2 * kA + 2 * kB : kA + kB;  // A, W_hi (+ A_lo, W_lo)
  static constexpr int kBytes = STAGES * kStage + 1024 /*barriers*/ + 1024 /*alignment slack*/;
  static_assert(kBytes <= 227 * 1024, "shared memory plan exceeds 227 KB");
};

constexpr int kWarpProducer = 0, kWarpMma = 1, kWarpSplit0 = 2, kWarpEpi0 = 6;

}  // namespace

// Persistent: CTA b owns tiles b, b + gridDim.x, ...; tile t covers rows (t / num_n) * 128 and
// columns (t % num_n) * BN. The smem ring and the two TMEM accumulators are shared by all the
// CTA's tiles, so the epilogue of one tile runs while the next tile's K loop is in the tensor
// cores.
template <int BN, int STAGES, bool kSplit>
__global__ void __launch_bounds__(kThreads, 1) gemm_tf32_kernel(const __grid_constant__ CUtensorMap tmA,
                                                                const __grid_constant__ CUtensorMap tmWh,
                                                                const __grid_constant__ CUtensorMap tmWl,
                                                                float* __restrict__ C, const float* __restrict__ bias,
                                                                int M, int N, int K, int64_t ldc, int* err) {
  using L = GemmSmem<BN, STAGES, kSplit>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar_full = reinterpret_cast<uint64_t*>(smem + STAGES * L::kStage);
  uint64_t* bar_split = bar_full + STAGES;
  uint64_t* bar_empty = bar_split + STAGES;
  uint64_t* bar_acc_full = bar_empty + STAGES;   // [2]
  uint64_t* bar_acc_empty = bar_acc_full + 2;    // [2]
  uint64_t* bar_done = bar_acc_empty + 2;        // MMA completion on the abort path
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_n = N / BN;
  const int num_tiles = ((M + kBM - 1) / kBM) * num_n;
  const int num_k = (K + kBK - 1) / kBK;  // a ragged last K step reads zeros past K (TMA out-of-range fill)
  // stage layout: [A | W_hi | A_lo | W_lo], every tile 1024-byte aligned (128-byte swizzle atoms)
  auto stage_A = [&](int s) { return smem + s * L::kStage; };
  auto stage_Wh = [&](int s) { return smem + s * L::kStage + L::kA; };
  auto stage_Alo = [&](int s) { return smem + s * L::kStage + L::kA + L::kB; };
  auto stage_Wl = [&](int s) { return smem + s * L::kStage + 2 * L::kA + L::kB; };
  constexpr uint32_t kAccCols = BN < 32 ? 32 : BN;       // one accumulator
  constexpr uint32_t kTmemCols = 2 * kAccCols;             // double buffered (power of 2, >= 32)

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_split[s], 128);
      mbar_init(&bar_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bar_acc_full[b], 1);
      mbar_init(&bar_acc_empty[b], 128);
    }
    mbar_init(bar_done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kWarpMma) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == kWarpProducer) {
    // ---------------- TMA producer
    if (lane == 0) {
      const uint32_t bytes = L::kA + (kSplit ? 2 : 1) * L::kB;
      int it = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
        const int m0 = (tile / num_n) * kBM, n0 = (tile % num_n) * BN;
        for (int kt = 0; kt < num_k; ++kt, ++it) {
          const int s = it % STAGES;
          if (it >= STAGES && !mbar_wait(&bar_empty[s], ((it / STAGES) - 1) & 1, abort_flag, err, 1)) break;
          mbar_expect_tx(&bar_full[s], bytes);
          tma_load_2d(stage_A(s), &tmA, kt * kBK, m0, &bar_full[s]);
          tma_load_2d(stage_Wh(s), &tmWh, kt * kBK, n0, &bar_full[s]);
          if (kSplit) tma_load_2d(stage_Wl(s), &tmWl, kt * kBK, n0, &bar_full[s]);
        }
      }
      if (*abort_flag) {
        // let the copies this thread started land before the CTA can exit
        for (int j = it - 1; j >= 0 && j >= it - STAGES; --j) {
          for (uint32_t i = 0; i < kWaitLimit && !mbar_try(&bar_full[j % STAGES], (j / STAGES) & 1); ++i) {
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == kWarpMma) {
    // ---------------- MMA issuer (one thread)
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc_tf32<BN>();
      int it = 0, lt = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++lt) {
        const int b = lt & 1;
        if (lt >= 2 && !mbar_wait(&bar_acc_empty[b], ((lt >> 1) - 1) & 1, abort_flag, err, 5)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t acc_tmem = tmem + (uint32_t)(b * kAccCols);
        for (int kt = 0; kt < num_k; ++kt, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(kSplit ? &bar_split[s] : &bar_full[s], (it / STAGES) & 1, abort_flag, err, 2)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t a_hi = smem_u32(stage_A(s)), a_lo = smem_u32(stage_Alo(s));
          const uint32_t w_hi = smem_u32(stage_Wh(s)), w_lo = smem_u32(stage_Wl(s));
#pragma unroll
          for (int kk = 0; kk < kBK / 8; ++kk) {
            const uint32_t off = kk * 32;  // 8 tf32 = 32 bytes along K inside the swizzle row
            const uint32_t acc = (kt > 0 || kk > 0) ? 1u : 0u;
            mma_tf32(acc_tmem, smem_desc_sw128(a_hi + off), smem_desc_sw128(w_hi + off), idesc, acc);
            if (kSplit) {
              mma_tf32(acc_tmem, smem_desc_sw128(a_hi + off), smem_desc_sw128(w_lo + off), idesc, 1u);
              mma_tf32(acc_tmem, smem_desc_sw128(a_lo + off), smem_desc_sw128(w_hi + off), idesc, 1u);
            }
          }
          mma_commit(&bar_empty[s]);
        }
        if (ok) mma_commit(&bar_acc_full[b]);
      }
      // completion of every MMA issued above (also on the abort path) before TMEM is released
      mma_commit(bar_done);
      for (uint32_t i = 0; i < kWaitLimit && !mbar_try(bar_done, 0); ++i) {
      }
    }
    __syncwarp();
  } else if (warp < kWarpEpi0) {
    // ---------------- split (warps 2-5): A_lo = rn_tf32(a - trunc_tf32(a)). The tensor core reads
    // the raw fp32 A tile as TF32 by truncation, so the hi part needs no rewrite.
    if (kSplit) {
      const int t = threadIdx.x - kWarpSplit0 * 32;  // 0..127
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        for (int kt = 0; kt < num_k; ++kt, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(&bar_full[s], (it / STAGES) & 1, abort_flag, err, 3)) {
            ok = false;
            break;
          }
          const uint4* a = reinterpret_cast<const uint4*>(stage_A(s));
          uint4* alo = reinterpret_cast<uint4*>(stage_Alo(s));
#pragma unroll
          for (int i = 0; i < L::kA / 16 / 128; ++i) {
            const int c = i * 128 + t;
            const uint4 v = a[c];
            alo[c] = make_uint4(lo_part(v.x), lo_part(v.y), lo_part(v.z), lo_part(v.w));
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          mbar_arrive(&bar_split[s]);
        }
      }
    }
  } else {
    // ---------------- epilogue (warps 6-9): TMEM -> registers -> (+bias) -> global
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    int lt = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++lt) {
      const int b = lt & 1;
      bool ok = mbar_wait(&bar_acc_full[b], (lt >> 1) & 1, abort_flag, err, 4);
      ok = __all_sync(kFull, ok && !*abort_flag);  // tcgen05.ld is warp-collective: decide per warp
      if (!ok) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int m0 = (tile / num_n) * kBM, n0 = (tile % num_n) * BN;
      const int row = m0 + q * 32 + lane;
      const uint32_t taddr = tmem + (uint32_t)(b * kAccCols) + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 16) {
        uint32_t r[16];
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
              "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
            : "r"(taddr + (uint32_t)c0));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (row < M) {
          float* out = C + (int64_t)row * ldc + n0 + c0;
#pragma unroll
          for (int j = 0; j < 16; j += 4) {
            float4 v = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                                   __uint_as_float(r[j + 3]));
            if (bias) v = v + ld4_keep(bias + n0 + c0 + j);
            st4(out + j, v);
          }
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      mbar_arrive(&bar_acc_empty[b]);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == kWarpMma) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// ---- host side ------------------------------------------------------------------------------

namespace {

thread_local char g_map_err[160] = "";

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    void* p = nullptr;
    const cudaError_t st = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (st == cudaSuccess && q == cudaDriverEntryPointSuccess && p)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    else
      snprintf(g_map_err, sizeof(g_map_err), "cuTensorMapEncodeTiled entry point not found (cuda %d, query %d)",
               (int)st, (int)q);
  }
  return fn;
}

}  // namespace

// 2-D tensor map over rows x cols (cols contiguous, row stride ld_bytes), box box_cols x box_rows;
// out-of-range elements read as zero.
bool make_map_t(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, int64_t rows, int64_t cols,
                int64_t ld_bytes, int box_cols, int box_rows, CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld_bytes};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    snprintf(g_map_err, sizeof(g_map_err),
             "cuTensorMapEncodeTiled failed (CUresult %d) for base=%p rows=%lld cols=%lld ld=%lldB box=%dx%d", (int)r,
             base, (long long)rows, (long long)cols, (long long)ld_bytes, box_cols, box_rows);
    return false;
  }
  return true;
}

namespace {

// fp32 operand: box 32 x box_rows (128-byte rows), 128-byte swizzle.
bool make_map(CUtensorMap* map, const float* base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  return make_map_t(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, base, rows, cols, ld * 4, kBK, box_rows,
                    CU_TENSOR_MAP_SWIZZLE_128B);
}

template <int BN, int STAGES, bool kSplit>
cudaError_t launch(const CUtensorMap& a, const CUtensorMap& wh, const CUtensorMap& wl, float* C, const float* bias,
                   int M, int N, int K, int64_t ldc, int* err, cudaStream_t s) {
  using L = GemmSmem<BN, STAGES, kSplit>;
  auto kern = gemm_tf32_kernel<BN, STAGES, kSplit>;
  static thread_local uint64_t configured = 0;  // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured >> (dev & 63) & 1)) {
    cudaError_t st = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    if (st != cudaSuccess) return st;
    configured |= uint64_t(1) << (dev & 63);
  }
  const int tiles = ((M + kBM - 1) / kBM) * (N / BN);
  const int grid = tiles < sm_count() ? tiles : sm_count();
  kern<<<grid, kThreads, L::kBytes, s>>>(a, wh, wl, C, bias, M, N, K, ldc, err);
  return cudaGetLastError();
}

}  // namespace

// Returns 0 on success, -1 if the tensor maps could not be built, else a CUDA error code.
int launch_gemm_tf32(const float* A, int64_t lda, const float* W_hi, const float* W_lo, const float* bias, float* C,
                     int64_t ldc, int64_t M, int N, int K, bool split, int* err, cudaStream_t s) {
  const int BN = (N % 128 == 0) ? 128 : (N % 64 == 0) ? 64 : (N % 32 == 0) ? 32 : 16;
  CUtensorMap ma, mh, ml;
  if (!make_map(&ma, A, M, K, lda, kBM)) return -1;
  if (!make_map(&mh, W_hi, N, K, K, BN)) return -1;
  if (!make_map(&ml, split ? W_lo : W_hi, N, K, K, BN)) return -1;
  cudaError_t st;
  const int m = (int)M;
  switch (BN) {
    case 128:
      st = split ? launch<128, 3, true>(ma, mh, ml, C, bias, m, N, K, ldc, err, s)
                 : launch<128, 4, false>(ma, mh, ml, C, bias, m, N, K, ldc, err, s);
      break;
    case 64:
      st = split ? launch<64, 4, true>(ma, mh, ml, C, bias, m, N, K, ldc, err, s)
                 : launch<64, 4, false>(ma, mh, ml, C, bias, m, N, K, ldc, err, s);
      break;
    case 32:
      st = split ? launch<32, 4, true>(ma, mh, ml, C, bias, m, N, K, ldc, err, s)
                 : launch<32, 4, false>(ma, mh, ml, C, bias, m, N, K, ldc, err, s);
      break;
    default:
      st = split ? launch<16, 4, true>(ma, mh, ml, C, bias, m, N, K, ldc, err, s)
                 : launch<16, 4, false>(ma, mh, ml, C, bias, m, N, K, ldc, err, s);
  }
  return st == cudaSuccess ? 0 : (int)st;
}

// hi = x rounded to TF32, lo = (x - hi) rounded to TF32 (see split_rn).
__global__ void split_tf32_kernel(const float* __restrict__ x, float* __restrict__ hi, float* __restrict__ lo,
                                  int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    uint32_t h, l;
    split_rn(__float_as_uint(x[i]), h, l);
    hi[i] = __uint_as_float(h);
    lo[i] = __uint_as_float(l);
  }
}

const char* gemm_map_error() { return g_map_err; }

void launch_split_tf32(const float* x, float* hi, float* lo, int64_t n, cudaStream_t s) {
  split_tf32_kernel<<<grid_for(n, 256, 4), 256, 0, s>>>(x, hi, lo, n);
}

}  // namespace fuma
