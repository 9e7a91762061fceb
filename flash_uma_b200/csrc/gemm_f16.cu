// Dense contraction C[M,N] = A[M,K] . W[N,K]^T (+ bias[N]) on the tcgen05 tensor cores in
// kind::f16 (fp16 operands, fp32 accumulation) with fp32-level accuracy: the "f16x3" split.
//
// Same role as the kind::tf32 kernel of gemm.cu (the reference's F.linear calls of the radial
// MLP and SO(2) convolutions, model.py:147-154, and their input-gradient GEMMs), at half the
// operand bytes per K: fp16 moves 2 bytes per element where TF32 moves 4, and the fp16 MMA
// covers K=16 per instruction at twice the TF32 rate. Operand traffic through shared memory,
// not the MMA count, bounds these GEMMs, so this roughly halves their time.
//
// Split (the scaled-residual scheme of Ootomo & Yokota, "Recovering single precision accuracy
// from Tensor Cores while surpassing the FP32 theoretical peak performance", IJHPCA 2022):
//   x = hi + lo * 2^-11,  hi = fp16_rn(x),  lo = fp16_rn((x - hi) * 2^11)
// for both operands (weights prepared once by split_f16_kernel; activations split in shared
// memory by the kernel). Scaling the residual by 2^11 keeps lo a normal fp16 number, so the
// pair carries ~22 significant bits for |x| from 2^-14 up to the fp16 limit and an absolute
// error below 2^-36 under it. Two fp32 TMEM accumulators per tile:
//   main  += A_hi . W_hi
//   cross += A_hi . W_lo + A_lo . W_hi
// and the epilogue forms (main + cross * 2^-11) * w_scale_inv + bias. The dropped lo.lo term
// is ~2^-22 relative. Keeping the cross terms in their own accumulator means only one
// truncating accumulation per K=16 step lands on the full-size sum.
//
// Range: an activation whose magnitude rounds beyond the fp16 maximum (|x| >= 65520) cannot be
// split; the kernel then records kErrRange in *err (the caller raises) - use the TF32 kernels
// for such data. Weights are pre-scaled by a power of two (w_scale_inv undoes it) so they never
// overflow.
//
// Structure (persistent, one CTA per SM, 320 threads, 128 x BN output tiles):
//   warp 0      TMA producer: raw fp32 A tile [128 x 32] (128-byte swizzle) and fp16 W_hi,
//               W_lo tiles [BN x 32] (64-byte swizzle) into a STAGES-deep ring.
//   warp 1      allocates 4 x BN TMEM columns (main + cross, double buffered); lane 0 issues
//               tcgen05.mma kind::f16 (M=128, N=BN, K=16) and the commits.
//   warps 2-5   split the raw A tile into A_hi / A_lo (fp16, 64-byte swizzle) next to it.
//   warps 6-9   epilogue of the other accumulator pair while the next tile's K loop runs.
// Every mbarrier wait is bounded (the error protocol of gemm.cu).
#include <cstdio>
#include <cstdlib>

#include <cuda.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace fuma {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 32;           // K elements per stage: raw fp32 A rows are 128 B, fp16 rows 64 B
constexpr int kThreads = 320;
constexpr int kWarpProducer = 0, kWarpMma = 1, kWarpSplit0 = 2, kWarpEpi0 = 6;
constexpr float kLoScaleInv = 1.0f / kSplitLoScale;

// kPre: A arrives pre-split (row-packed hi | lo fp16, see split_rows_f16_kernel), so a stage
// holds no raw fp32 tile and no split work is done in the kernel.
// kX3 = false (pre-split A only): the single-product mode, main += A_hi . W_hi; the lo halves
// are neither loaded nor multiplied (fp16 operand precision, the accuracy class of TF32).
template <int BN, int STAGES, bool kPre, bool kX3 = true>
struct F16Smem {
  static constexpr int kRaw = kPre ? 0 : kBM * kBK * 4;   // 16 KB fp32 A, 128-byte swizzle
  static constexpr int kA16 = kBM * kBK * 2;   // 8 KB fp16 A half, 64-byte swizzle
  static constexpr int kW16 = BN * kBK * 2;    // fp16 W half, 64-byte swizzle
  static constexpr int kHalves = kX3 ? 2 : 1;  // hi (+ lo) tiles of each operand per stage
  static constexpr int kStage = kRaw + kHalves * kA16 + kHalves * kW16;
  // epilogue staging for the TMA store: per epilogue warp two [32 rows x 32 fp32] boxes
  static constexpr bool kTmaStore = BN >= 32;
  static constexpr int kStaging = kTmaStore ? 4 * 2 * 4096 : 0;
  static constexpr int kBytes = STAGES * kStage + kStaging + 1024 /*barriers*/ + 1024 /*alignment slack*/;
  static_assert(kBytes <= 227 * 1024, "shared memory plan exceeds 227 KB");
  static_assert(kW16 % 512 == 0, "fp16 tiles must stay aligned to the 512-byte swizzle atom");
};

// K-major operand, 64-byte swizzle: 8-row groups 512 B apart.
__device__ __forceinline__ uint64_t smem_desc_sw64(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);   // start address
  d |= (uint64_t)1u << 16;                   // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(512u >> 4) << 32;          // stride byte offset: 8 rows x 64 B
  d |= (uint64_t)1u << 46;                   // descriptor version (sm100)
  d |= (uint64_t)4u << 61;                   // layout: SWIZZLE_64B
  return d;
}

// kind::f16 instruction descriptor: fp16 A and B (format 0), fp32 accumulator, K-major, M=128.
template <int BN>
__device__ __forceinline__ constexpr uint32_t instr_desc_f16() {
  return (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// TMA tile store shared -> global (bulk async-group completion).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(smem_u32(src))
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

}  // namespace

// kOutHalf (single-product mode only): C is fp16 [M, ldc] (the 16-bit activation storage of
// the "f16" mode), written through [32 x 32] fp16 boxes with a 64-byte swizzle; a finite result
// at or beyond the fp16 limit records kErrRange.
template <int BN, int STAGES, bool kPre, bool kX3, bool kOutHalf = false>
__global__ void __launch_bounds__(kThreads, 1) gemm_f16x3_kernel(const __grid_constant__ CUtensorMap tmA,
                                                                 const __grid_constant__ CUtensorMap tmAl,
                                                                 const __grid_constant__ CUtensorMap tmWh,
                                                                 const __grid_constant__ CUtensorMap tmWl,
                                                                 const __grid_constant__ CUtensorMap tmC,
                                                                 float* __restrict__ C, const float* __restrict__ bias,
                                                                 float w_scale_inv, int M, int N, int K, int64_t ldc,
                                                                 int* err) {
  static_assert(kX3 || kPre, "the single-product mode takes pre-split operands");
  static_assert(!kOutHalf || !kX3, "fp16 results belong to the single-product mode");
  using L = F16Smem<BN, STAGES, kPre, kX3>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_c = smem + STAGES * L::kStage;   // epilogue staging (TMA store path)
  uint64_t* bar_full = reinterpret_cast<uint64_t*>(smem_c + L::kStaging);
  uint64_t* bar_split = bar_full + STAGES;
  uint64_t* bar_empty = bar_split + STAGES;
  uint64_t* bar_acc_full = bar_empty + STAGES;   // [2]
  uint64_t* bar_acc_empty = bar_acc_full + 2;    // [2]
  uint64_t* bar_done = bar_acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_n = N / BN;
  const int num_tiles = ((M + kBM - 1) / kBM) * num_n;
  const int num_k = (K + kBK - 1) / kBK;
  // stage layout: [raw A | A_hi | A_lo | W_hi | W_lo] (no lo tiles in the single-product mode)
  constexpr int kH = L::kHalves;
  auto stage_raw = [&](int s) { return smem + s * L::kStage; };
  auto stage_Ah = [&](int s) { return smem + s * L::kStage + L::kRaw; };
  auto stage_Al = [&](int s) { return smem + s * L::kStage + L::kRaw + L::kA16; };
  auto stage_Wh = [&](int s) { return smem + s * L::kStage + L::kRaw + kH * L::kA16; };
  auto stage_Wl = [&](int s) { return smem + s * L::kStage + L::kRaw + kH * L::kA16 + L::kW16; };
  constexpr uint32_t kBufCols = kX3 ? 2 * BN : BN;       // main (+ cross) of one buffer
  constexpr int kAcc = kBufCols <= 256 ? 2 : 1;          // accumulator buffers (TMEM holds 512 columns)
  constexpr uint32_t kTmemCols = kAcc * kBufCols;  // 64..512, a power of 2

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
    if (lane == 0) {
      constexpr uint32_t bytes = (kPre ? kH * L::kA16 : L::kRaw) + kH * L::kW16;
      int it = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
        const int m0 = (tile / num_n) * kBM, n0 = (tile % num_n) * BN;
        for (int kt = 0; kt < num_k; ++kt, ++it) {
          const int s = it % STAGES;
          if (it >= STAGES && !mbar_wait(&bar_empty[s], ((it / STAGES) - 1) & 1, abort_flag, err, kErrWaitEmpty))
            break;
          mbar_expect_tx(&bar_full[s], bytes);
          if (kPre) {
            tma_load_2d(stage_Ah(s), &tmA, kt * kBK, m0, &bar_full[s]);
            if (kX3) tma_load_2d(stage_Al(s), &tmAl, kt * kBK, m0, &bar_full[s]);
          } else {
            tma_load_2d(stage_raw(s), &tmA, kt * kBK, m0, &bar_full[s]);
          }
          tma_load_2d(stage_Wh(s), &tmWh, kt * kBK, n0, &bar_full[s]);
          if (kX3) tma_load_2d(stage_Wl(s), &tmWl, kt * kBK, n0, &bar_full[s]);
        }
      }
      if (*abort_flag) {
        for (int j = it - 1; j >= 0 && j >= it - STAGES; --j) {
          for (uint32_t i = 0; i < kWaitLimit && !mbar_try(&bar_full[j % STAGES], (j / STAGES) & 1); ++i) {
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == kWarpMma) {
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc_f16<BN>();
      int it = 0, lt = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++lt) {
        const int b = kAcc == 2 ? (lt & 1) : 0;
        if (lt >= kAcc && !mbar_wait(&bar_acc_empty[b], ((lt / kAcc) - 1) & 1, abort_flag, err, kErrWaitAccEmpty))
          break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t acc_main = tmem + (uint32_t)(b * kBufCols);
        const uint32_t acc_cross = acc_main + (uint32_t)BN;
        for (int kt = 0; kt < num_k; ++kt, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(kPre ? &bar_full[s] : &bar_split[s], (it / STAGES) & 1, abort_flag, err, kErrWaitSplit)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t a_hi = smem_u32(stage_Ah(s)), a_lo = smem_u32(stage_Al(s));
          const uint32_t w_hi = smem_u32(stage_Wh(s)), w_lo = smem_u32(stage_Wl(s));
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint32_t off = kk * 32;  // 16 fp16 = 32 bytes along K inside the 64-byte swizzle row
            const uint32_t acc = (kt > 0 || kk > 0) ? 1u : 0u;
            mma_f16(acc_main, smem_desc_sw64(a_hi + off), smem_desc_sw64(w_hi + off), idesc, acc);
            if constexpr (kX3) {
              mma_f16(acc_cross, smem_desc_sw64(a_hi + off), smem_desc_sw64(w_lo + off), idesc, acc);
              mma_f16(acc_cross, smem_desc_sw64(a_lo + off), smem_desc_sw64(w_hi + off), idesc, 1u);
            }
          }
          mma_commit(&bar_empty[s]);
        }
        if (ok) mma_commit(&bar_acc_full[b]);
      }
      mma_commit(bar_done);
      for (uint32_t i = 0; i < kWaitLimit && !mbar_try(bar_done, 0); ++i) {
      }
    }
    __syncwarp();
  } else if (warp < kWarpEpi0) {
    if constexpr (!kPre) {
      // ---------------- split (warps 2-5): raw fp32 [128 x 32] (128-byte swizzle: logical 16-byte
      // chunk j of row r sits at chunk j ^ (r & 7)) -> A_hi, A_lo fp16 [128 x 32] (64-byte swizzle:
      // logical chunk j of row r at chunk j ^ ((r >> 1) & 3)). Thread t converts float chunks
      // (row i*16 + t/8, chunk t%8), i = 0..7: 4 floats -> 8 bytes of A_hi and of A_lo.
      const int t = threadIdx.x - kWarpSplit0 * 32;  // 0..127
      const int j = t & 7;
      int it = 0;
      bool ok = true, bad = false;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        for (int kt = 0; kt < num_k; ++kt, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(&bar_full[s], (it / STAGES) & 1, abort_flag, err, kErrWaitFull)) {
            ok = false;
            break;
          }
          const uint8_t* raw = stage_raw(s);
          uint8_t* ah = stage_Ah(s);
          uint8_t* al = stage_Al(s);
  #pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = i * 16 + (t >> 3);
            const float4 v = *reinterpret_cast<const float4*>(raw + r * 128 + ((j ^ (r & 7)) << 4));
            uint2 hi, lo;
            split_f16x4(v, hi, lo, bad);
            const int off = r * 64 + (((j >> 1) ^ ((r >> 1) & 3)) << 4) + ((j & 1) << 3);
            *reinterpret_cast<uint2*>(ah + off) = hi;
            *reinterpret_cast<uint2*>(al + off) = lo;
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          mbar_arrive(&bar_split[s]);
        }
      }
      if (bad && err) atomicCAS(err, 0, (int)kErrRange);
    }
  } else {
    // ---------------- epilogue (warps 6-9)
    const int q = warp & 3;
    int lt = 0, nbox = 0;
    bool out_bad = false;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++lt) {
      const int b = kAcc == 2 ? (lt & 1) : 0;
      bool ok = mbar_wait(&bar_acc_full[b], (lt / kAcc) & 1, abort_flag, err, kErrWaitAcc);
      ok = __all_sync(kFull, ok && !*abort_flag);
      if (!ok) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int m0 = (tile / num_n) * kBM, n0 = (tile % num_n) * BN;
      const uint32_t taddr = tmem + (uint32_t)(b * kBufCols) + ((uint32_t)(q * 32) << 16);
      if constexpr (L::kTmaStore) {
        // 32-column chunks, lane = row of this warp's 32-row quadrant. The row's 32 results go
        // to a [32 x 32] fp32 staging box (128-byte swizzle: 16-byte chunk j of row r at
        // j ^ (r & 7), conflict-free) that one TMA store writes out; rows beyond M are clipped
        // by the tensor map. Two boxes per warp alternate, so the next chunk's TMEM loads and
        // arithmetic overlap the previous store.
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 32) {
          uint32_t rm[32], rc[32];
          tmem_ld32(taddr + (uint32_t)c0, rm);
          if constexpr (kX3) tmem_ld32(taddr + (uint32_t)(BN + c0), rc);
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
          if constexpr (!kX3) {
#pragma unroll
            for (int u = 0; u < 32; ++u) rc[u] = 0u;
          }
          uint8_t* box = smem_c + (q * 2 + (nbox & 1)) * 4096;
          if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
          __syncwarp();
          if constexpr (kOutHalf) {
            // row = lane, 64 bytes (32 halves); 16-byte chunk j of row r at j ^ ((r >> 1) & 3)
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              uint32_t h[4];
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const int c = 8 * jj + 2 * u;
                float a = __uint_as_float(rm[c]) * w_scale_inv, b = __uint_as_float(rm[c + 1]) * w_scale_inv;
                if (bias) {
                  a += bias[n0 + c0 + c];
                  b += bias[n0 + c0 + c + 1];
                }
                const float m = fmaxf(fabsf(a), fabsf(b));
                out_bad |= (m >= 65520.0f) & (m <= 3.402823466e38f);
                h[u] = h2_bits(__floats2half2_rn(a, b));
              }
              *reinterpret_cast<uint4*>(box + lane * 64 + ((jj ^ ((lane >> 1) & 3)) << 4)) =
                  make_uint4(h[0], h[1], h[2], h[3]);
            }
          } else {
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
              float o[4];
#pragma unroll
              for (int u = 0; u < 4; ++u)
                o[u] = fmaf(__uint_as_float(rc[4 * jj + u]), kLoScaleInv, __uint_as_float(rm[4 * jj + u])) * w_scale_inv;
              float4 v = make_float4(o[0], o[1], o[2], o[3]);
              if (bias) v = v + ld4_keep(bias + n0 + c0 + 4 * jj);
              *reinterpret_cast<float4*>(box + lane * 128 + ((jj ^ (lane & 7)) << 4)) = v;
            }
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, box, n0 + c0, m0 + q * 32);
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          }
          ++nbox;
        }
      } else {
        const int row = m0 + q * 32 + lane;
  #pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          uint32_t rm[16], rc[16];
          tmem_ld16(taddr + (uint32_t)c0, rm);
          if constexpr (kX3) tmem_ld16(taddr + (uint32_t)(BN + c0), rc);
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
          if constexpr (!kX3) {
#pragma unroll
            for (int u = 0; u < 16; ++u) rc[u] = 0u;
          }
          if (row < M) {
  #pragma unroll
            for (int jj = 0; jj < 16; jj += 4) {
              float o[4];
  #pragma unroll
              for (int u = 0; u < 4; ++u)
                o[u] = fmaf(__uint_as_float(rc[jj + u]), kLoScaleInv, __uint_as_float(rm[jj + u])) * w_scale_inv;
              float4 v = make_float4(o[0], o[1], o[2], o[3]);
              if (bias) v = v + ld4_keep(bias + n0 + c0 + jj);
              if constexpr (kOutHalf) {
                const float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
                out_bad |= (m >= 65520.0f) & (m <= 3.402823466e38f);
                __half* out = reinterpret_cast<__half*>(C) + (int64_t)row * ldc + n0 + c0 + jj;
                *reinterpret_cast<uint2*>(out) =
                    make_uint2(h2_bits(__floats2half2_rn(v.x, v.y)), h2_bits(__floats2half2_rn(v.z, v.w)));
              } else {
                st4(C + (int64_t)row * ldc + n0 + c0 + jj, v);
              }
            }
          }
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      mbar_arrive(&bar_acc_empty[b]);
    }
    if constexpr (L::kTmaStore) {
      // the staging boxes must stay alive (and the results land) before the CTA exits
      if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
      __syncwarp();
    }
    if (kOutHalf && out_bad && err) atomicCAS(err, 0, (int)kErrRange);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == kWarpMma) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// Transposed tiles: D[f, e] = sum_k W[f, k] A[e, k] with the 128 output features f of a tile on
// the MMA's M side and 256 edges e on its N side (tcgen05 M=128, N=256), for output widths that
// are a multiple of 128 but not of 256 (or K below the 256-wide threshold): those shapes
// otherwise run 128-wide tiles,
// whose per-instruction operand traffic (A and W tiles of equal size for half the products)
// keeps the tensor pipe near two thirds of its rate. Same f16x3 arithmetic as
// gemm_f16x3_kernel (main += W_hi A_hi, cross += W_lo A_hi + W_hi A_lo, one pre-split operand
// format); the epilogue transposes through the staging boxes: the TMEM lane of a thread is an
// output feature, its registers run over edges, and each [32 edges x 32 features] box goes out
// with one TMA store. One accumulator pair fills TMEM, so the epilogue is not overlapped.
constexpr int kTF = 128;   // output features per tile (MMA M)
constexpr int kTE = 256;   // edges per tile (MMA N)

template <int STAGES, bool kX3>
struct F16TSmem {
  static constexpr int kW16 = kTF * kBK * 2;   // 8 KB
  static constexpr int kA16 = kTE * kBK * 2;   // 16 KB
  static constexpr int kStage = kX3 ? 2 * kW16 + 2 * kA16 : kW16 + kA16;   // the single product loads hi only
  static constexpr int kStaging = 4 * 2 * 4096;
  static constexpr int kBytes = STAGES * kStage + kStaging + 1024 + 1024;
  static_assert(kBytes <= 227 * 1024, "shared memory plan exceeds 227 KB");
};

// kX3 = false: the single-product mode (main += W_hi A_hi): one 256-column accumulator per tile,
// so two of them fill TMEM and the epilogue of one tile overlaps the MMAs of the next; with
// kOutHalf the results are stored as fp16 (64-byte [32 edges x 32 features] boxes).
template <int STAGES, bool kX3, bool kOutHalf>
__global__ void __launch_bounds__(kThreads, 1) gemm_f16x3_t_kernel(const __grid_constant__ CUtensorMap tmA,
                                                                   const __grid_constant__ CUtensorMap tmAl,
                                                                   const __grid_constant__ CUtensorMap tmWh,
                                                                   const __grid_constant__ CUtensorMap tmWl,
                                                                   const __grid_constant__ CUtensorMap tmC,
                                                                   const float* __restrict__ bias, float w_scale_inv,
                                                                   int M, int N, int K, int* err) {
  static_assert(!kOutHalf || !kX3, "fp16 results belong to the single-product mode");
  using L = F16TSmem<STAGES, kX3>;
  constexpr int kAcc = kX3 ? 1 : 2;   // accumulator buffers: main + cross, or two mains
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_c = smem + STAGES * L::kStage;
  uint64_t* bar_full = reinterpret_cast<uint64_t*>(smem_c + L::kStaging);
  uint64_t* bar_empty = bar_full + STAGES;
  uint64_t* bar_acc_full = bar_empty + STAGES;    // [kAcc]
  uint64_t* bar_acc_empty = bar_acc_full + 2;     // [kAcc]
  uint64_t* bar_done = bar_acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_f = N / kTF;
  const int num_tiles = ((M + kTE - 1) / kTE) * num_f;
  const int num_k = (K + kBK - 1) / kBK;
  // stage layout: [W_hi | W_lo | A_hi | A_lo] (f16x3) or [W_hi | A_hi] (single product)
  auto stage_Wh = [&](int s) { return smem + s * L::kStage; };
  auto stage_Wl = [&](int s) { return smem + s * L::kStage + L::kW16; };
  auto stage_Ah = [&](int s) { return smem + s * L::kStage + (kX3 ? 2 : 1) * L::kW16; };
  auto stage_Al = [&](int s) { return smem + s * L::kStage + 2 * L::kW16 + L::kA16; };
  constexpr uint32_t kTmemCols = 2 * kTE;   // main + cross, or two mains

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    for (int b = 0; b < kAcc; ++b) {
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
    if (lane == 0) {
      constexpr uint32_t bytes = L::kStage;
      int it = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
        const int e0 = (tile / num_f) * kTE, f0 = (tile % num_f) * kTF;
        for (int kt = 0; kt < num_k; ++kt, ++it) {
          const int s = it % STAGES;
          if (it >= STAGES && !mbar_wait(&bar_empty[s], ((it / STAGES) - 1) & 1, abort_flag, err, kErrWaitEmpty))
            break;
          mbar_expect_tx(&bar_full[s], bytes);
          tma_load_2d(stage_Wh(s), &tmWh, kt * kBK, f0, &bar_full[s]);
          if constexpr (kX3) tma_load_2d(stage_Wl(s), &tmWl, kt * kBK, f0, &bar_full[s]);
          tma_load_2d(stage_Ah(s), &tmA, kt * kBK, e0, &bar_full[s]);
          if constexpr (kX3) tma_load_2d(stage_Al(s), &tmAl, kt * kBK, e0, &bar_full[s]);
        }
      }
      if (*abort_flag) {
        for (int j = it - 1; j >= 0 && j >= it - STAGES; --j) {
          for (uint32_t i = 0; i < kWaitLimit && !mbar_try(&bar_full[j % STAGES], (j / STAGES) & 1); ++i) {
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == kWarpMma) {
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc_f16<kTE>();   // M = 128, N = 256
      int it = 0, lt = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++lt) {
        const int b = kAcc == 2 ? (lt & 1) : 0;
        if (lt >= kAcc && !mbar_wait(&bar_acc_empty[b], ((lt / kAcc) - 1) & 1, abort_flag, err, kErrWaitAccEmpty))
          break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t acc_main = tmem + (uint32_t)(b * kTE), acc_cross = tmem + (uint32_t)kTE;
        for (int kt = 0; kt < num_k; ++kt, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(&bar_full[s], (it / STAGES) & 1, abort_flag, err, kErrWaitFull)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t w_hi = smem_u32(stage_Wh(s)), a_hi = smem_u32(stage_Ah(s));
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint32_t off = kk * 32;
            const uint32_t acc = (kt > 0 || kk > 0) ? 1u : 0u;
            mma_f16(acc_main, smem_desc_sw64(w_hi + off), smem_desc_sw64(a_hi + off), idesc, acc);
            if constexpr (kX3) {
              const uint32_t w_lo = smem_u32(stage_Wl(s)), a_lo = smem_u32(stage_Al(s));
              mma_f16(acc_cross, smem_desc_sw64(w_lo + off), smem_desc_sw64(a_hi + off), idesc, acc);
              mma_f16(acc_cross, smem_desc_sw64(w_hi + off), smem_desc_sw64(a_lo + off), idesc, 1u);
            }
          }
          mma_commit(&bar_empty[s]);
        }
        if (ok) mma_commit(&bar_acc_full[b]);
      }
      mma_commit(bar_done);
      for (uint32_t i = 0; i < kWaitLimit && !mbar_try(bar_done, 0); ++i) {
      }
    }
    __syncwarp();
  } else if (warp >= kWarpEpi0) {
    // epilogue (warps 6-9): TMEM lane quadrant q = output features f0 + 32q .. f0 + 32q + 31
    const int q = warp & 3;
    int lt = 0, nbox = 0;
    bool out_bad = false;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++lt) {
      const int b = kAcc == 2 ? (lt & 1) : 0;
      bool ok = mbar_wait(&bar_acc_full[b], (lt / kAcc) & 1, abort_flag, err, kErrWaitAcc);
      ok = __all_sync(kFull, ok && !*abort_flag);
      if (!ok) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int e0 = (tile / num_f) * kTE, f0 = (tile % num_f) * kTF;
      const uint32_t taddr = tmem + (uint32_t)(b * kTE) + ((uint32_t)(q * 32) << 16);
      const float bv = bias ? bias[f0 + q * 32 + lane] : 0.0f;
#pragma unroll 1
      for (int c0 = 0; c0 < kTE; c0 += 32) {
        if (e0 + c0 >= M) break;   // whole box beyond the last edge
        uint32_t rm[32], rc[32];
        tmem_ld32(taddr + (uint32_t)c0, rm);
        if constexpr (kX3) tmem_ld32(taddr + (uint32_t)(kTE + c0), rc);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if constexpr (!kX3) {
#pragma unroll
          for (int u = 0; u < 32; ++u) rc[u] = 0u;
        }
        uint8_t* box = smem_c + (q * 2 + (nbox & 1)) * 4096;
        if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
        __syncwarp();
        if constexpr (kOutHalf) {
          // box row j = edge e0 + c0 + j (64 bytes = 32 fp16 features), 64-byte swizzle: 16-byte
          // chunk (lane / 8) of row j at chunk (lane / 8) ^ ((j >> 1) & 3); two lanes share a word
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float v = __uint_as_float(rm[j]) * w_scale_inv + bv;
            out_bad |= (fabsf(v) >= 65520.0f) & (fabsf(v) <= 3.402823466e38f);
            *reinterpret_cast<__half*>(box + j * 64 + (((lane >> 3) ^ ((j >> 1) & 3)) << 4) + ((lane & 7) << 1)) =
                __float2half_rn(v);
          }
        } else {
          // box row j = edge e0 + c0 + j (128 bytes = 32 features), 128-byte swizzle: 16-byte chunk
          // (lane / 4) of row j at chunk (lane / 4) ^ (j & 7); one row per store instruction
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float v = fmaf(__uint_as_float(rc[j]), kLoScaleInv, __uint_as_float(rm[j])) * w_scale_inv + bv;
            *reinterpret_cast<float*>(box + j * 128 + ((((lane >> 2) ^ (j & 7))) << 4) + ((lane & 3) << 2)) = v;
          }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmC, box, f0 + q * 32, e0 + c0);
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
        ++nbox;
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      mbar_arrive(&bar_acc_empty[b]);
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    __syncwarp();
    if (kOutHalf && out_bad && err) atomicCAS(err, 0, (int)kErrRange);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == kWarpMma) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

namespace {

template <int BN, int STAGES, bool kPre, bool kX3, bool kOutHalf = false>
cudaError_t launch_f16(const CUtensorMap& a, const CUtensorMap& al, const CUtensorMap& wh, const CUtensorMap& wl,
                       const CUtensorMap& mc, float* C, const float* bias, float w_scale_inv, int M, int N, int K, int64_t ldc, int* err,
                       cudaStream_t s) {
  using L = F16Smem<BN, STAGES, kPre, kX3>;
  auto kern = gemm_f16x3_kernel<BN, STAGES, kPre, kX3, kOutHalf>;
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
  kern<<<grid, kThreads, L::kBytes, s>>>(a, al, wh, wl, mc, C, bias, w_scale_inv, M, N, K, ldc, err);
  return cudaGetLastError();
}

template <bool kPre>
cudaError_t launch_bn(int BN, const CUtensorMap& a, const CUtensorMap& al, const CUtensorMap& wh,
                      const CUtensorMap& wl, const CUtensorMap& mc, float* C, const float* bias, float inv, int M, int N, int K,
                      int64_t ldc, int* err, cudaStream_t s) {
  switch (BN) {
    case 256: return launch_f16<256, kPre ? 4 : 3, kPre, true>(a, al, wh, wl, mc, C, bias, inv, M, N, K, ldc, err, s);
    case 128: return launch_f16<128, kPre ? 5 : 4, kPre, true>(a, al, wh, wl, mc, C, bias, inv, M, N, K, ldc, err, s);
    case 64: return launch_f16<64, kPre ? 6 : 4, kPre, true>(a, al, wh, wl, mc, C, bias, inv, M, N, K, ldc, err, s);
    case 32: return launch_f16<32, kPre ? 8 : 5, kPre, true>(a, al, wh, wl, mc, C, bias, inv, M, N, K, ldc, err, s);
    default: return launch_f16<16, kPre ? 8 : 6, kPre, true>(a, al, wh, wl, mc, C, bias, inv, M, N, K, ldc, err, s);
  }
}

template <int STAGES, bool kX3, bool kOutHalf>
cudaError_t launch_f16_t(const CUtensorMap& a, const CUtensorMap& al, const CUtensorMap& wh, const CUtensorMap& wl,
                         const CUtensorMap& mc, const float* bias, float w_scale_inv, int M, int N, int K, int* err,
                         cudaStream_t s) {
  using L = F16TSmem<STAGES, kX3>;
  auto kern = gemm_f16x3_t_kernel<STAGES, kX3, kOutHalf>;
  static thread_local uint64_t configured = 0;  // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured >> (dev & 63) & 1)) {
    cudaError_t st = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    if (st != cudaSuccess) return st;
    configured |= uint64_t(1) << (dev & 63);
  }
  const int tiles = ((M + kTE - 1) / kTE) * (N / kTF);
  const int grid = tiles < sm_count() ? tiles : sm_count();
  kern<<<grid, kThreads, L::kBytes, s>>>(a, al, wh, wl, mc, bias, w_scale_inv, M, N, K, err);
  return cudaGetLastError();
}

// single-product mode (pre-split A): half the operand bytes per stage, so deeper rings
template <bool kOutHalf>
cudaError_t launch_bn_x1(int BN, const CUtensorMap& a, const CUtensorMap& wh, const CUtensorMap& mc, float* C,
                         const float* bias, float inv, int M, int N, int K, int64_t ldc, int* err, cudaStream_t s) {
  switch (BN) {
    case 256: return launch_f16<256, 8, true, false, kOutHalf>(a, a, wh, wh, mc, C, bias, inv, M, N, K, ldc, err, s);
    case 128: return launch_f16<128, 8, true, false, kOutHalf>(a, a, wh, wh, mc, C, bias, inv, M, N, K, ldc, err, s);
    case 64: return launch_f16<64, 8, true, false, kOutHalf>(a, a, wh, wh, mc, C, bias, inv, M, N, K, ldc, err, s);
    case 32: return launch_f16<32, 8, true, false, kOutHalf>(a, a, wh, wh, mc, C, bias, inv, M, N, K, ldc, err, s);
    default: return launch_f16<16, 8, true, false, kOutHalf>(a, a, wh, wh, mc, C, bias, inv, M, N, K, ldc, err, s);
  }
}

}  // namespace

// 256-wide tiles for N % 256 == 0 and K >= this. They hold one TMEM accumulator pair (the
// epilogue is not overlapped with the next tile) but halve the A-operand traffic per FLOP:
// measured on B200 with pre-split A, M = 120,000: K = 1024, N = 512: 0.356 -> 0.287 ms;
// K = 512, N = 512: 0.189 -> 0.156 ms; K = 256, N = 256: 0.059 -> 0.066 ms (slower).
// FUMA_BN256_MIN_K overrides the default.
const int g_bn256_min_k = [] {
  const char* e = getenv("FUMA_BN256_MIN_K");
  return e ? atoi(e) : 512;
}();

// Transposed 128 x 256 tiles (gemm_f16x3_t_kernel) for pre-split products (f16x3 and single
// product) whose N is a multiple of 128 that would otherwise run 128-wide tiles, when K >= 384: measured on B200 at
// M = 120,000, K = 768, N = 640 0.346 -> 0.290 ms, K = 384, N = 384 0.116 -> 0.109 ms,
// K = 1536, N = 128 0.179 -> 0.169 ms; shorter K is faster with the double-buffered 128-wide
// tiles (K = 128: 0.027 -> 0.031 ms). FUMA_GEMM_T=0 / 1 forces them off / on for every
// eligible shape (read at every call).
bool use_t(int K) {
  const char* e = getenv("FUMA_GEMM_T");
  if (e) return atoi(e) != 0;
  return K >= 384;
}

int launch_gemm_f16x3(const float* A, int64_t lda, bool a_split, const void* W_hi, const void* W_lo, int64_t ldw,
                      float w_scale_inv, const float* bias, float* C, int64_t ldc, int64_t M, int N, int K, int* err,
                      cudaStream_t s, bool x1, bool out_half) {
  // single-product mode: one accumulator, so 256-wide tiles stay double-buffered at any K
  const int BN = (N % 256 == 0 && (x1 || K >= g_bn256_min_k)) ? 256
                 : (N % 128 == 0) ? 128 : (N % 64 == 0) ? 64 : (N % 32 == 0) ? 32 : 16;
  CUtensorMap ma, mal, mh, ml;
  if (a_split && !x1 && BN == 128 && N % 128 == 0 && use_t(K)) {
    const uint8_t* base = reinterpret_cast<const uint8_t*>(A);
    if (!make_map_t(&ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, base, M, K, lda * 4, kBK, kTE, CU_TENSOR_MAP_SWIZZLE_64B) ||
        !make_map_t(&mal, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, base + lda * 2, M, K, lda * 4, kBK, kTE,
                    CU_TENSOR_MAP_SWIZZLE_64B) ||
        !make_map_t(&mh, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, W_hi, N, K, ldw * 2, kBK, kTF, CU_TENSOR_MAP_SWIZZLE_64B) ||
        !make_map_t(&ml, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, W_lo, N, K, ldw * 2, kBK, kTF, CU_TENSOR_MAP_SWIZZLE_64B))
      return -1;
    CUtensorMap mc;
    if (!make_map_t(&mc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, C, M, N, ldc * 4, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B))
      return -1;
    const cudaError_t st = launch_f16_t<4, true, false>(ma, mal, mh, ml, mc, bias, w_scale_inv, (int)M, N, K, err, s);
    return st == cudaSuccess ? 0 : (int)st;
  }
  if (a_split && x1 && BN == 128 && N % 128 == 0 && use_t(K)) {
    // single product: hi halves only, eight stages, two accumulators (overlapped epilogue)
    const uint8_t* base = reinterpret_cast<const uint8_t*>(A);
    if (!make_map_t(&ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, base, M, K, lda * 4, kBK, kTE, CU_TENSOR_MAP_SWIZZLE_64B) ||
        !make_map_t(&mh, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, W_hi, N, K, ldw * 2, kBK, kTF, CU_TENSOR_MAP_SWIZZLE_64B))
      return -1;
    CUtensorMap mc;
    if (!(out_half ? make_map_t(&mc, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, C, M, N, ldc * 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B)
                   : make_map_t(&mc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, C, M, N, ldc * 4, 32, 32,
                                CU_TENSOR_MAP_SWIZZLE_128B)))
      return -1;
    const cudaError_t st =
        out_half ? launch_f16_t<8, false, true>(ma, ma, mh, mh, mc, bias, w_scale_inv, (int)M, N, K, err, s)
                 : launch_f16_t<8, false, false>(ma, ma, mh, mh, mc, bias, w_scale_inv, (int)M, N, K, err, s);
    return st == cudaSuccess ? 0 : (int)st;
  }
  if (a_split) {
    // row-packed split operand: row r holds K fp16 hi values at byte 4*lda*r and the K lo values
    // 2*lda bytes further
    const uint8_t* base = reinterpret_cast<const uint8_t*>(A);
    if (!make_map_t(&ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, base, M, K, lda * 4, kBK, kBM, CU_TENSOR_MAP_SWIZZLE_64B))
      return -1;
    if (!make_map_t(&mal, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, base + lda * 2, M, K, lda * 4, kBK, kBM,
                    CU_TENSOR_MAP_SWIZZLE_64B))
      return -1;
  } else {
    if (!make_map_t(&ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, A, M, K, lda * 4, kBK, kBM, CU_TENSOR_MAP_SWIZZLE_128B))
      return -1;
    mal = ma;
  }
  if (!make_map_t(&mh, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, W_hi, N, K, ldw * 2, kBK, BN, CU_TENSOR_MAP_SWIZZLE_64B))
    return -1;
  if (!make_map_t(&ml, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, W_lo, N, K, ldw * 2, kBK, BN, CU_TENSOR_MAP_SWIZZLE_64B))
    return -1;
  // output: fp32 [M, N] rows ldc apart, [32 x 32] boxes with 128-byte swizzle, or fp16 [M, N]
  // (ldc in halves) with 64-byte boxes and a 64-byte swizzle (unused for BN = 16)
  CUtensorMap mc = ma;
  if (BN >= 32 && !(out_half ? make_map_t(&mc, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, C, M, N, ldc * 2, 32, 32,
                                          CU_TENSOR_MAP_SWIZZLE_64B)
                             : make_map_t(&mc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, C, M, N, ldc * 4, 32, 32,
                                          CU_TENSOR_MAP_SWIZZLE_128B)))
    return -1;
  const int m = (int)M;
  const cudaError_t st =
      x1 ? (out_half ? launch_bn_x1<true>(BN, ma, mh, mc, C, bias, w_scale_inv, m, N, K, ldc, err, s)
                     : launch_bn_x1<false>(BN, ma, mh, mc, C, bias, w_scale_inv, m, N, K, ldc, err, s))
      : a_split ? launch_bn<true>(BN, ma, mal, mh, ml, mc, C, bias, w_scale_inv, m, N, K, ldc, err, s)
                : launch_bn<false>(BN, ma, mal, mh, ml, mc, C, bias, w_scale_inv, m, N, K, ldc, err, s);
  return st == cudaSuccess ? 0 : (int)st;
}

// Weight split: hi = fp16_rn(x * scale), lo = fp16_rn((x * scale - hi) * 2^11).
__global__ void split_f16_kernel(const float* __restrict__ x, __half* __restrict__ hi, __half* __restrict__ lo,
                                 float scale, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    bool bad = false;
    uint2 h, l;
    split_f16x4(make_float4(x[i] * scale, 0.f, 0.f, 0.f), h, l, bad);
    hi[i] = __ushort_as_half((unsigned short)(h.x & 0xFFFFu));
    lo[i] = __ushort_as_half((unsigned short)(l.x & 0xFFFFu));
  }
}

void launch_split_f16(const float* x, void* hi, void* lo, float scale, int64_t n, cudaStream_t s) {
  split_f16_kernel<<<grid_for(n, 256, 4), 256, 0, s>>>(x, static_cast<__half*>(hi), static_cast<__half*>(lo), scale,
                                                      n);
}

// Activation split into the row-packed operand of the kPre kernels: out row r (4*ldp bytes) holds
// fp16_rn(x[r, :K]) at byte 0 and fp16_rn((x - hi) * 2^11) at byte 2*ldp. One thread per 4 values.
__global__ void split_rows_f16_kernel(const float* __restrict__ x, int64_t lda, int64_t M, int K,
                                      uint8_t* __restrict__ out, int64_t ldp, int* err) {
  const int k4 = K >> 2;
  const int64_t total = M * k4;
  bool bad = false;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / k4;
    const int c = (int)(i - r * k4) * 4;
    uint2 hi, lo;
    split_f16x4(ld4_stream(x + r * lda + c), hi, lo, bad);
    uint8_t* row = out + r * ldp * 4;
    *reinterpret_cast<uint2*>(row + c * 2) = hi;
    *reinterpret_cast<uint2*>(row + ldp * 2 + c * 2) = lo;
  }
  if (bad && err) atomicCAS(err, 0, (int)kErrRange);
}

void launch_split_rows_f16(const float* x, int64_t lda, int64_t M, int K, void* out, int64_t ldp, int* err,
                           cudaStream_t s) {
  split_rows_f16_kernel<<<grid_resident(split_rows_f16_kernel, 256, M * (K / 4), 256), 256, 0, s>>>(x, lda, M, K, static_cast<uint8_t*>(out), ldp,
                                                                     err);
}

}  // namespace fuma
