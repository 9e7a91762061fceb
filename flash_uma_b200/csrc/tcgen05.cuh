// Shared building blocks of the tcgen05 GEMM kernels (sm_100a): mbarriers with bounded waits,
// TMA tile loads, shared-memory matrix descriptors and tcgen05 commit.
#pragma once

#include <cstdint>

#include <cuda.h>

namespace fuma {

constexpr uint32_t kWaitLimit = 1u << 24;   // try_wait iterations before a pipeline wait gives up

// Error codes a GEMM kernel leaves in its error flag (first one wins).
enum GemmErr : int {
  kErrWaitEmpty = 1, kErrWaitFull = 2, kErrWaitSplit = 3, kErrWaitAcc = 4, kErrWaitAccEmpty = 5,
  kErrRange = 16,   // an activation is finite in fp32 but beyond the fp16 range of the f16x3 split
};

namespace {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait. Returns false (and records `code`) if the phase did not complete, or if
// another role of this CTA already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err,
                                          int code) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (mbar_try(bar, parity)) return true;
    if ((i & 1023u) == 1023u && *abort_flag) return false;
  }
  *abort_flag = 1;
  if (err) atomicCAS(err, 0, code);
  return false;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);          // start address
  d |= (uint64_t)1u << 16;                          // leading byte offset (unused for SW128 K-major)
  d |= (uint64_t)(1024u >> 4) << 32;                // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1u << 46;                          // descriptor version (sm100)
  d |= (uint64_t)2u << 61;                          // layout: SWIZZLE_128B
  return d;
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

}  // namespace

// 2-D tensor map (cols contiguous, row stride ld_bytes), box box_cols x box_rows, zero fill out of range.
// On failure returns false and leaves a message for gemm_map_error().
bool make_map_t(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, int64_t rows, int64_t cols,
                int64_t ld_bytes, int box_cols, int box_rows, CUtensorMapSwizzle swz);

}  // namespace fuma
