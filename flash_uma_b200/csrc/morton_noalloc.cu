// Allocation-free variant of the gather backward (fuma_gather_bwd_noalloc).
//
// Who needs it: some callers cannot let a library allocate device memory. Examples are
// molecular-dynamics engines and other host frameworks that own the whole device memory
// budget and hand out only the buffers they planned for, callers that must not pay for
// (or be serialised by) cudaMalloc / cudaFree inside a time-critical step, and callers
// that have no allocator of their own to lend. fuma_gather_bwd asks such callers for a
// scratch buffer of E*9*C floats; this entry point instead uses a fixed scratch array
// that lives in this file, so the caller passes only its inputs and outputs.
//
// The scratch array is a file-scope __device__ array of kNoAllocScratchFloats floats
// (32 MiB). Every GPU that loads this library holds it until the process exits. Host
// code cannot use the array's name as a device address, so the first call on each
// device looks the address up with cudaGetSymbolAddress (with that device current) and
// remembers it; that first call should therefore happen before any stream capture.
// Calls whose E*9*C exceeds the array are rejected with FUMA_E_INVALID.
//
// Nothing in the scratch array has to start at zero: pass A of the backward writes the
// source-side row of every edge before pass B reads it, within the same call. All calls
// share the one array, so calls that can overlap on the GPU (different streams, or
// different host threads on the same device) race on it and must be serialised by the
// caller.
#include <mutex>

#include "../../include/flash_uma_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace fuma {
namespace {

constexpr int64_t kNoAllocScratchFloats = int64_t(8) << 20;  // 8 Mi floats = 32 MiB
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mutex;
float* g_noalloc_addr[kMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once per device).
cudaError_t noalloc_scratch(float** out) {
  int dev = 0;
  cudaError_t st = cudaGetDevice(&dev);
  if (st != cudaSuccess) return st;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    st = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (st != cudaSuccess) return st;
    g_noalloc_addr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_addr[dev];
  return cudaSuccess;
}

int reject(int code, const char* msg) { return report_error(code, "gather_bwd_noalloc: %s", msg); }

}  // namespace
}  // namespace fuma

using namespace fuma;

extern "C" {

int fuma_gather_bwd_noalloc(const float* g_X_m0, const float* g_X_m1, const float* g_X_m2, const float* x,
                            const int64_t* idx_i, const float* wigner, const float* rad, const float* csd,
                            const int64_t* batch, const int32_t* dst_row_ptr, const int32_t* dst_col,
                            const int32_t* src_row_ptr, const int32_t* src_col, int64_t N, int64_t E, int32_t C,
                            float* g_x, float* g_wigner, float* g_rad, void* stream) {
  if (C <= 0 || (C & 3) != 0 || C > 512) return reject(FUMA_E_INVALID, "C must be a positive multiple of 4, <= 512");
  if (N < 0 || E < 0) return reject(FUMA_E_INVALID, "negative size");
  if (E * 9 * (int64_t)C > kNoAllocScratchFloats)
    return reject(FUMA_E_INVALID, "E*9*C exceeds the 8 Mi-float (32 MiB) built-in scratch array");
  if (N == 0) return FUMA_OK;
  if (!x || !csd || !batch || !dst_row_ptr || !src_row_ptr || !g_x) return reject(FUMA_E_INVALID, "null pointer");
  if (E > 0 && !(idx_i && wigner && rad && dst_col && src_col && g_wigner && g_rad && g_X_m0 && g_X_m1 && g_X_m2))
    return reject(FUMA_E_INVALID, "null per-edge pointer");
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, x) != cudaSuccess || a.type != cudaMemoryTypeDevice) {
    cudaGetLastError();
    return reject(FUMA_E_INVALID, "x is not device memory");
  }
  cudaError_t st = cudaSetDevice(a.device);
  if (st != cudaSuccess) return reject((int)st, "cudaSetDevice failed");
  float* scratch = nullptr;
  st = noalloc_scratch(&scratch);
  if (st != cudaSuccess) return reject((int)st, "cudaGetSymbolAddress of the scratch array failed");
  launch_gather_bwd(g_X_m0, g_X_m1, g_X_m2, x, idx_i, wigner, rad, csd, batch, dst_row_ptr, dst_col, src_row_ptr,
                    src_col, g_x, g_wigner, g_rad, scratch, N, C, false, nullptr, (cudaStream_t)stream);
  st = cudaGetLastError();
  if (st != cudaSuccess) return reject((int)st, "kernel launch failed");
  return report_error(FUMA_OK, "");
}

}  // extern "C"
