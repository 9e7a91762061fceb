// Allocation-free variant of the Morton reorder (fuma_morton_reorder_noalloc).
//
// Who needs it: some callers cannot let a library allocate device memory, or cannot allocate
// scratch themselves at the point where they call in. Examples are molecular-dynamics engines
// and other host programs that own the whole device memory budget and hand out only the
// buffers they planned for, code that must not pay for or be serialised by cudaMalloc /
// cudaFree inside a time-critical step, and foreign-language bindings that can pass the
// caller's arrays but have no device allocator to lend. fuma_morton_reorder asks such callers
// for a scratch buffer as soon as a system has more than 16,384 atoms (its multi-block radix
// sort ping-pongs the keys and atom indices through it, about 24 bytes per atom); this entry
// point uses a scratch array that lives in this file instead, so the caller passes only its
// inputs and outputs.
//
// The array is a file-scope __device__ array of kNoAllocScratchBytes bytes (13 MiB), enough for
// kNoAllocMaxAtoms = 524,288 atoms; every GPU that loads this library holds it until the process
// exits. Larger systems are refused with FUMA_E_INVALID. In host code the array's name is not a
// device address, so the first call on each device looks the address up with
// cudaGetSymbolAddress (with that device current) and remembers it; make that first call on a
// device before any stream capture. Every call shares the one array and the array keeps the last
// call's contents: nothing in it has to start at zero (each call writes the keys, atom indices,
// digit counts and bounding-box partials it reads), but calls that can overlap on the GPU
// (different streams, or different host threads on the same device) race on it and must be
// serialised by the caller. No cudaMalloc, cudaFree or allocating library routine is called.
#include <mutex>

#include "../../include/flash_uma_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace fuma {
namespace {

constexpr int64_t kNoAllocMaxAtoms = int64_t(1) << 19;        // 524,288 atoms
constexpr int64_t kNoAllocScratchBytes = int64_t(13) << 20;   // 13 MiB
static __device__ __align__(256) unsigned char g_morton_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_addr_mutex;
void* g_addr[kMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once per device).
cudaError_t scratch_address(void** out) {
  int dev = 0;
  cudaError_t st = cudaGetDevice(&dev);
  if (st != cudaSuccess) return st;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_addr_mutex);
  if (!g_addr[dev]) {
    void* p = nullptr;
    st = cudaGetSymbolAddress(&p, g_morton_scratch);
    if (st != cudaSuccess) return st;
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return cudaSuccess;
}

}  // namespace
}  // namespace fuma

using namespace fuma;

extern "C" {

int fuma_morton_reorder_noalloc(const float* pos, const int64_t* Z, const int64_t* batch, const int64_t* idx_i,
                                const int64_t* idx_j, int64_t N, int64_t E, int64_t* perm, int64_t* inv_perm,
                                float* pos_s, int64_t* Z_s, int64_t* batch_s, int64_t* ii, int64_t* jj, int* err_flag,
                                void* stream) {
  if (N < 0 || N > kNoAllocMaxAtoms)
    return report_error(FUMA_E_INVALID,
                        "morton_reorder_noalloc: N=%lld is beyond the %lld atoms its built-in %lld-byte scratch "
                        "array holds (use fuma_morton_reorder with a caller scratch buffer)",
                        (long long)N, (long long)kNoAllocMaxAtoms, (long long)kNoAllocScratchBytes);
  if (E < 0) return report_error(FUMA_E_INVALID, "morton_reorder_noalloc: bad E=%lld", (long long)E);
  if (N == 0 && E == 0) return report_error(FUMA_OK, "");
  if (!(pos && Z && batch && perm && inv_perm && Z_s && batch_s))
    return report_error(FUMA_E_INVALID, "morton_reorder_noalloc: null atom pointer");
  if (E > 0 && !(idx_i && idx_j && ii && jj))
    return report_error(FUMA_E_INVALID, "morton_reorder_noalloc: null edge pointer");
  if (morton_scratch_bytes(N) > kNoAllocScratchBytes)
    return report_error(FUMA_E_INVALID, "morton_reorder_noalloc: N=%lld needs more scratch than the array holds",
                        (long long)N);
  if (int rc = bind_device_of(pos)) return rc;
  void* scratch = nullptr;
  cudaError_t st = scratch_address(&scratch);
  if (st != cudaSuccess)
    return report_error((int)st, "morton_reorder_noalloc: cudaGetSymbolAddress of the scratch array failed: %s",
                        cudaGetErrorString(st));
  st = launch_morton_reorder(pos, Z, batch, idx_i, idx_j, N, E, perm, inv_perm, pos_s, Z_s, batch_s, ii, jj, scratch,
                             err_flag, (cudaStream_t)stream);
  if (st != cudaSuccess)
    return report_error((int)st, "morton_reorder_noalloc: launch failed: %s", cudaGetErrorString(st));
  return launch_status("morton_reorder_noalloc");
}

}  // extern "C"
