// CSR of a renumbered graph from the CSR of the original numbering (the per-step graph build of
// the reference, model.py:17-46 and :189-191, without a sort).
//
// The reference renumbers the atoms every forward (Morton order, model.py:47-74) and then
// builds the destination CSR of the renumbered edge list with a stable argsort, keyed on the
// renumbered index tensors, which are new every step, so the sort runs on every call. The
// edges themselves keep their ids; only node ids change. Row a of the renumbered CSR therefore
// holds exactly the edges of original node perm[a], and a stable argsort keeps them in
// increasing edge id, which is their order in row perm[a] of the original CSR. So
//   new_row_ptr = exclusive scan over a of deg(perm[a]),
//   new_col[new_row_ptr[a] + t] = col[row_ptr[perm[a]] + t],
// bitwise the CSR of the stable argsort, from the original CSR (cached across steps because the
// caller's edge list does not change) in O(N + E) with no sort.
//
// Two launches for up to two CSRs at once (blockIdx.y selects the CSR): a one-block scan of the
// permuted degrees (1024 threads, a contiguous chunk each), then a warp-per-row segment copy.
#include "common.cuh"
#include "kernels.h"

namespace fuma {

namespace {

constexpr int kScanThreads = 1024;

struct CsrPair {
  const int32_t* row_ptr[2];
  const int32_t* col[2];
  int32_t* new_row_ptr[2];
  int32_t* new_col[2];
};

}  // namespace

__global__ void __launch_bounds__(kScanThreads) csr_permute_scan_kernel(CsrPair p, const int64_t* __restrict__ perm,
                                                                        int64_t N) {
  const int g = blockIdx.y;
  const int32_t* __restrict__ rp = p.row_ptr[g];
  int32_t* __restrict__ out = p.new_row_ptr[g];
  __shared__ int32_t s_part[kScanThreads];
  const int t = threadIdx.x;
  const int64_t chunk = (N + kScanThreads - 1) / kScanThreads;
  const int64_t lo = t * chunk, hi = (lo + chunk < N) ? lo + chunk : N;
  int32_t sum = 0;
  for (int64_t a = lo; a < hi; ++a) {
    const int64_t o = perm[a];
    sum += rp[o + 1] - rp[o];
  }
  s_part[t] = sum;
  __syncthreads();
  // inclusive scan of the 1024 partial sums (Hillis-Steele in shared memory)
  for (int off = 1; off < kScanThreads; off <<= 1) {
    const int32_t v = t >= off ? s_part[t - off] : 0;
    __syncthreads();
    s_part[t] += v;
    __syncthreads();
  }
  int32_t run = t ? s_part[t - 1] : 0;
  for (int64_t a = lo; a < hi; ++a) {
    out[a] = run;
    const int64_t o = perm[a];
    run += rp[o + 1] - rp[o];
  }
  if (t == kScanThreads - 1) out[N] = s_part[kScanThreads - 1];
}

__global__ void __launch_bounds__(256) csr_permute_copy_kernel(CsrPair p, const int64_t* __restrict__ perm, int64_t N) {
  const int g = blockIdx.y;
  const int32_t* __restrict__ rp = p.row_ptr[g];
  const int32_t* __restrict__ col = p.col[g];
  const int32_t* __restrict__ nrp = p.new_row_ptr[g];
  int32_t* __restrict__ ncol = p.new_col[g];
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t a = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); a < N; a += warps) {
    const int64_t o = perm[a];
    const int32_t src = rp[o], len = rp[o + 1] - src, dst = nrp[a];
    for (int32_t t = lane; t < len; t += 32) ncol[dst + t] = col[src + t];
  }
}

void launch_csr_permute(int ngraphs, const int32_t* const* row_ptr, const int32_t* const* col, const int64_t* perm,
                        int64_t N, int32_t* const* new_row_ptr, int32_t* const* new_col, cudaStream_t s) {
  CsrPair p{};
  for (int g = 0; g < ngraphs; ++g) {
    p.row_ptr[g] = row_ptr[g];
    p.col[g] = col[g];
    p.new_row_ptr[g] = new_row_ptr[g];
    p.new_col[g] = new_col[g];
  }
  csr_permute_scan_kernel<<<dim3(1, ngraphs), kScanThreads, 0, s>>>(p, perm, N);
  const unsigned gx = grid_resident(csr_permute_copy_kernel, 256, N, 8);
  csr_permute_copy_kernel<<<dim3(gx, ngraphs), 256, 0, s>>>(p, perm, N);
}

}  // namespace fuma
