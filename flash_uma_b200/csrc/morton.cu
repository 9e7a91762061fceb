// Morton order of the atoms and the renumbered graph (the reference's reorder_graph_morton,
// model.py:47-74, run at the start of every forward, model.py:189).
//
// The reference quantises every position to 10 bits per axis over the global bounding box,
//   q = int32((pos - pos_min) * (1023 / max(pos_max - pos_min, 1e-5)))   (per axis, fp32)
// interleaves the bits into a 30-bit code (x in bit 0, y in bit 1, z in bit 2 of every triple),
// sorts the atoms stably by key = code | (system << 32), and renumbers the edges. The fp32
// operations here are the reference's (subtract, then multiply by the per-axis scale,
// truncating conversion), so the order is identical to its stable argsort.
//
// Two sort paths:
//  * up to kMortonMaxAtoms atoms, one block of 1024 threads does the bounding box, the codes and
//    the sort in shared memory: a bitonic sort of (key, atom index) pairs, which orders ties by
//    index, i.e. the stable order (no scratch memory);
//  * any number of atoms (caller scratch, morton_scratch_bytes): a least-significant-digit radix
//    sort of the 64-bit keys with 8-bit digits over tiles of 4,096 keys. Per pass: a per-tile
//    digit histogram, one exclusive scan of the histograms in (digit, tile) order, and a stable
//    scatter in which every warp ranks its keys round by round (32 consecutive keys per round,
//    __match_any_sync peers) and the tile adds the earlier warps' counts. Passes 0-3 cover the
//    30-bit code; passes 4-7 cover the system id and run only while it has bits left (the pass
//    kernels read the largest system id from device memory, so nothing synchronises with the
//    host and the whole sort can be captured in a CUDA graph).
// A final grid-stride kernel gathers positions, species and system ids and renumbers both edge
// index rows; an edge index outside [0, N) is recorded in the error flag (code 32) and that edge
// is renumbered to atom 0, so that later kernels stay inside their arrays.
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

// ---- radix sort path (any N) ----------------------------------------------------------------

namespace {

constexpr int kBins = 256;                                  // 8-bit digits
constexpr int kTileWarps = 8;
constexpr int kTileRounds = 16;
constexpr int kTile = kTileWarps * 32 * kTileRounds;       // 4,096 keys per tile
constexpr int kMaxPasses = 8;                               // 32 code bits + 32 system-id bits
constexpr int kBboxBlocks = 148;
constexpr int kErrIndexRange = 32;                          // error-flag code: edge index outside [0, N)

// Scratch layout: keys[2][N] uint64, vals[2][N] int32, counts[kBins * tiles] int32,
// bbox[kBboxBlocks * 6] float, ctrl[4] int32 (ctrl[0]: largest system id).
struct MortonScratch {
  uint64_t* keys[2];
  int32_t* vals[2];
  int32_t* counts;
  float* bbox;
  int32_t* ctrl;
};

size_t align256(size_t b) { return (b + 255) & ~size_t(255); }

int64_t tiles_of(int64_t N) { return (N + kTile - 1) / kTile; }

size_t scratch_layout(int64_t N, char* base, MortonScratch* out) {
  size_t off = 0;
  auto take = [&](size_t bytes) {
    char* p = base ? base + off : nullptr;
    off += align256(bytes);
    return p;
  };
  MortonScratch m;
  m.keys[0] = reinterpret_cast<uint64_t*>(take(sizeof(uint64_t) * N));
  m.keys[1] = reinterpret_cast<uint64_t*>(take(sizeof(uint64_t) * N));
  m.vals[0] = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * N));
  m.vals[1] = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * N));
  m.counts = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * kBins * tiles_of(N)));
  m.bbox = reinterpret_cast<float*>(take(sizeof(float) * 6 * kBboxBlocks));
  m.ctrl = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * 4));
  if (out) *out = m;
  return off;
}

// passes needed for keys whose system id is at most maxb: 4 for the code, then one per 8 bits
__device__ __forceinline__ int radix_passes(int32_t maxb) {
  const int bits = maxb > 0 ? 32 - __clz(maxb) : 0;
  return 4 + (bits + 7) / 8;
}

}  // namespace

__global__ void __launch_bounds__(256) morton_bbox_kernel(const float* __restrict__ pos, int N,
                                                          float* __restrict__ bbox, int32_t* __restrict__ ctrl) {
  __shared__ float s_red[6][8];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  if (blockIdx.x == 0 && t == 0) ctrl[0] = 0;
  float mn[3] = {3.402823466e38f, 3.402823466e38f, 3.402823466e38f};
  float mx[3] = {-3.402823466e38f, -3.402823466e38f, -3.402823466e38f};
  for (int a = blockIdx.x * blockDim.x + t; a < N; a += gridDim.x * blockDim.x)
#pragma unroll
    for (int d = 0; d < 3; ++d) {
      const float v = pos[(int64_t)a * 3 + d];
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
  if (t < 6) {
    float v = s_red[t][0];
    for (int w = 1; w < 8; ++w) v = t < 3 ? fminf(v, s_red[t][w]) : fmaxf(v, s_red[t][w]);
    bbox[blockIdx.x * 6 + t] = v;
  }
}

__global__ void __launch_bounds__(256) morton_keys_kernel(const float* __restrict__ pos,
                                                          const int64_t* __restrict__ batch, int N,
                                                          const float* __restrict__ bbox, uint64_t* __restrict__ keys,
                                                          int32_t* __restrict__ vals, int32_t* __restrict__ ctrl) {
  __shared__ float s_lo[3], s_sc[3];
  __shared__ int32_t s_maxb;
  const int t = threadIdx.x;
  if (t < 3) {
    float a = bbox[t], b = bbox[3 + t];
    for (int k = 1; k < kBboxBlocks; ++k) {
      a = fminf(a, bbox[k * 6 + t]);
      b = fmaxf(b, bbox[k * 6 + 3 + t]);
    }
    s_lo[t] = a;
    s_sc[t] = 1023.0f / fmaxf(b - a, 1e-5f);
  }
  if (t == 0) s_maxb = 0;
  __syncthreads();
  int32_t mb = 0;
  for (int a = blockIdx.x * blockDim.x + t; a < N; a += gridDim.x * blockDim.x) {
    uint32_t code = 0;
#pragma unroll
    for (int d = 0; d < 3; ++d) {
      const int32_t q = (int32_t)((pos[(int64_t)a * 3 + d] - s_lo[d]) * s_sc[d]);
      code |= expand_bits10((uint32_t)q) << d;
    }
    const int64_t b = batch[a];
    keys[a] = (uint64_t)code | ((uint64_t)b << 32);
    vals[a] = a;
    mb = max(mb, (int32_t)min(b, (int64_t)0x7fffffff));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mb = max(mb, __shfl_xor_sync(kFull, mb, o));
  if ((t & 31) == 0) atomicMax(&s_maxb, mb);
  __syncthreads();
  if (t == 0) atomicMax(ctrl, s_maxb);
}

// per-tile histogram of the pass's digit -> counts[digit * tiles + tile]
__global__ void __launch_bounds__(256) morton_radix_count_kernel(const uint64_t* __restrict__ keys, int N, int pass,
                                                                 int tiles, int32_t* __restrict__ counts,
                                                                 const int32_t* __restrict__ ctrl) {
  if (pass >= radix_passes(ctrl[0])) return;
  __shared__ int32_t h[kBins];
  const int t = threadIdx.x;
  h[t] = 0;
  __syncthreads();
  const int shift = 8 * pass;
  const int end = min(N, (blockIdx.x + 1) * kTile);
  for (int i = blockIdx.x * kTile + t; i < end; i += blockDim.x) atomicAdd(&h[(int)((keys[i] >> shift) & 255)], 1);
  __syncthreads();
  counts[t * tiles + blockIdx.x] = h[t];
}

// exclusive scan of counts[kBins * tiles] in place (one block)
__global__ void __launch_bounds__(1024) morton_radix_scan_kernel(int32_t* __restrict__ counts, int total, int pass,
                                                                 const int32_t* __restrict__ ctrl) {
  if (pass >= radix_passes(ctrl[0])) return;
  __shared__ int32_t s_warp[32];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int chunk = (total + 1023) / 1024;
  const int b0 = min(total, t * chunk), b1 = min(total, b0 + chunk);
  int sum = 0;
  for (int i = b0; i < b1; ++i) sum += counts[i];
  int incl = sum;   // inclusive scan over the block
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = s_warp[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(kFull, w, o);
      if (lane >= o) w += v;
    }
    s_warp[lane] = w;
  }
  __syncthreads();
  int run = incl - sum + (warp > 0 ? s_warp[warp - 1] : 0);
  for (int i = b0; i < b1; ++i) {
    const int c = counts[i];
    counts[i] = run;
    run += c;
  }
}

// stable scatter of one tile by the pass's digit
__global__ void __launch_bounds__(kTileWarps * 32) morton_radix_scatter_kernel(
    const uint64_t* __restrict__ keys_in, const int32_t* __restrict__ vals_in, uint64_t* __restrict__ keys_out,
    int32_t* __restrict__ vals_out, int N, int pass, int tiles, const int32_t* __restrict__ offsets,
    const int32_t* __restrict__ ctrl) {
  if (pass >= radix_passes(ctrl[0])) return;
  __shared__ int32_t s_cnt[kTileWarps][kBins];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  for (int i = t; i < kTileWarps * kBins; i += blockDim.x) (&s_cnt[0][0])[i] = 0;
  __syncthreads();
  const int shift = 8 * pass;
  const int wbase = blockIdx.x * kTile + warp * 32 * kTileRounds;
  uint64_t key[kTileRounds];
  int32_t val[kTileRounds];
  int dig[kTileRounds], rnk[kTileRounds];
#pragma unroll
  for (int r = 0; r < kTileRounds; ++r) {
    const int idx = wbase + r * 32 + lane;
    const bool valid = idx < N;
    key[r] = valid ? keys_in[idx] : 0;
    val[r] = valid ? vals_in[idx] : 0;
    const int d = valid ? (int)((key[r] >> shift) & 255) : 0;
    dig[r] = d;
    rnk[r] = 0;
    const unsigned active = __ballot_sync(kFull, valid);
    if (valid) {
      const unsigned peers = __match_any_sync(active, d);
      const int before = __popc(peers & ((1u << lane) - 1u));
      const int base = s_cnt[warp][d];
      rnk[r] = base + before;
      __syncwarp(active);
      if (before == 0) s_cnt[warp][d] = base + __popc(peers);   // the group's lowest lane
      __syncwarp(active);
    }
  }
  __syncthreads();
  {   // per digit: the tile's global offset plus the counts of the warps before
    int run = offsets[t * tiles + blockIdx.x];
#pragma unroll
    for (int w = 0; w < kTileWarps; ++w) {
      const int c = s_cnt[w][t];
      s_cnt[w][t] = run;
      run += c;
    }
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < kTileRounds; ++r) {
    const int idx = wbase + r * 32 + lane;
    if (idx < N) {
      const int p = s_cnt[warp][dig[r]] + rnk[r];
      keys_out[p] = key[r];
      vals_out[p] = val[r];
    }
  }
}

// perm / inv_perm from the sorted values (the buffer the last pass wrote)
__global__ void __launch_bounds__(256) morton_finalize_kernel(const int32_t* __restrict__ vals0,
                                                              const int32_t* __restrict__ vals1, int N,
                                                              const int32_t* __restrict__ ctrl,
                                                              int64_t* __restrict__ perm,
                                                              int64_t* __restrict__ inv_perm) {
  const int32_t* v = (radix_passes(ctrl[0]) & 1) ? vals1 : vals0;
  for (int a = blockIdx.x * blockDim.x + threadIdx.x; a < N; a += gridDim.x * blockDim.x) {
    const int32_t o = v[a];
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
                                                           int64_t* __restrict__ jj, int* __restrict__ err) {
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
      const int64_t i = idx_i[t], j = idx_j[t];
      if ((uint64_t)i < (uint64_t)N && (uint64_t)j < (uint64_t)N) {
        ii[t] = inv_perm[i];
        jj[t] = inv_perm[j];
      } else {   // invalid edge: recorded, renumbered to atom 0 so later kernels stay in bounds
        ii[t] = 0;
        jj[t] = 0;
        if (err) atomicCAS(err, 0, kErrIndexRange);   // the first recorded error is kept
      }
    }
  }
}

int64_t morton_scratch_bytes(int64_t N) { return N <= kMortonMaxAtoms ? 0 : (int64_t)scratch_layout(N, nullptr, nullptr); }

cudaError_t launch_morton_reorder(const float* pos, const int64_t* Z, const int64_t* batch, const int64_t* idx_i,
                                  const int64_t* idx_j, int64_t N, int64_t E, int64_t* perm, int64_t* inv_perm,
                                  float* pos_s, int64_t* Z_s, int64_t* batch_s, int64_t* ii, int64_t* jj,
                                  void* scratch, int* err, cudaStream_t s) {
  if (N > 0 && N <= kMortonMaxAtoms) {
    int P = 1;
    while (P < N) P <<= 1;
    if (P < 2) P = 2;
    const size_t smem = (size_t)P * (sizeof(uint64_t) + sizeof(int32_t));
    static thread_local uint64_t configured = 0;   // one bit per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(configured >> (dev & 63) & 1)) {
      const size_t mx = (size_t)kMortonMaxAtoms * (sizeof(uint64_t) + sizeof(int32_t));
      const cudaError_t st = cudaFuncSetAttribute(morton_sort_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  (int)mx);
      if (st != cudaSuccess) return st;
      configured |= uint64_t(1) << (dev & 63);
    }
    morton_sort_kernel<<<1, kSortThreads, smem, s>>>(pos, batch, (int)N, P, perm, inv_perm);
  } else if (N > kMortonMaxAtoms) {
    MortonScratch m;
    scratch_layout(N, static_cast<char*>(scratch), &m);
    const int n = (int)N;
    const int tiles = (int)tiles_of(N);
    morton_bbox_kernel<<<kBboxBlocks, 256, 0, s>>>(pos, n, m.bbox, m.ctrl);
    morton_keys_kernel<<<grid_resident(morton_keys_kernel, 256, N, 256), 256, 0, s>>>(pos, batch, n, m.bbox,
                                                                                       m.keys[0], m.vals[0], m.ctrl);
    for (int p = 0; p < kMaxPasses; ++p) {
      const int a = p & 1, b = a ^ 1;
      morton_radix_count_kernel<<<tiles, kBins, 0, s>>>(m.keys[a], n, p, tiles, m.counts, m.ctrl);
      morton_radix_scan_kernel<<<1, 1024, 0, s>>>(m.counts, kBins * tiles, p, m.ctrl);
      morton_radix_scatter_kernel<<<tiles, kTileWarps * 32, 0, s>>>(m.keys[a], m.vals[a], m.keys[b], m.vals[b], n, p,
                                                                    tiles, m.counts, m.ctrl);
    }
    morton_finalize_kernel<<<grid_resident(morton_finalize_kernel, 256, N, 256), 256, 0, s>>>(m.vals[0], m.vals[1], n,
                                                                                               m.ctrl, perm, inv_perm);
  }
  const int64_t n = N > E ? N : E;
  if (n > 0)
    morton_apply_kernel<<<grid_resident(morton_apply_kernel, 256, n, 256), 256, 0, s>>>(
        pos, Z, batch, idx_i, idx_j, perm, inv_perm, N, E, pos_s, Z_s, batch_s, ii, jj, err);
  return cudaGetLastError();
}

}  // namespace fuma
