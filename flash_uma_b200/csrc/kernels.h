// Host launchers of the device kernels (one per operation; see the .cu files for the math
// and the reference citations). Arguments are validated by the C ABI layer (capi.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace fuma {

void launch_geom_fwd(const float* pos, const int64_t* Z, const int64_t* idx_i, const int64_t* idx_j,
                     const float* shifts, const float* W_src, const float* W_tgt, const float* offset_g,
                     float* x_edge, float* wig, float* env_out, int64_t E, int B, int C, float cutoff, float coeff,
                     cudaStream_t s);
void launch_geom_bwd(const float* pos, const int64_t* idx_i, const int64_t* idx_j, const float* shifts,
                     const float* offset_g, const float* g_xe, int64_t xe_stride, const float* g_wig,
                     const float* g_env, float* g_vec, int64_t E, int B, float cutoff, float coeff, cudaStream_t s);
void launch_node_vec3_segment(const int32_t* src_ptr, const int32_t* src_col, const int32_t* dst_ptr,
                              const int32_t* dst_col, const float* g_vec, float* g_pos, int64_t N, cudaStream_t s);

void launch_gather_fwd(const float* x, const int64_t* idx_i, const int64_t* idx_j, const float* wig, const float* rad,
                       const float* csd, const int64_t* batch, float* X0, float* X1, float* X2, int64_t E, int C,
                       int split, int* err, cudaStream_t s, bool act_half = false);
void launch_gather_bwd(const float* gX0, const float* gX1, const float* gX2, const float* x, const int64_t* idx_i,
                       const float* wig, const float* rad, const float* csd, const int64_t* batch,
                       const int32_t* dst_ptr, const int32_t* dst_col, const int32_t* src_ptr, const int32_t* src_col,
                       float* g_x, float* g_wig, float* g_rad, float* scratch, int64_t N, int C, int split, int* err,
                       cudaStream_t s, bool act_half = false);

// act_half (the single-product mode's 16-bit storage): the GEMM results these kernels read are
// fp16 arrays passed as float*, with the same element offsets: Y and gZ (gating), rad and gX
// (gather), the conv2 output Z (rotate-scatter).
void launch_gating_fwd(const float* Y0, const float* Y1, const float* Y2, float* Z0, float* Z1, float* Z2, int64_t E,
                       int C, int split, int* err, cudaStream_t s, bool act_half = false);
void launch_gating_bwd(const float* gZ0, const float* gZ1, const float* gZ2, const float* Y0, const float* Y1,
                       const float* Y2, float* gY0, float* gY1, float* gY2, int64_t E, int C, int split, int* err,
                       cudaStream_t s, bool act_half = false);

void launch_ln_silu_fwd(const float* x, const float* gamma, const float* beta, float* out, float* mean, float* rstd,
                        int64_t M, int D, float eps, int split, int* err, cudaStream_t s);
void launch_ln_silu_bwd(const float* x, const float* gamma, const float* beta, const float* mean, const float* rstd,
                        const float* g_out, float* g_x, int64_t M, int D, int split, int* err, cudaStream_t s);

void launch_rotate_scatter_fwd(const int32_t* row_ptr, const int32_t* col_idx, const float* Z0, const float* Z1,
                               const float* Z2, const float* wig, const float* env, const float* x_res, float* x_out,
                               int64_t N, int C, cudaStream_t s, bool act_half = false);
void launch_rotate_scatter_bwd(const int32_t* row_ptr, const int32_t* col_idx, const float* g_out, const float* Z0,
                               const float* Z1, const float* Z2, const float* wig, const float* env, float* gZ0,
                               float* gZ1, float* gZ2, float* g_wig, float* g_env, int64_t N, int C, int split,
                               int* err, cudaStream_t s, bool act_half = false);
void launch_init_scatter_fwd(const int32_t* row_ptr, const int32_t* col_idx, const float* rad, const float* wig,
                             const float* env, const int64_t* Z, const int64_t* batch, const float* W_sphere,
                             const float* csd, float* x_out, int64_t N, int C, cudaStream_t s);
void launch_init_scatter_bwd(const int32_t* row_ptr, const int32_t* col_idx, const float* g_out, const float* rad,
                             const float* wig, const float* env, float* g_rad, float* g_wig, float* g_env, int64_t N,
                             int C, int split, int* err, cudaStream_t s);

int launch_gemm_tf32(const float* A, int64_t lda, const float* W_hi, const float* W_lo, const float* bias, float* C,
                     int64_t ldc, int64_t M, int N, int K, bool split, int* err, cudaStream_t s);
void launch_split_tf32(const float* x, float* hi, float* lo, int64_t n, cudaStream_t s);
const char* gemm_map_error();
void launch_rmsnorm_sh_fwd(const float* x, const float* aw, const float* ab, const float* bal, float eps, int64_t N,
                           int C, float* out, float* rstd, cudaStream_t s);
void launch_rmsnorm_sh_bwd(const float* x, const float* aw, const float* bal, const float* rstd, const float* g_out,
                           int64_t N, int C, float* g_x, cudaStream_t s);
// Atom-wise block on coefficient rows (row k * N + n = coefficient k of atom n). h / gz: row
// stride ldh; blocked: the degree-blocked output of one GEMM against the three stacked degree
// weights (column block deg(k) * H). split 0 writes fp32, 1 / 2 the row-packed split.
void launch_atomwise_gate_fwd(const float* h, int64_t ldh, bool blocked, const float* u, const float* b1, int64_t N,
                              int H, float* z, int split, int* err, cudaStream_t s);
void launch_atomwise_gate_bwd(const float* gz, const float* h, int64_t ldh, bool blocked, const float* u,
                              const float* b1, int64_t N, int H, float* gh, float* gu, int split, int* err,
                              cudaStream_t s);
void launch_coef_to_node(const float* src, int64_t lds, bool blocked, const float* add, const float* row0,
                         int row0_per_node, int64_t N, int W, float* out, cudaStream_t s);
void launch_node_to_coef(const float* x, int64_t N, int W, float* out, int split, int* err, cudaStream_t s);
constexpr int kMortonMaxAtoms = 16384;   // up to this many atoms one block sorts them in shared memory
// scratch bytes of the radix-sort path (0 up to kMortonMaxAtoms atoms)
int64_t morton_scratch_bytes(int64_t N);
cudaError_t launch_morton_reorder(const float* pos, const int64_t* Z, const int64_t* batch, const int64_t* idx_i,
                                  const int64_t* idx_j, int64_t N, int64_t E, int64_t* perm, int64_t* inv_perm,
                                  float* pos_s, int64_t* Z_s, int64_t* batch_s, int64_t* ii, int64_t* jj,
                                  void* scratch, int* err, cudaStream_t s);
void launch_csr_permute(int ngraphs, const int32_t* const* row_ptr, const int32_t* const* col, const int64_t* perm,
                        int64_t N, int32_t* const* new_row_ptr, int32_t* const* new_col, cudaStream_t s);
int launch_gemm_f16x3(const float* A, int64_t lda, bool a_split, const void* W_hi, const void* W_lo, int64_t ldw,
                      float w_scale_inv, const float* bias, float* C, int64_t ldc, int64_t M, int N, int K, int* err,
                      cudaStream_t s, bool x1 = false, bool out_half = false);
void launch_split_rows_f16(const float* x, int64_t lda, int64_t M, int K, void* out, int64_t ldp, int* err,
                           cudaStream_t s);
void launch_split_f16(const float* x, void* hi, void* lo, float scale, int64_t n, cudaStream_t s);

int64_t neighbor_scratch_bytes(int64_t N, int64_t nbins);
cudaError_t launch_neighbor_list(const double* pos, int64_t N, const double* cell, const double* inv,
                                 const int32_t* nb, const int32_t* lo, const int32_t* hi, const int32_t* pbc,
                                 double cutoff, int max_nb, void* scratch, int32_t* counts, int64_t* out_src,
                                 int64_t* out_off, double* out_dist, int* err, cudaStream_t s);

// The C ABI's shared argument handling (capi.cu): make the device owning `p` current (returns
// FUMA_E_INVALID for memory that is not a CUDA allocation), and the status after a launch.
int bind_device_of(const void* p);
int launch_status(const char* what);

// Record `fmt` as the calling thread's fuma_last_error() message and return `code`.
int report_error(int code, const char* fmt, ...);

}  // namespace fuma
