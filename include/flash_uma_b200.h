/*
 * flash_uma_b200 - C ABI of the B200 (sm_100a) eSCN/UMA message-passing hot path.
 *
 * Every entry point launches its kernels asynchronously on `stream` (a cudaStream_t
 * passed as void*, NULL = legacy default stream) and returns 0 on success, a
 * negative FUMA_E_* code for an invalid argument (nothing is launched), or a
 * positive CUDA error code if the launch failed. fuma_last_error() describes the
 * last failure of the calling thread.
 *
 * Conventions: all pointers are device pointers to contiguous row-major arrays;
 * features are fp32; atom/edge indices, atomic numbers and system ids are int64
 * (as the reference passes them); CSR arrays are int32. Vector-accessed feature
 * arrays must be 16-byte aligned and C (channels) a multiple of 4, C <= 512.
 * Outputs are written in full (no zero-initialised buffers are required) unless
 * a comment says otherwise. With E == 0 the per-edge pointers may be NULL (the
 * data pointer of an empty tensor). No entry point allocates memory, synchronises the
 * device or keeps state between calls.
 *
 * Each function replaces one reference op; the citation is the reference
 * interface (path:line in the FlashUMA source tree) whose semantics it implements.
 */
#ifndef FLASH_UMA_B200_H
#define FLASH_UMA_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FUMA_OK 0
#define FUMA_E_INVALID (-1)     /* bad size / null pointer / unsupported shape */
#define FUMA_E_ALIGN (-2)       /* pointer not 16-byte aligned */

/* Library version (major*10000 + minor*100 + patch). */
int fuma_version(void);
/* Message for the last failure on the calling thread ("" if none). */
const char* fuma_last_error(void);

/* ---- geometry ---------------------------------------------------------------------------
 * Replaces PrecomputeGeometry.forward (ops/geom.py:496-531, kernel :36-214).
 * pos[N,3], Z[N], idx_i/idx_j[E] (edge source i -> destination j), shifts[E,3],
 * W_src/W_tgt[num_z,C], offset_g[B]  ->  x_edge_raw[E,B+2C], wigner[E,34], env[E]. */
int fuma_geometry_fwd(const float* pos, const int64_t* Z, const int64_t* idx_i, const int64_t* idx_j,
                      const float* shifts, const float* W_src, const float* W_tgt, const float* offset_g,
                      float coeff_g, float cutoff, int64_t N, int64_t E, int32_t B, int32_t C,
                      float* x_edge_raw, float* wigner, float* env, void* stream);

/* Replaces PrecomputeGeometry.backward (ops/geom.py:533-589, kernel :220-493), split in two:
 * per-edge gradient w.r.t. the edge vector (= g_shifts[E,3]); only the first B columns of
 * g_x_edge (row stride g_x_edge_stride floats) are read. */
int fuma_geometry_bwd(const float* pos, const int64_t* idx_i, const int64_t* idx_j, const float* shifts,
                      const float* offset_g, float coeff_g, float cutoff, const float* g_x_edge,
                      int64_t g_x_edge_stride, const float* g_wigner, const float* g_env, int64_t E, int32_t B,
                      float* g_shifts, void* stream);
/* ...and the deterministic per-atom reduction that replaces the reference's fp32 atomics
 * (ops/geom.py:483-488): g_pos[n] = sum_{src CSR n} g_vec - sum_{dst CSR n} g_vec (fp64 sums). */
int fuma_edge_vec_to_nodes(const int32_t* src_row_ptr, const int32_t* src_col, const int32_t* dst_row_ptr,
                           const int32_t* dst_col, const float* g_vec, int64_t N, int64_t E, float* g_pos,
                           void* stream);

/* ---- fused LayerNorm + SiLU -------------------------------------------------------------
 * Replaces _LayerNormSiLUFn (ops/ln_silu.py:126-185): x[M,D] -> out[M,D], mean[M], rstd[M].
 * D a multiple of 4, D <= 2048. */
int fuma_ln_silu_fwd(const float* x, const float* gamma, const float* beta, float eps, int64_t M, int32_t D,
                     float* out, float* mean, float* rstd, void* stream);
/* dx only (gamma/beta are frozen), ops/ln_silu.py:156-177. */
int fuma_ln_silu_bwd(const float* x, const float* gamma, const float* beta, const float* mean, const float* rstd,
                     const float* g_out, int64_t M, int32_t D, float* g_x, void* stream);

/* ---- gather + rotate into the edge frame ------------------------------------------------
 * Replaces GatherWignerSplit.forward (ops/gather.py:408-433, kernel :34-154).
 * x[N,9,C], wigner[E,34], rad[E,12C], csd[nsys,C], batch[N] -> X_m0[E,6C], X_m1[E,8C], X_m2[E,4C]. */
int fuma_gather_fwd(const float* x, const int64_t* idx_i, const int64_t* idx_j, const float* wigner,
                    const float* rad, const float* csd, const int64_t* batch, int64_t N, int64_t E, int32_t C,
                    float* X_m0, float* X_m1, float* X_m2, void* stream);
/* Replaces GatherWignerSplit.backward (ops/gather.py:435-514) without atomics: needs the
 * destination CSR (dst_row_ptr[N+1], dst_col[E]) and source CSR of the same edges (a target-
 * side pass over the first, a source-side pass over the second). Writes g_x[N,9,C],
 * g_wigner[E,34], g_rad[E,12C]. scratch / scratch_floats are unused (may be NULL / 0); they
 * stay in the signature for callers written against the earlier scratch-row version. */
int fuma_gather_bwd(const float* g_X_m0, const float* g_X_m1, const float* g_X_m2, const float* x,
                    const int64_t* idx_i, const float* wigner, const float* rad, const float* csd,
                    const int64_t* batch, const int32_t* dst_row_ptr, const int32_t* dst_col,
                    const int32_t* src_row_ptr, const int32_t* src_col, int64_t N, int64_t E, int32_t C,
                    float* scratch, int64_t scratch_floats, float* g_x, float* g_wigner, float* g_rad, void* stream);

/* ---- split gating -----------------------------------------------------------------------
 * Replaces FusedGatingSplit (ops/gating.py:188-236): Y_m0[E,5C], Y_m1[E,4C], Y_m2[E,2C] ->
 * Z_m0[E,3C], Z_m1[E,4C], Z_m2[E,2C]. */
int fuma_gating_fwd(const float* Y_m0, const float* Y_m1, const float* Y_m2, int64_t E, int32_t C, float* Z_m0,
                    float* Z_m1, float* Z_m2, void* stream);
int fuma_gating_bwd(const float* g_Z_m0, const float* g_Z_m1, const float* g_Z_m2, const float* Y_m0,
                    const float* Y_m1, const float* Y_m2, int64_t E, int32_t C, float* g_Y_m0, float* g_Y_m1,
                    float* g_Y_m2, void* stream);

/* ---- rotate back + envelope + FP64 CSR segment sum + residual ----------------------------
 * Replaces RotateScatterSplit.forward (ops/scatter.py:295-315, kernel :45-140).
 * Z_m0[E,3C], Z_m1[E,4C], Z_m2[E,2C], wigner, env, x_res[N,9,C], dst CSR -> x_out[N,9,C]. */
int fuma_rotate_scatter_fwd(const float* Z_m0, const float* Z_m1, const float* Z_m2, const float* wigner,
                            const float* env, const float* x_res, const int32_t* row_ptr, const int32_t* col_idx,
                            int64_t N, int64_t E, int32_t C, float* x_out, void* stream);
/* Replaces RotateScatterSplit.backward (ops/scatter.py:317-352); g_x_res equals g_out. */
int fuma_rotate_scatter_bwd(const float* g_out, const float* Z_m0, const float* Z_m1, const float* Z_m2,
                            const float* wigner, const float* env, const int32_t* row_ptr, const int32_t* col_idx,
                            int64_t N, int64_t E, int32_t C, float* g_Z_m0, float* g_Z_m1, float* g_Z_m2,
                            float* g_wigner, float* g_env, void* stream);

/* ---- initial (edge-degree) node embedding -----------------------------------------------
 * Replaces InitNodeScatter.forward (ops/scatter.py:484-501, kernel :360-423).
 * rad[E,3C], wigner, env, Z[N], batch[N], W_sphere[num_z,C], csd[nsys,C], dst CSR -> x[N,9,C]. */
int fuma_init_scatter_fwd(const float* rad, const float* wigner, const float* env, const int64_t* Z,
                          const int64_t* batch, const float* W_sphere, const float* csd, const int32_t* row_ptr,
                          const int32_t* col_idx, int64_t N, int64_t E, int32_t C, float* x_out, void* stream);
/* Replaces InitNodeScatter.backward (ops/scatter.py:503-525, kernel :426-481) for g_rad,
 * g_wigner (full 34-wide rows, zeros outside the m=0 rows) and g_env. */
int fuma_init_scatter_bwd(const float* g_out, const float* rad, const float* wigner, const float* env,
                          const int32_t* row_ptr, const int32_t* col_idx, int64_t N, int64_t E, int32_t C,
                          float* g_rad, float* g_wigner, float* g_env, void* stream);

/* ---- dense contractions on tcgen05 tensor cores ------------------------------------------
 * Replaces the F.linear (cuBLAS) calls of the radial MLP and SO(2) convolutions
 * (model.py:147-154, weights packed at model.py:101-141) and their input gradients:
 * C[M,N] = A[M,K] . W[N,K]^T (+ bias[N]); A rows lda floats apart, C rows ldc floats apart.
 * split != 0: 3xTF32 (fp32-level accuracy); W_hi / W_lo come from fuma_split_tf32(W).
 * split == 0: single-pass TF32 with W_hi = W (W_lo unused).
 * N a multiple of 16, K a multiple of 4, lda and ldc multiples of 4.
 * err_flag (device int, may be NULL) receives a non-zero code if a pipeline wait of the
 * kernel timed out; the kernel then returns without writing C. */
int fuma_linear(const float* A, int64_t lda, const float* W_hi, const float* W_lo, const float* bias, int64_t M,
                int32_t N, int32_t K, int32_t split, float* C, int64_t ldc, int* err_flag, void* stream);
/* hi = x rounded to nearest TF32, lo = (x - hi) rounded to nearest TF32 (3xTF32 weight split). */
int fuma_split_tf32(const float* x, int64_t n, float* hi, float* lo, void* stream);
/* Same contraction as fuma_linear (same reference call sites) in the f16x3 mode: fp16 tensor
 * cores with fp32-level accuracy. Both operands are split as x = hi + lo * 2^-11 with
 * hi = fp16(x), lo = fp16((x - hi) * 2^11). The weight split (W_hi, W_lo: fp16 [N, ldw] of
 * W * scale) comes from fuma_split_f16 and w_scale_inv = 1 / scale is applied in the epilogue.
 * a_split == 0: A is fp32 [M, lda] and the kernel splits it in shared memory.
 * a_split == 1: A is the row-packed split from fuma_split_rows_f16 (lda = its ldp, a multiple
 *               of 8), the fast path: no conversion inside the GEMM.
 * K a multiple of 4, ldw >= K a multiple of 8. err_flag additionally receives 16 when an
 * activation is finite in fp32 but beyond the fp16 range (|x| >= 65520); use fuma_linear for
 * such data. */
int fuma_linear_f16x3(const float* A, int64_t lda, int32_t a_split, const void* W_hi, const void* W_lo, int64_t ldw,
                      float w_scale_inv, const float* bias, int64_t M, int32_t N, int32_t K, float* C, int64_t ldc,
                      int* err_flag, void* stream);
/* Same contraction (same reference call sites) in the single-product mode: C = A_hi . W_hi^T
 * * w_scale_inv (+ bias), fp16 operands with fp32 accumulation - the accuracy class of TF32
 * (about 11 significant bits per operand, what the reference runs with allow_tf32, its published
 * setting) at a third of the f16x3 tensor work. A is a row-packed split (the layout of
 * fuma_split_rows_f16 and of the *_f16x3 producers; only its hi half is read), W_hi the hi half
 * of fuma_split_f16. K a multiple of 8; lda, ldw multiples of 8. c_half != 0: C is fp16 [M, ldc]
 * (ldc in halves, a multiple of 8; the 16-bit activation storage of this mode; a finite result at
 * or beyond the fp16 limit sets code 16 in err_flag), else fp32. */
int fuma_linear_f16(const float* A, int64_t lda, const void* W_hi, int64_t ldw, float w_scale_inv, const float* bias,
                    int64_t M, int32_t N, int32_t K, void* C, int64_t ldc, int32_t c_half, int* err_flag,
                    void* stream);
/* Row-packed f16x3 split of an activation matrix x [M, K] (rows lda floats apart) into out,
 * whose row r spans 4 * ldp bytes: fp16 hi values of x[r, :K] at byte 0, the scaled fp16 lo
 * values at byte 2 * ldp (the same footprint as fp32 [M, ldp]). ldp >= K, a multiple of 8.
 * err_flag receives 16 on an out-of-range value. */
int fuma_split_rows_f16(const float* x, int64_t lda, int64_t M, int32_t K, void* out, int64_t ldp, int* err_flag,
                        void* stream);
/* Equivariant RMS norm of node embeddings x [N, 9, C] (the norm_1 / norm_2 / final_norm
 * modules the reference's layers call, model.py:145,157,218; here the stand-in
 * EquivariantRMSNormSH): l = 0 row centred over channels, all rows scaled by
 * 1 / sqrt(mean_c sum_k w_k f_k^2 + eps) with degree_weight w [9], then by affine_weight
 * [3, C] (per degree) and affine_bias [C] (l = 0). rstd [N] receives the per-atom scale for the
 * backward, which returns g_x (frozen affine parameters). C a multiple of 4, at most 256. */
int fuma_rmsnorm_sh_fwd(const float* x, const float* affine_weight, const float* affine_bias,
                        const float* degree_weight, float eps, int64_t N, int32_t C, float* out, float* rstd,
                        void* stream);
int fuma_rmsnorm_sh_bwd(const float* x, const float* affine_weight, const float* degree_weight, const float* rstd,
                        const float* g_out, int64_t N, int32_t C, float* g_x, void* stream);
/* Gated atom-wise block (the atom_wise module the reference's layers call, model.py:157; here
 * the stand-in SpectralAtomwise). h [9N, H]: the per-coefficient output of its first
 * per-degree linear map without bias, coefficient-major; u [N, 2H]: its scalar MLP
 * pre-activation (bias included). z_0 = SiLU(h_0 + b1), z_k = h_k sigmoid(SiLU(u))[degree - 1]
 * for k >= 1, written [9, N, H]. The backward returns gh [9, N, H] and gu [N, 2H] from gz.
 * H a multiple of 4. */
int fuma_atomwise_gate_fwd(const float* h, const float* u, const float* b1, int64_t N, int32_t H, float* z,
                           void* stream);
int fuma_atomwise_gate_bwd(const float* gz, const float* h, const float* u, const float* b1, int64_t N, int32_t H,
                           float* gh, float* gu, void* stream);
/* out[n, k, :] = src[k, n, :] + add[n, k, :] (add may be NULL) + row0 on k = 0 (row0 [N, W] when
 * row0_per_node, else [W]; may be NULL): coefficient-major [9, N, W] rows back to the node-major
 * [N, 9, W] embedding layout. W a multiple of 4. */
int fuma_coef_to_node(const float* src, const float* add, const float* row0, int32_t row0_per_node, int64_t N,
                      int32_t W, float* out, void* stream);
/* The same block with its per-degree linear maps on the fp16 tensor cores (fuma_linear_f16x3 /
 * fuma_linear_f16); no counterpart in the reference, whose atom_wise module is FAIRChem code.
 * Coefficient rows: row k * N + n holds coefficient k of atom n. Each map is ONE GEMM over all
 * 9N rows against the three degree weights stacked ([W_0; W_1; W_2]); its output is
 * "degree-blocked" [9N, 3 * width]: row k * N + n, column block deg(k) * width (deg 0 for k = 0,
 * 1 for k = 1..3, 2 for k = 4..8) is the product with coefficient k's own weight.
 * - fuma_node_to_coef_f16x3: x [N, 9, W] -> the row-packed split (parts 1 or 2, as for the
 *   producer entry points below) of its coefficient rows [9N, W]; W a multiple of 8.
 * - fuma_atomwise_gate_fwd_f16x3: h degree-blocked [9N, 3H] -> z, the row-packed split [9N, H].
 * - fuma_atomwise_gate_bwd_f16x3: gz and h degree-blocked [9N, 3H] -> gh split [9N, H] and
 *   gu split [N, 2H]. H a multiple of 8.
 * - fuma_coef_to_node_blocked: fuma_coef_to_node with src degree-blocked [9N, 3W].
 * err_flag receives 16 on a value beyond the fp16 range. */
int fuma_node_to_coef_f16x3(const float* x, int64_t N, int32_t W, float* out, int32_t parts, int* err_flag,
                            void* stream);
int fuma_atomwise_gate_fwd_f16x3(const float* h, const float* u, const float* b1, int64_t N, int32_t H, float* z,
                                 int32_t parts, int* err_flag, void* stream);
int fuma_atomwise_gate_bwd_f16x3(const float* gz, const float* h, const float* u, const float* b1, int64_t N,
                                 int32_t H, float* gh, float* gu, int32_t parts, int* err_flag, void* stream);
int fuma_coef_to_node_blocked(const float* src, const float* add, const float* row0, int32_t row0_per_node,
                              int64_t N, int32_t W, float* out, void* stream);
/* Morton order of the atoms and the renumbered graph (replaces reorder_graph_morton,
 * model.py:47-74): 30-bit codes of the positions quantised to 10 bits per axis over their
 * bounding box, a stable sort by (system << 32 | code), perm [N] (new -> old) and inv_perm [N],
 * the permuted pos_s [N, 3] (may be NULL), Z_s and batch_s [N], and the renumbered edge rows
 * ii = inv_perm[idx_i], jj = inv_perm[idx_j] [E]. Same arithmetic and order as the reference.
 * System ids must be non-negative. Up to 16,384 atoms one block sorts in shared memory and no
 * scratch is needed; above that a multi-block radix sort uses scratch_bytes >=
 * fuma_morton_scratch_bytes(N) bytes of device scratch (256-byte aligned, contents irrelevant;
 * about 24 bytes per atom). An edge index outside [0, N) sets code 32 in err_flag (device int,
 * may be NULL) and renumbers that edge to atom 0. */
int64_t fuma_morton_scratch_bytes(int64_t N);
int fuma_morton_reorder(const float* pos, const int64_t* Z, const int64_t* batch, const int64_t* idx_i,
                        const int64_t* idx_j, int64_t N, int64_t E, int64_t* perm, int64_t* inv_perm, float* pos_s,
                        int64_t* Z_s, int64_t* batch_s, int64_t* ii, int64_t* jj, void* scratch,
                        int64_t scratch_bytes, int* err_flag, void* stream);
/* Deterministic capped periodic neighbour list. Replaces the graph generation the reference
 * leaves to FAIRChem / pymatgen outside its backbone (readme.md:35-72, external_graph_gen; its
 * output is the edge_index / cell_offsets the backbone reads at wrapper.py:171-197), with this
 * build's deterministic rule: every (source i, destination j, integer offset s) with
 * |pos_i - pos_j + s @ cell| < cutoff (self pairs only with s != 0), per destination ordered by
 * (distance, i, s_0, s_1, s_2) in fp64, the first max_neighbors kept.
 * pos [N, 3] fp64 (device). geom (HOST memory): cell [3, 3] row-major (rows = lattice vectors)
 * then its inverse [3, 3]. grid (HOST memory, int32 [12]): bins per axis nb[3] (fractional bins
 * of side >= cutoff), the bin-offset range lo[3], hi[3] searched around an atom's bin (periodic
 * images included), pbc[3] (0/1). Outputs per destination d (device): counts[d], and for its
 * r < counts[d] neighbours src[d * max + r], offsets[(d * max + r) * 3 + k] (int64), dist[d *
 * max + r] (fp64). Scratch: fuma_neighbor_scratch_bytes(N, grid) bytes, 256-byte aligned.
 * More than 512 candidates for one destination sets code 64 in err_flag (device int, may be
 * NULL). Integer offsets must stay within +-511. */
int64_t fuma_neighbor_scratch_bytes(int64_t N, const int32_t* grid);
int fuma_neighbor_list(const double* pos, int64_t N, const double* geom, const int32_t* grid, double cutoff,
                       int32_t max_neighbors, void* scratch, int64_t scratch_bytes, int32_t* counts, int64_t* src,
                       int64_t* offsets, double* dist, int* err_flag, void* stream);

/* Destination (and optionally source) CSR of a renumbered edge list, from the CSR of the
 * original numbering: new node a is original node perm[a] (perm: int64 [N]), edge ids are
 * unchanged. Replaces the per-step stable-argsort CSR build of the reference on its renumbered
 * (Morton-ordered) edges (model.py:17-46, called at model.py:189-191): the result is bitwise
 * that CSR, since row a holds the edges of node perm[a] in increasing edge id. Inputs and
 * outputs are int32 [N + 1] row pointers and [E] columns (edge ids); src_* may all be NULL. */
int fuma_csr_permute(const int32_t* dst_row_ptr, const int32_t* dst_col, const int32_t* src_row_ptr,
                     const int32_t* src_col, const int64_t* perm, int64_t N, int64_t E, int32_t* new_dst_row_ptr,
                     int32_t* new_dst_col, int32_t* new_src_row_ptr, int32_t* new_src_col, void* stream);
/* hi = fp16_rn(x * scale), lo = fp16_rn((x * scale - hi) * 2^11), n elements (f16x3 weight split). */
int fuma_split_f16(const float* x, int64_t n, float scale, void* hi, void* lo, void* stream);

/* ---- split-output variants for the f16x3 GEMM -----------------------------------------------
 * No counterpart in the reference (its GEMM inputs are plain fp32 tensors). Each takes the
 * arguments of the entry point without the suffix plus err_flag, and writes the outputs that
 * feed a dense contraction in the row-packed f16x3 split layout of fuma_split_rows_f16
 * (ldp = the output's row width) instead of fp32, so fuma_linear_f16x3 (a_split = 1) reads
 * them without a conversion pass:
 *   ln_silu_fwd: out          ln_silu_bwd: g_x              gather_fwd: X_m0, X_m1, X_m2
 *   gather_bwd: g_rad         gating_fwd: Z_m0, Z_m1, Z_m2  gating_bwd: g_Y_m0, g_Y_m1, g_Y_m2
 *   rotate_scatter_bwd: g_Z_m0, g_Z_m1, g_Z_m2              init_scatter_bwd: g_rad
 * parts = 2 writes both halves of every split row (the operand of fuma_linear_f16x3); parts = 1
 * writes only the fp16 hi halves (the operand of the single-product fuma_linear_f16, which reads
 * nothing else; the lo halves of the rows are left as they are, so the call moves half the
 * bytes). All other outputs are unchanged. C (D for ln_silu) must be a multiple of 8. err_flag
 * (device int, may be NULL) receives 16 if a finite value is at or beyond the fp16 limit (65520).
 * act_half != 0 (gather, gating and rotate-scatter variants; the 16-bit storage of the
 * single-product mode, where fuma_linear_f16 writes its results as fp16 with c_half): the radial
 * rows `rad` (gather fwd / bwd), the conv1 results Y_m0..2 (gating fwd / bwd), the conv2
 * results Z_m0..2 (rotate-scatter fwd / bwd) and the input gradients read by the backward
 * variants, g_X_m0..2 (gather bwd) and g_Z_m0..2 (gating bwd), are fp16 arrays of the same
 * shapes, passed as the same pointers; everything else stays fp32.
 * fuma_rotate_scatter_fwd_f16x3 is fuma_rotate_scatter_fwd with that flag. */
int fuma_ln_silu_fwd_f16x3(const float* x, const float* gamma, const float* beta, float eps, int64_t M, int32_t D,
                           float* out, float* mean, float* rstd, int32_t parts, int* err_flag, void* stream);
int fuma_ln_silu_bwd_f16x3(const float* x, const float* gamma, const float* beta, const float* mean,
                           const float* rstd, const float* g_out, int64_t M, int32_t D, float* g_x, int32_t parts, int* err_flag,
                           void* stream);
int fuma_gather_fwd_f16x3(const float* x, const int64_t* idx_i, const int64_t* idx_j, const float* wigner,
                          const float* rad, const float* csd, const int64_t* batch, int64_t N, int64_t E, int32_t C,
                          float* X_m0, float* X_m1, float* X_m2, int32_t parts, int32_t act_half, int* err_flag, void* stream);
int fuma_gather_bwd_f16x3(const float* g_X_m0, const float* g_X_m1, const float* g_X_m2, const float* x,
                          const int64_t* idx_i, const float* wigner, const float* rad, const float* csd,
                          const int64_t* batch, const int32_t* dst_row_ptr, const int32_t* dst_col,
                          const int32_t* src_row_ptr, const int32_t* src_col, int64_t N, int64_t E, int32_t C,
                          float* scratch, int64_t scratch_floats, float* g_x, float* g_wigner, float* g_rad,
                          int32_t parts, int32_t act_half, int* err_flag, void* stream);
int fuma_rotate_scatter_fwd_f16x3(const float* Z_m0, const float* Z_m1, const float* Z_m2, const float* wigner,
                                  const float* env, const float* x_res, const int32_t* row_ptr, const int32_t* col_idx,
                                  int64_t N, int64_t E, int32_t C, float* x_out, int32_t act_half, void* stream);
int fuma_gating_fwd_f16x3(const float* Y_m0, const float* Y_m1, const float* Y_m2, int64_t E, int32_t C, float* Z_m0,
                          float* Z_m1, float* Z_m2, int32_t parts, int32_t act_half, int* err_flag, void* stream);
int fuma_gating_bwd_f16x3(const float* g_Z_m0, const float* g_Z_m1, const float* g_Z_m2, const float* Y_m0,
                          const float* Y_m1, const float* Y_m2, int64_t E, int32_t C, float* g_Y_m0, float* g_Y_m1,
                          float* g_Y_m2, int32_t parts, int32_t act_half, int* err_flag, void* stream);
int fuma_rotate_scatter_bwd_f16x3(const float* g_out, const float* Z_m0, const float* Z_m1, const float* Z_m2,
                                  const float* wigner, const float* env, const int32_t* row_ptr,
                                  const int32_t* col_idx, int64_t N, int64_t E, int32_t C, float* g_Z_m0,
                                  float* g_Z_m1, float* g_Z_m2, float* g_wigner, float* g_env, int32_t parts, int32_t act_half, int* err_flag,
                                  void* stream);
int fuma_init_scatter_bwd_f16x3(const float* g_out, const float* rad, const float* wigner, const float* env,
                                const int32_t* row_ptr, const int32_t* col_idx, int64_t N, int64_t E, int32_t C,
                                float* g_rad, float* g_wigner, float* g_env, int32_t parts, int* err_flag, void* stream);

/* ---- allocation-free Morton reorder -------------------------------------------------------
 * No counterpart in the reference. For callers that cannot allocate device memory or lend a
 * device allocator at the point of the call (host programs that own the whole device memory
 * budget, steps that must not pay for or be serialised by cudaMalloc / cudaFree, bindings that
 * only pass the caller's arrays): the same computation and outputs as fuma_morton_reorder, but
 * its radix-sort scratch lives in a 13 MiB array built into the library (held on every GPU that
 * loads it until the process exits), so only inputs and outputs are passed. Limit: N <= 524,288
 * atoms; larger calls return FUMA_E_INVALID before launching anything. The first call on a device
 * looks up the array's address; make it before any stream capture. All calls share the array
 * and it keeps the last call's contents (nothing in it needs to start at zero); calls that can
 * overlap on the GPU race on it and must be serialised by the caller. Allocates nothing. */
int fuma_morton_reorder_noalloc(const float* pos, const int64_t* Z, const int64_t* batch, const int64_t* idx_i,
                                const int64_t* idx_j, int64_t N, int64_t E, int64_t* perm, int64_t* inv_perm,
                                float* pos_s, int64_t* Z_s, int64_t* batch_s, int64_t* ii, int64_t* jj, int* err_flag,
                                void* stream);

#ifdef __cplusplus
}
#endif
#endif /* FLASH_UMA_B200_H */
