// extern "C" entry points: argument validation, launch configuration, error reporting.
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "../../include/flash_uma_b200.h"
#include "common.cuh"
#include "kernels.h"

using namespace fuma;

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int launched(const char* what) {
  const cudaError_t st = cudaGetLastError();
  if (st != cudaSuccess) return fail((int)st, "%s: launch failed: %s", what, cudaGetErrorString(st));
  g_err[0] = '\0';
  return FUMA_OK;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Make the device that owns `p` current on the calling thread (and its primary context
// current for driver-API calls). Callers such as PyTorch's autograd worker threads may
// have no current context, or a different current device, when they call in.
int bind_device(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return fail(FUMA_E_INVALID, "pointer %p is not a CUDA allocation", p);
  }
  if (a.type != cudaMemoryTypeDevice && a.type != cudaMemoryTypeManaged)
    return fail(FUMA_E_INVALID, "pointer %p is not device memory", p);
  const cudaError_t st = cudaSetDevice(a.device);
  if (st != cudaSuccess) return fail((int)st, "cudaSetDevice(%d): %s", a.device, cudaGetErrorString(st));
  return FUMA_OK;
}

#define BIND(p)                            \
  do {                                     \
    if (int rc_ = bind_device(p)) return rc_; \
  } while (0)

#define REQUIRE(cond, ...)                                  \
  do {                                                      \
    if (!(cond)) return fail(FUMA_E_INVALID, __VA_ARGS__);  \
  } while (0)
#define REQUIRE_ALIGNED(p, name)                                                     \
  do {                                                                               \
    if (!al16(p)) return fail(FUMA_E_ALIGN, "%s must be 16-byte aligned", name);     \
  } while (0)

int check_C(int32_t C) {
  if (C <= 0 || (C & 3) != 0 || C > 512) return fail(FUMA_E_INVALID, "C=%d must be a positive multiple of 4, <= 512", C);
  return FUMA_OK;
}

}  // namespace

int fuma::bind_device_of(const void* p) { return bind_device(p); }

int fuma::launch_status(const char* what) { return launched(what); }

int fuma::report_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

extern "C" {

int fuma_version(void) { return 100; }
const char* fuma_last_error(void) { return g_err; }

int fuma_geometry_fwd(const float* pos, const int64_t* Z, const int64_t* idx_i, const int64_t* idx_j,
                      const float* shifts, const float* W_src, const float* W_tgt, const float* offset_g,
                      float coeff_g, float cutoff, int64_t N, int64_t E, int32_t B, int32_t C, float* x_edge_raw,
                      float* wigner, float* env, void* stream) {
  REQUIRE(N >= 0 && E >= 0 && B > 0 && C > 0, "geometry_fwd: bad sizes N=%lld E=%lld B=%d C=%d", (long long)N,
          (long long)E, B, C);
  REQUIRE(cutoff > 0.f, "geometry_fwd: cutoff must be > 0");
  if (E == 0) return FUMA_OK;
  REQUIRE(pos && Z && idx_i && idx_j && shifts && W_src && W_tgt && offset_g && x_edge_raw && wigner && env,
          "geometry_fwd: null pointer");
  if (((B | C) & 3) == 0) {
    REQUIRE_ALIGNED(x_edge_raw, "x_edge_raw"); REQUIRE_ALIGNED(W_src, "W_src"); REQUIRE_ALIGNED(W_tgt, "W_tgt");
  }
  BIND(pos);
  launch_geom_fwd(pos, Z, idx_i, idx_j, shifts, W_src, W_tgt, offset_g, x_edge_raw, wigner, env, E, B, C, cutoff,
                  coeff_g, (cudaStream_t)stream);
  return launched("geometry_fwd");
}

int fuma_geometry_bwd(const float* pos, const int64_t* idx_i, const int64_t* idx_j, const float* shifts,
                      const float* offset_g, float coeff_g, float cutoff, const float* g_x_edge,
                      int64_t g_x_edge_stride, const float* g_wigner, const float* g_env, int64_t E, int32_t B,
                      float* g_shifts, void* stream) {
  REQUIRE(E >= 0 && B > 0 && g_x_edge_stride >= B, "geometry_bwd: bad sizes");
  if (E == 0) return FUMA_OK;
  REQUIRE(pos && idx_i && idx_j && shifts && offset_g && g_x_edge && g_wigner && g_env && g_shifts,
          "geometry_bwd: null pointer");
  BIND(pos);
  launch_geom_bwd(pos, idx_i, idx_j, shifts, offset_g, g_x_edge, g_x_edge_stride, g_wigner, g_env, g_shifts, E, B,
                  cutoff, coeff_g, (cudaStream_t)stream);
  return launched("geometry_bwd");
}

int fuma_edge_vec_to_nodes(const int32_t* src_row_ptr, const int32_t* src_col, const int32_t* dst_row_ptr,
                           const int32_t* dst_col, const float* g_vec, int64_t N, int64_t E, float* g_pos,
                           void* stream) {
  REQUIRE(N >= 0 && E >= 0, "edge_vec_to_nodes: bad sizes");
  if (N == 0) return FUMA_OK;
  REQUIRE(src_row_ptr && dst_row_ptr && g_pos, "edge_vec_to_nodes: null pointer");
  REQUIRE(E == 0 || (src_col && dst_col && g_vec), "edge_vec_to_nodes: null per-edge pointer");
  BIND(g_pos);
  launch_node_vec3_segment(src_row_ptr, src_col, dst_row_ptr, dst_col, g_vec, g_pos, N, (cudaStream_t)stream);
  return launched("edge_vec_to_nodes");
}

static int ln_silu_fwd_impl(const float* x, const float* gamma, const float* beta, float eps, int64_t M, int32_t D,
                     float* out, float* mean, float* rstd, int split, int* err_flag, void* stream) {
  REQUIRE(!split || D % 8 == 0, "ln_silu_fwd_f16x3: the split output needs D %% 8 == 0");
  REQUIRE(M >= 0 && D > 0 && (D & 3) == 0 && D <= 2048, "ln_silu_fwd: D=%d must be a multiple of 4, <= 2048", D);
  if (M == 0) return FUMA_OK;
  REQUIRE(x && gamma && beta && out && mean && rstd, "ln_silu_fwd: null pointer");
  REQUIRE_ALIGNED(x, "x"); REQUIRE_ALIGNED(out, "out"); REQUIRE_ALIGNED(gamma, "gamma"); REQUIRE_ALIGNED(beta, "beta");
  BIND(x);
  launch_ln_silu_fwd(x, gamma, beta, out, mean, rstd, M, D, eps, split, err_flag, (cudaStream_t)stream);
  return launched("ln_silu_fwd");
}

int fuma_ln_silu_fwd(const float* x, const float* gamma, const float* beta, float eps, int64_t M, int32_t D,
                     float* out, float* mean, float* rstd, void* stream) {
  return ln_silu_fwd_impl(x, gamma, beta, eps, M, D, out, mean, rstd, false, nullptr, stream);
}

int fuma_ln_silu_fwd_f16x3(const float* x, const float* gamma, const float* beta, float eps, int64_t M, int32_t D,
                     float* out, float* mean, float* rstd, int32_t parts, int* err_flag, void* stream) {
  REQUIRE(parts == 1 || parts == 2, "ln_silu_fwd_f16x3: parts=%d must be 1 (hi) or 2 (hi and lo)", parts);
  return ln_silu_fwd_impl(x, gamma, beta, eps, M, D, out, mean, rstd, parts, err_flag, stream);
}

static int ln_silu_bwd_impl(const float* x, const float* gamma, const float* beta, const float* mean, const float* rstd,
                     const float* g_out, int64_t M, int32_t D, float* g_x, int split, int* err_flag, void* stream) {
  REQUIRE(!split || D % 8 == 0, "ln_silu_bwd_f16x3: the split output needs D %% 8 == 0");
  REQUIRE(M >= 0 && D > 0 && (D & 3) == 0 && D <= 2048, "ln_silu_bwd: D=%d must be a multiple of 4, <= 2048", D);
  if (M == 0) return FUMA_OK;
  REQUIRE(x && gamma && beta && mean && rstd && g_out && g_x, "ln_silu_bwd: null pointer");
  REQUIRE_ALIGNED(x, "x"); REQUIRE_ALIGNED(g_out, "g_out"); REQUIRE_ALIGNED(g_x, "g_x");
  BIND(x);
  launch_ln_silu_bwd(x, gamma, beta, mean, rstd, g_out, g_x, M, D, split, err_flag, (cudaStream_t)stream);
  return launched("ln_silu_bwd");
}

int fuma_ln_silu_bwd(const float* x, const float* gamma, const float* beta, const float* mean, const float* rstd,
                     const float* g_out, int64_t M, int32_t D, float* g_x, void* stream) {
  return ln_silu_bwd_impl(x, gamma, beta, mean, rstd, g_out, M, D, g_x, false, nullptr, stream);
}

int fuma_ln_silu_bwd_f16x3(const float* x, const float* gamma, const float* beta, const float* mean, const float* rstd,
                     const float* g_out, int64_t M, int32_t D, float* g_x, int32_t parts, int* err_flag, void* stream) {
  REQUIRE(parts == 1 || parts == 2, "ln_silu_bwd_f16x3: parts=%d must be 1 (hi) or 2 (hi and lo)", parts);
  return ln_silu_bwd_impl(x, gamma, beta, mean, rstd, g_out, M, D, g_x, parts, err_flag, stream);
}

static int gather_fwd_impl(const float* x, const int64_t* idx_i, const int64_t* idx_j, const float* wigner,
                    const float* rad, const float* csd, const int64_t* batch, int64_t N, int64_t E, int32_t C,
                    float* X_m0, float* X_m1, float* X_m2, int split, bool act_half, int* err_flag, void* stream) {
  REQUIRE(!split || C % 8 == 0, "gather_fwd_f16x3: the split output needs C %% 8 == 0");
  if (int r = check_C(C)) return r;
  REQUIRE(N >= 0 && E >= 0, "gather_fwd: bad sizes");
  if (E == 0) return FUMA_OK;
  REQUIRE(x && idx_i && idx_j && wigner && rad && csd && batch && X_m0 && X_m1 && X_m2, "gather_fwd: null pointer");
  REQUIRE_ALIGNED(x, "x"); REQUIRE_ALIGNED(rad, "rad"); REQUIRE_ALIGNED(csd, "csd");
  REQUIRE_ALIGNED(X_m0, "X_m0"); REQUIRE_ALIGNED(X_m1, "X_m1"); REQUIRE_ALIGNED(X_m2, "X_m2");
  BIND(x);
  launch_gather_fwd(x, idx_i, idx_j, wigner, rad, csd, batch, X_m0, X_m1, X_m2, E, C, split, err_flag, (cudaStream_t)stream, act_half);
  return launched("gather_fwd");
}

int fuma_gather_fwd(const float* x, const int64_t* idx_i, const int64_t* idx_j, const float* wigner,
                    const float* rad, const float* csd, const int64_t* batch, int64_t N, int64_t E, int32_t C,
                    float* X_m0, float* X_m1, float* X_m2, void* stream) {
  return gather_fwd_impl(x, idx_i, idx_j, wigner, rad, csd, batch, N, E, C, X_m0, X_m1, X_m2, false, false, nullptr, stream);
}

int fuma_gather_fwd_f16x3(const float* x, const int64_t* idx_i, const int64_t* idx_j, const float* wigner,
                    const float* rad, const float* csd, const int64_t* batch, int64_t N, int64_t E, int32_t C,
                    float* X_m0, float* X_m1, float* X_m2, int32_t parts, int32_t act_half, int* err_flag, void* stream) {
  REQUIRE(parts == 1 || parts == 2, "gather_fwd_f16x3: parts=%d must be 1 (hi) or 2 (hi and lo)", parts);
  return gather_fwd_impl(x, idx_i, idx_j, wigner, rad, csd, batch, N, E, C, X_m0, X_m1, X_m2, parts, act_half != 0, err_flag, stream);
}

static int gather_bwd_impl(const float* g_X_m0, const float* g_X_m1, const float* g_X_m2, const float* x,
                    const int64_t* idx_i, const float* wigner, const float* rad, const float* csd,
                    const int64_t* batch, const int32_t* dst_row_ptr, const int32_t* dst_col,
                    const int32_t* src_row_ptr, const int32_t* src_col, int64_t N, int64_t E, int32_t C,
                    float* scratch, int64_t scratch_floats, float* g_x, float* g_wigner, float* g_rad,
                    int split, bool act_half, int* err_flag, void* stream) {
  REQUIRE(!split || C % 8 == 0, "gather_bwd_f16x3: the split output needs C %% 8 == 0");
  if (int r = check_C(C)) return r;
  REQUIRE(N >= 0 && E >= 0, "gather_bwd: bad sizes");
  if (N == 0) return FUMA_OK;
  REQUIRE(x && csd && batch && dst_row_ptr && src_row_ptr && g_x, "gather_bwd: null pointer");
  REQUIRE(E == 0 || (idx_i && wigner && rad && dst_col && src_col && g_wigner && g_rad && g_X_m0 && g_X_m1 && g_X_m2),
          "gather_bwd: null per-edge pointer");
  (void)scratch;
  (void)scratch_floats;   // unused since the backward runs as two passes (source / target side)
  REQUIRE_ALIGNED(x, "x"); REQUIRE_ALIGNED(csd, "csd"); REQUIRE_ALIGNED(g_x, "g_x");
  if (E > 0) {
    REQUIRE_ALIGNED(rad, "rad"); REQUIRE_ALIGNED(g_rad, "g_rad"); REQUIRE_ALIGNED(g_X_m0, "g_X_m0");
    REQUIRE_ALIGNED(g_X_m1, "g_X_m1"); REQUIRE_ALIGNED(g_X_m2, "g_X_m2");
  }
  BIND(x);
  launch_gather_bwd(g_X_m0, g_X_m1, g_X_m2, x, idx_i, wigner, rad, csd, batch, dst_row_ptr, dst_col, src_row_ptr,
                    src_col, g_x, g_wigner, g_rad, scratch, N, C, split, err_flag, (cudaStream_t)stream, act_half);
  return launched("gather_bwd");
}

int fuma_gather_bwd(const float* g_X_m0, const float* g_X_m1, const float* g_X_m2, const float* x,
                    const int64_t* idx_i, const float* wigner, const float* rad, const float* csd,
                    const int64_t* batch, const int32_t* dst_row_ptr, const int32_t* dst_col,
                    const int32_t* src_row_ptr, const int32_t* src_col, int64_t N, int64_t E, int32_t C,
                    float* scratch, int64_t scratch_floats, float* g_x, float* g_wigner, float* g_rad,
                    void* stream) {
  return gather_bwd_impl(g_X_m0, g_X_m1, g_X_m2, x, idx_i, wigner, rad, csd, batch, dst_row_ptr, dst_col, src_row_ptr,
                         src_col, N, E, C, scratch, scratch_floats, g_x, g_wigner, g_rad, false, false, nullptr, stream);
}

int fuma_gather_bwd_f16x3(const float* g_X_m0, const float* g_X_m1, const float* g_X_m2, const float* x,
                    const int64_t* idx_i, const float* wigner, const float* rad, const float* csd,
                    const int64_t* batch, const int32_t* dst_row_ptr, const int32_t* dst_col,
                    const int32_t* src_row_ptr, const int32_t* src_col, int64_t N, int64_t E, int32_t C,
                    float* scratch, int64_t scratch_floats, float* g_x, float* g_wigner, float* g_rad,
                    int32_t parts, int32_t act_half, int* err_flag, void* stream) {
  REQUIRE(parts == 1 || parts == 2, "gather_bwd_f16x3: parts=%d must be 1 (hi) or 2 (hi and lo)", parts);
  return gather_bwd_impl(g_X_m0, g_X_m1, g_X_m2, x, idx_i, wigner, rad, csd, batch, dst_row_ptr, dst_col, src_row_ptr,
                         src_col, N, E, C, scratch, scratch_floats, g_x, g_wigner, g_rad, parts, act_half != 0, err_flag, stream);
}

static int gating_fwd_impl(const float* Y_m0, const float* Y_m1, const float* Y_m2, int64_t E, int32_t C, float* Z_m0,
                    float* Z_m1, float* Z_m2, int split, bool act_half, int* err_flag, void* stream) {
  REQUIRE(!split || C % 8 == 0, "gating_fwd_f16x3: the split output needs C %% 8 == 0");
  if (int r = check_C(C)) return r;
  REQUIRE(E >= 0, "gating_fwd: bad E");
  if (E == 0) return FUMA_OK;
  REQUIRE(Y_m0 && Y_m1 && Y_m2 && Z_m0 && Z_m1 && Z_m2, "gating_fwd: null pointer");
  REQUIRE_ALIGNED(Y_m0, "Y_m0"); REQUIRE_ALIGNED(Y_m1, "Y_m1"); REQUIRE_ALIGNED(Y_m2, "Y_m2");
  REQUIRE_ALIGNED(Z_m0, "Z_m0"); REQUIRE_ALIGNED(Z_m1, "Z_m1"); REQUIRE_ALIGNED(Z_m2, "Z_m2");
  BIND(Y_m0);
  launch_gating_fwd(Y_m0, Y_m1, Y_m2, Z_m0, Z_m1, Z_m2, E, C, split, err_flag, (cudaStream_t)stream, act_half);
  return launched("gating_fwd");
}

int fuma_gating_fwd(const float* Y_m0, const float* Y_m1, const float* Y_m2, int64_t E, int32_t C, float* Z_m0,
                    float* Z_m1, float* Z_m2, void* stream) {
  return gating_fwd_impl(Y_m0, Y_m1, Y_m2, E, C, Z_m0, Z_m1, Z_m2, false, false, nullptr, stream);
}

int fuma_gating_fwd_f16x3(const float* Y_m0, const float* Y_m1, const float* Y_m2, int64_t E, int32_t C, float* Z_m0,
                    float* Z_m1, float* Z_m2, int32_t parts, int32_t act_half, int* err_flag, void* stream) {
  REQUIRE(parts == 1 || parts == 2, "gating_fwd_f16x3: parts=%d must be 1 (hi) or 2 (hi and lo)", parts);
  return gating_fwd_impl(Y_m0, Y_m1, Y_m2, E, C, Z_m0, Z_m1, Z_m2, parts, act_half != 0, err_flag, stream);
}

static int gating_bwd_impl(const float* g_Z_m0, const float* g_Z_m1, const float* g_Z_m2, const float* Y_m0,
                    const float* Y_m1, const float* Y_m2, int64_t E, int32_t C, float* g_Y_m0, float* g_Y_m1,
                    float* g_Y_m2, int split, bool act_half, int* err_flag, void* stream) {
  REQUIRE(!split || C % 8 == 0, "gating_bwd_f16x3: the split output needs C %% 8 == 0");
  if (int r = check_C(C)) return r;
  REQUIRE(E >= 0, "gating_bwd: bad E");
  if (E == 0) return FUMA_OK;
  REQUIRE(g_Z_m0 && g_Z_m1 && g_Z_m2 && Y_m0 && Y_m1 && Y_m2 && g_Y_m0 && g_Y_m1 && g_Y_m2, "gating_bwd: null pointer");
  REQUIRE_ALIGNED(g_Z_m0, "g_Z_m0"); REQUIRE_ALIGNED(g_Z_m1, "g_Z_m1"); REQUIRE_ALIGNED(g_Z_m2, "g_Z_m2");
  REQUIRE_ALIGNED(Y_m0, "Y_m0"); REQUIRE_ALIGNED(Y_m1, "Y_m1"); REQUIRE_ALIGNED(Y_m2, "Y_m2");
  REQUIRE_ALIGNED(g_Y_m0, "g_Y_m0"); REQUIRE_ALIGNED(g_Y_m1, "g_Y_m1"); REQUIRE_ALIGNED(g_Y_m2, "g_Y_m2");
  BIND(Y_m0);
  launch_gating_bwd(g_Z_m0, g_Z_m1, g_Z_m2, Y_m0, Y_m1, Y_m2, g_Y_m0, g_Y_m1, g_Y_m2, E, C, split, err_flag, (cudaStream_t)stream, act_half);
  return launched("gating_bwd");
}

int fuma_gating_bwd(const float* g_Z_m0, const float* g_Z_m1, const float* g_Z_m2, const float* Y_m0,
                    const float* Y_m1, const float* Y_m2, int64_t E, int32_t C, float* g_Y_m0, float* g_Y_m1,
                    float* g_Y_m2, void* stream) {
  return gating_bwd_impl(g_Z_m0, g_Z_m1, g_Z_m2, Y_m0, Y_m1, Y_m2, E, C, g_Y_m0, g_Y_m1, g_Y_m2, false, false, nullptr, stream);
}

int fuma_gating_bwd_f16x3(const float* g_Z_m0, const float* g_Z_m1, const float* g_Z_m2, const float* Y_m0,
                    const float* Y_m1, const float* Y_m2, int64_t E, int32_t C, float* g_Y_m0, float* g_Y_m1,
                    float* g_Y_m2, int32_t parts, int32_t act_half, int* err_flag, void* stream) {
  REQUIRE(parts == 1 || parts == 2, "gating_bwd_f16x3: parts=%d must be 1 (hi) or 2 (hi and lo)", parts);
  return gating_bwd_impl(g_Z_m0, g_Z_m1, g_Z_m2, Y_m0, Y_m1, Y_m2, E, C, g_Y_m0, g_Y_m1, g_Y_m2, parts, act_half != 0, err_flag, stream);
}

static int rotate_scatter_fwd_impl(const float* Z_m0, const float* Z_m1, const float* Z_m2, const float* wigner,
                                   const float* env, const float* x_res, const int32_t* row_ptr,
                                   const int32_t* col_idx, int64_t N, int64_t E, int32_t C, float* x_out,
                                   int32_t act_half, void* stream) {
  if (int r = check_C(C)) return r;
  REQUIRE(N >= 0 && E >= 0, "rotate_scatter_fwd: bad sizes");
  if (N == 0) return FUMA_OK;
  REQUIRE(x_res && row_ptr && x_out && (E == 0 || (Z_m0 && Z_m1 && Z_m2 && wigner && env && col_idx)),
          "rotate_scatter_fwd: null pointer");
  REQUIRE_ALIGNED(x_res, "x_res"); REQUIRE_ALIGNED(x_out, "x_out");
  if (E > 0) { REQUIRE_ALIGNED(Z_m0, "Z_m0"); REQUIRE_ALIGNED(Z_m1, "Z_m1"); REQUIRE_ALIGNED(Z_m2, "Z_m2"); }
  BIND(x_res);
  launch_rotate_scatter_fwd(row_ptr, col_idx, Z_m0, Z_m1, Z_m2, wigner, env, x_res, x_out, N, C, (cudaStream_t)stream,
                            act_half != 0);
  return launched("rotate_scatter_fwd");
}

int fuma_rotate_scatter_fwd(const float* Z_m0, const float* Z_m1, const float* Z_m2, const float* wigner,
                            const float* env, const float* x_res, const int32_t* row_ptr, const int32_t* col_idx,
                            int64_t N, int64_t E, int32_t C, float* x_out, void* stream) {
  return rotate_scatter_fwd_impl(Z_m0, Z_m1, Z_m2, wigner, env, x_res, row_ptr, col_idx, N, E, C, x_out, 0, stream);
}

int fuma_rotate_scatter_fwd_f16x3(const float* Z_m0, const float* Z_m1, const float* Z_m2, const float* wigner,
                                  const float* env, const float* x_res, const int32_t* row_ptr, const int32_t* col_idx,
                                  int64_t N, int64_t E, int32_t C, float* x_out, int32_t act_half, void* stream) {
  return rotate_scatter_fwd_impl(Z_m0, Z_m1, Z_m2, wigner, env, x_res, row_ptr, col_idx, N, E, C, x_out, act_half,
                                 stream);
}

static int rotate_scatter_bwd_impl(const float* g_out, const float* Z_m0, const float* Z_m1, const float* Z_m2,
                            const float* wigner, const float* env, const int32_t* row_ptr, const int32_t* col_idx,
                            int64_t N, int64_t E, int32_t C, float* g_Z_m0, float* g_Z_m1, float* g_Z_m2,
                            float* g_wigner, float* g_env, int split, bool act_half, int* err_flag, void* stream) {
  REQUIRE(!split || C % 8 == 0, "rotate_scatter_bwd_f16x3: the split output needs C %% 8 == 0");
  if (int r = check_C(C)) return r;
  REQUIRE(N >= 0 && E >= 0, "rotate_scatter_bwd: bad sizes");
  if (E == 0 || N == 0) return FUMA_OK;
  REQUIRE(g_out && Z_m0 && Z_m1 && Z_m2 && wigner && env && row_ptr && col_idx && g_Z_m0 && g_Z_m1 && g_Z_m2 &&
              g_wigner && g_env,
          "rotate_scatter_bwd: null pointer");
  REQUIRE_ALIGNED(g_out, "g_out"); REQUIRE_ALIGNED(Z_m0, "Z_m0"); REQUIRE_ALIGNED(Z_m1, "Z_m1");
  REQUIRE_ALIGNED(Z_m2, "Z_m2"); REQUIRE_ALIGNED(g_Z_m0, "g_Z_m0"); REQUIRE_ALIGNED(g_Z_m1, "g_Z_m1");
  REQUIRE_ALIGNED(g_Z_m2, "g_Z_m2");
  BIND(g_out);
  launch_rotate_scatter_bwd(row_ptr, col_idx, g_out, Z_m0, Z_m1, Z_m2, wigner, env, g_Z_m0, g_Z_m1, g_Z_m2, g_wigner,
                            g_env, N, C, split, err_flag, (cudaStream_t)stream, act_half);
  return launched("rotate_scatter_bwd");
}

int fuma_rotate_scatter_bwd(const float* g_out, const float* Z_m0, const float* Z_m1, const float* Z_m2,
                            const float* wigner, const float* env, const int32_t* row_ptr, const int32_t* col_idx,
                            int64_t N, int64_t E, int32_t C, float* g_Z_m0, float* g_Z_m1, float* g_Z_m2,
                            float* g_wigner, float* g_env, void* stream) {
  return rotate_scatter_bwd_impl(g_out, Z_m0, Z_m1, Z_m2, wigner, env, row_ptr, col_idx, N, E, C, g_Z_m0, g_Z_m1,
                                 g_Z_m2, g_wigner, g_env, false, false, nullptr, stream);
}

int fuma_rotate_scatter_bwd_f16x3(const float* g_out, const float* Z_m0, const float* Z_m1, const float* Z_m2,
                            const float* wigner, const float* env, const int32_t* row_ptr, const int32_t* col_idx,
                            int64_t N, int64_t E, int32_t C, float* g_Z_m0, float* g_Z_m1, float* g_Z_m2,
                            float* g_wigner, float* g_env, int32_t parts, int32_t act_half, int* err_flag, void* stream) {
  REQUIRE(parts == 1 || parts == 2, "rotate_scatter_bwd_f16x3: parts=%d must be 1 (hi) or 2 (hi and lo)", parts);
  return rotate_scatter_bwd_impl(g_out, Z_m0, Z_m1, Z_m2, wigner, env, row_ptr, col_idx, N, E, C, g_Z_m0, g_Z_m1,
                                 g_Z_m2, g_wigner, g_env, parts, act_half != 0, err_flag, stream);
}

int fuma_init_scatter_fwd(const float* rad, const float* wigner, const float* env, const int64_t* Z,
                          const int64_t* batch, const float* W_sphere, const float* csd, const int32_t* row_ptr,
                          const int32_t* col_idx, int64_t N, int64_t E, int32_t C, float* x_out, void* stream) {
  if (int r = check_C(C)) return r;
  REQUIRE(N >= 0 && E >= 0, "init_scatter_fwd: bad sizes");
  if (N == 0) return FUMA_OK;
  REQUIRE(Z && batch && W_sphere && csd && row_ptr && x_out && (E == 0 || (rad && wigner && env && col_idx)),
          "init_scatter_fwd: null pointer");
  REQUIRE_ALIGNED(W_sphere, "W_sphere"); REQUIRE_ALIGNED(csd, "csd"); REQUIRE_ALIGNED(x_out, "x_out");
  if (E > 0) REQUIRE_ALIGNED(rad, "rad");
  BIND(x_out);
  launch_init_scatter_fwd(row_ptr, col_idx, rad, wigner, env, Z, batch, W_sphere, csd, x_out, N, C,
                          (cudaStream_t)stream);
  return launched("init_scatter_fwd");
}

static int init_scatter_bwd_impl(const float* g_out, const float* rad, const float* wigner, const float* env,
                          const int32_t* row_ptr, const int32_t* col_idx, int64_t N, int64_t E, int32_t C,
                          float* g_rad, float* g_wigner, float* g_env, int split, int* err_flag, void* stream) {
  REQUIRE(!split || C % 8 == 0, "init_scatter_bwd_f16x3: the split output needs C %% 8 == 0");
  if (int r = check_C(C)) return r;
  REQUIRE(N >= 0 && E >= 0, "init_scatter_bwd: bad sizes");
  if (E == 0 || N == 0) return FUMA_OK;
  REQUIRE(g_out && rad && wigner && env && row_ptr && col_idx && g_rad && g_wigner && g_env,
          "init_scatter_bwd: null pointer");
  REQUIRE_ALIGNED(g_out, "g_out"); REQUIRE_ALIGNED(rad, "rad"); REQUIRE_ALIGNED(g_rad, "g_rad");
  BIND(g_out);
  launch_init_scatter_bwd(row_ptr, col_idx, g_out, rad, wigner, env, g_rad, g_wigner, g_env, N, C,
                          split, err_flag, (cudaStream_t)stream);
  return launched("init_scatter_bwd");
}

int fuma_init_scatter_bwd(const float* g_out, const float* rad, const float* wigner, const float* env,
                          const int32_t* row_ptr, const int32_t* col_idx, int64_t N, int64_t E, int32_t C,
                          float* g_rad, float* g_wigner, float* g_env, void* stream) {
  return init_scatter_bwd_impl(g_out, rad, wigner, env, row_ptr, col_idx, N, E, C, g_rad, g_wigner, g_env, false,
                               nullptr, stream);
}

int fuma_init_scatter_bwd_f16x3(const float* g_out, const float* rad, const float* wigner, const float* env,
                          const int32_t* row_ptr, const int32_t* col_idx, int64_t N, int64_t E, int32_t C,
                          float* g_rad, float* g_wigner, float* g_env, int32_t parts, int* err_flag, void* stream) {
  REQUIRE(parts == 1 || parts == 2, "init_scatter_bwd_f16x3: parts=%d must be 1 (hi) or 2 (hi and lo)", parts);
  return init_scatter_bwd_impl(g_out, rad, wigner, env, row_ptr, col_idx, N, E, C, g_rad, g_wigner, g_env, parts,
                               err_flag, stream);
}

int fuma_linear(const float* A, int64_t lda, const float* W_hi, const float* W_lo, const float* bias, int64_t M,
                int32_t N, int32_t K, int32_t split, float* C, int64_t ldc, int* err_flag, void* stream) {
  REQUIRE(M >= 0 && M < (int64_t(1) << 31), "linear: M=%lld out of range", (long long)M);
  REQUIRE(N > 0 && N % 16 == 0 && N <= 65536 * 16, "linear: N=%d must be a positive multiple of 16", N);
  REQUIRE(K > 0 && K % 4 == 0, "linear: K=%d must be a positive multiple of 4", K);
  REQUIRE(lda >= K && lda % 4 == 0 && ldc >= N && ldc % 4 == 0, "linear: bad leading dimensions");
  if (M == 0) return FUMA_OK;
  REQUIRE(A && W_hi && C && (!split || W_lo), "linear: null pointer");
  REQUIRE_ALIGNED(A, "A"); REQUIRE_ALIGNED(W_hi, "W_hi"); REQUIRE_ALIGNED(C, "C");
  if (split) REQUIRE_ALIGNED(W_lo, "W_lo");
  if (bias) REQUIRE_ALIGNED(bias, "bias");
  BIND(A);
  const int r = launch_gemm_tf32(A, lda, W_hi, W_lo, bias, C, ldc, M, N, K, split != 0, err_flag,
                                 (cudaStream_t)stream);
  if (r == -1) return fail(FUMA_E_INVALID, "linear: could not encode the TMA tensor maps: %s", gemm_map_error());
  if (r != 0) return fail(r, "linear: launch failed: %s", cudaGetErrorString((cudaError_t)r));
  return launched("linear");
}

int fuma_split_tf32(const float* x, int64_t n, float* hi, float* lo, void* stream) {
  REQUIRE(n >= 0, "split_tf32: bad n");
  if (n == 0) return FUMA_OK;
  REQUIRE(x && hi && lo, "split_tf32: null pointer");
  BIND(x);
  launch_split_tf32(x, hi, lo, n, (cudaStream_t)stream);
  return launched("split_tf32");
}

int fuma_linear_f16x3(const float* A, int64_t lda, int32_t a_split, const void* W_hi, const void* W_lo, int64_t ldw,
                      float w_scale_inv, const float* bias, int64_t M, int32_t N, int32_t K, float* C, int64_t ldc,
                      int* err_flag, void* stream) {
  REQUIRE(M >= 0 && M < (int64_t(1) << 31), "linear_f16x3: M=%lld out of range", (long long)M);
  REQUIRE(N > 0 && N % 16 == 0 && N <= 65536 * 16, "linear_f16x3: N=%d must be a positive multiple of 16", N);
  REQUIRE(K > 0 && K % 4 == 0, "linear_f16x3: K=%d must be a positive multiple of 4", K);
  REQUIRE(lda >= K && lda % 4 == 0 && ldc >= N && ldc % 4 == 0, "linear_f16x3: bad leading dimensions of A or C");
  REQUIRE(!a_split || lda % 8 == 0, "linear_f16x3: a row-packed split A needs lda %% 8 == 0 (lda=%lld)",
          (long long)lda);
  REQUIRE(ldw >= K && ldw % 8 == 0, "linear_f16x3: ldw=%lld must be >= K and a multiple of 8", (long long)ldw);
  REQUIRE(w_scale_inv > 0.0f, "linear_f16x3: w_scale_inv must be positive");
  if (M == 0) return FUMA_OK;
  REQUIRE(A && W_hi && W_lo && C, "linear_f16x3: null pointer");
  REQUIRE_ALIGNED(A, "A"); REQUIRE_ALIGNED(W_hi, "W_hi"); REQUIRE_ALIGNED(W_lo, "W_lo"); REQUIRE_ALIGNED(C, "C");
  if (bias) REQUIRE_ALIGNED(bias, "bias");
  BIND(A);
  const int r = launch_gemm_f16x3(A, lda, a_split != 0, W_hi, W_lo, ldw, w_scale_inv, bias, C, ldc, M, N, K, err_flag,
                                  (cudaStream_t)stream);
  if (r == -1) return fail(FUMA_E_INVALID, "linear_f16x3: could not encode the TMA tensor maps: %s", gemm_map_error());
  if (r != 0) return fail(r, "linear_f16x3: launch failed: %s", cudaGetErrorString((cudaError_t)r));
  return launched("linear_f16x3");
}

int fuma_linear_f16(const float* A, int64_t lda, const void* W_hi, int64_t ldw, float w_scale_inv, const float* bias,
                    int64_t M, int32_t N, int32_t K, void* C, int64_t ldc, int32_t c_half, int* err_flag,
                    void* stream) {
  REQUIRE(M >= 0 && M < (int64_t(1) << 31), "linear_f16: M=%lld out of range", (long long)M);
  REQUIRE(N > 0 && N % 16 == 0 && N <= 65536 * 16, "linear_f16: N=%d must be a positive multiple of 16", N);
  REQUIRE(K > 0 && K % 8 == 0, "linear_f16: K=%d must be a positive multiple of 8", K);
  REQUIRE(lda >= K && lda % 8 == 0 && ldc >= N && ldc % (c_half ? 8 : 4) == 0,
          "linear_f16: bad leading dimensions of A or C");
  REQUIRE(ldw >= K && ldw % 8 == 0, "linear_f16: ldw=%lld must be >= K and a multiple of 8", (long long)ldw);
  REQUIRE(w_scale_inv > 0.0f, "linear_f16: w_scale_inv must be positive");
  if (M == 0) return FUMA_OK;
  REQUIRE(A && W_hi && C, "linear_f16: null pointer");
  REQUIRE_ALIGNED(A, "A"); REQUIRE_ALIGNED(W_hi, "W_hi"); REQUIRE_ALIGNED(C, "C");
  if (bias) REQUIRE_ALIGNED(bias, "bias");
  BIND(A);
  const int r = launch_gemm_f16x3(A, lda, true, W_hi, W_hi, ldw, w_scale_inv, bias, static_cast<float*>(C), ldc, M, N,
                                  K, err_flag, (cudaStream_t)stream, true, c_half != 0);
  if (r == -1) return fail(FUMA_E_INVALID, "linear_f16: could not encode the TMA tensor maps: %s", gemm_map_error());
  if (r != 0) return fail(r, "linear_f16: launch failed: %s", cudaGetErrorString((cudaError_t)r));
  return launched("linear_f16");
}

int fuma_split_rows_f16(const float* x, int64_t lda, int64_t M, int32_t K, void* out, int64_t ldp, int* err_flag,
                        void* stream) {
  REQUIRE(M >= 0 && K > 0 && K % 4 == 0, "split_rows_f16: bad shape M=%lld K=%d", (long long)M, K);
  REQUIRE(lda >= K && lda % 4 == 0 && ldp >= K && ldp % 8 == 0, "split_rows_f16: bad leading dimensions");
  if (M == 0) return FUMA_OK;
  REQUIRE(x && out, "split_rows_f16: null pointer");
  REQUIRE_ALIGNED(x, "x"); REQUIRE_ALIGNED(out, "out");
  BIND(x);
  launch_split_rows_f16(x, lda, M, K, out, ldp, err_flag, (cudaStream_t)stream);
  return launched("split_rows_f16");
}

int fuma_rmsnorm_sh_fwd(const float* x, const float* affine_weight, const float* affine_bias,
                        const float* degree_weight, float eps, int64_t N, int32_t C, float* out, float* rstd,
                        void* stream) {
  REQUIRE(N >= 0 && C > 0 && C % 4 == 0 && C <= 256, "rmsnorm_sh_fwd: C=%d must be a multiple of 4 up to 256", C);
  REQUIRE(eps > 0.0f, "rmsnorm_sh_fwd: eps must be positive");
  if (N == 0) return FUMA_OK;
  REQUIRE(x && affine_weight && affine_bias && degree_weight && out && rstd, "rmsnorm_sh_fwd: null pointer");
  REQUIRE_ALIGNED(x, "x"); REQUIRE_ALIGNED(out, "out"); REQUIRE_ALIGNED(affine_weight, "affine_weight");
  REQUIRE_ALIGNED(affine_bias, "affine_bias");
  BIND(x);
  launch_rmsnorm_sh_fwd(x, affine_weight, affine_bias, degree_weight, eps, N, C, out, rstd, (cudaStream_t)stream);
  return launched("rmsnorm_sh_fwd");
}

int fuma_rmsnorm_sh_bwd(const float* x, const float* affine_weight, const float* degree_weight, const float* rstd,
                        const float* g_out, int64_t N, int32_t C, float* g_x, void* stream) {
  REQUIRE(N >= 0 && C > 0 && C % 4 == 0 && C <= 256, "rmsnorm_sh_bwd: C=%d must be a multiple of 4 up to 256", C);
  if (N == 0) return FUMA_OK;
  REQUIRE(x && affine_weight && degree_weight && rstd && g_out && g_x, "rmsnorm_sh_bwd: null pointer");
  REQUIRE_ALIGNED(x, "x"); REQUIRE_ALIGNED(g_out, "g_out"); REQUIRE_ALIGNED(g_x, "g_x");
  REQUIRE_ALIGNED(affine_weight, "affine_weight");
  BIND(x);
  launch_rmsnorm_sh_bwd(x, affine_weight, degree_weight, rstd, g_out, N, C, g_x, (cudaStream_t)stream);
  return launched("rmsnorm_sh_bwd");
}

int fuma_atomwise_gate_fwd(const float* h, const float* u, const float* b1, int64_t N, int32_t H, float* z,
                           void* stream) {
  REQUIRE(N >= 0 && H > 0 && H % 4 == 0, "atomwise_gate_fwd: H=%d must be a positive multiple of 4", H);
  if (N == 0) return FUMA_OK;
  REQUIRE(h && u && b1 && z, "atomwise_gate_fwd: null pointer");
  REQUIRE_ALIGNED(h, "h"); REQUIRE_ALIGNED(u, "u"); REQUIRE_ALIGNED(b1, "b1"); REQUIRE_ALIGNED(z, "z");
  BIND(h);
  launch_atomwise_gate_fwd(h, H, false, u, b1, N, H, z, 0, nullptr, (cudaStream_t)stream);
  return launched("atomwise_gate_fwd");
}

int fuma_atomwise_gate_bwd(const float* gz, const float* h, const float* u, const float* b1, int64_t N, int32_t H,
                           float* gh, float* gu, void* stream) {
  REQUIRE(N >= 0 && H > 0 && H % 4 == 0, "atomwise_gate_bwd: H=%d must be a positive multiple of 4", H);
  if (N == 0) return FUMA_OK;
  REQUIRE(gz && h && u && b1 && gh && gu, "atomwise_gate_bwd: null pointer");
  REQUIRE_ALIGNED(gz, "gz"); REQUIRE_ALIGNED(h, "h"); REQUIRE_ALIGNED(u, "u"); REQUIRE_ALIGNED(b1, "b1");
  REQUIRE_ALIGNED(gh, "gh"); REQUIRE_ALIGNED(gu, "gu");
  BIND(h);
  launch_atomwise_gate_bwd(gz, h, H, false, u, b1, N, H, gh, gu, 0, nullptr, (cudaStream_t)stream);
  return launched("atomwise_gate_bwd");
}

int fuma_coef_to_node(const float* src, const float* add, const float* row0, int32_t row0_per_node, int64_t N,
                      int32_t W, float* out, void* stream) {
  REQUIRE(N >= 0 && W > 0 && W % 4 == 0, "coef_to_node: W=%d must be a positive multiple of 4", W);
  if (N == 0) return FUMA_OK;
  REQUIRE(src && out, "coef_to_node: null pointer");
  REQUIRE_ALIGNED(src, "src"); REQUIRE_ALIGNED(out, "out");
  if (add) REQUIRE_ALIGNED(add, "add");
  if (row0) REQUIRE_ALIGNED(row0, "row0");
  BIND(src);
  launch_coef_to_node(src, W, false, add, row0, row0_per_node != 0, N, W, out, (cudaStream_t)stream);
  return launched("coef_to_node");
}

int fuma_node_to_coef_f16x3(const float* x, int64_t N, int32_t W, float* out, int32_t parts, int* err_flag,
                            void* stream) {
  REQUIRE(N >= 0 && W > 0 && W % 8 == 0, "node_to_coef_f16x3: W=%d must be a positive multiple of 8", W);
  REQUIRE(parts == 1 || parts == 2, "node_to_coef_f16x3: parts=%d must be 1 or 2", parts);
  if (N == 0) return FUMA_OK;
  REQUIRE(x && out, "node_to_coef_f16x3: null pointer");
  REQUIRE_ALIGNED(x, "x"); REQUIRE_ALIGNED(out, "out");
  BIND(x);
  launch_node_to_coef(x, N, W, out, parts, err_flag, (cudaStream_t)stream);
  return launched("node_to_coef_f16x3");
}

int fuma_atomwise_gate_fwd_f16x3(const float* h, const float* u, const float* b1, int64_t N, int32_t H, float* z,
                                 int32_t parts, int* err_flag, void* stream) {
  REQUIRE(N >= 0 && H > 0 && H % 8 == 0, "atomwise_gate_fwd_f16x3: H=%d must be a positive multiple of 8", H);
  REQUIRE(parts == 1 || parts == 2, "atomwise_gate_fwd_f16x3: parts=%d must be 1 or 2", parts);
  if (N == 0) return FUMA_OK;
  REQUIRE(h && u && b1 && z, "atomwise_gate_fwd_f16x3: null pointer");
  REQUIRE_ALIGNED(h, "h"); REQUIRE_ALIGNED(u, "u"); REQUIRE_ALIGNED(b1, "b1"); REQUIRE_ALIGNED(z, "z");
  BIND(h);
  launch_atomwise_gate_fwd(h, 3 * (int64_t)H, true, u, b1, N, H, z, parts, err_flag, (cudaStream_t)stream);
  return launched("atomwise_gate_fwd_f16x3");
}

int fuma_atomwise_gate_bwd_f16x3(const float* gz, const float* h, const float* u, const float* b1, int64_t N,
                                 int32_t H, float* gh, float* gu, int32_t parts, int* err_flag, void* stream) {
  REQUIRE(N >= 0 && H > 0 && H % 8 == 0, "atomwise_gate_bwd_f16x3: H=%d must be a positive multiple of 8", H);
  REQUIRE(parts == 1 || parts == 2, "atomwise_gate_bwd_f16x3: parts=%d must be 1 or 2", parts);
  if (N == 0) return FUMA_OK;
  REQUIRE(gz && h && u && b1 && gh && gu, "atomwise_gate_bwd_f16x3: null pointer");
  REQUIRE_ALIGNED(gz, "gz"); REQUIRE_ALIGNED(h, "h"); REQUIRE_ALIGNED(u, "u"); REQUIRE_ALIGNED(b1, "b1");
  REQUIRE_ALIGNED(gh, "gh"); REQUIRE_ALIGNED(gu, "gu");
  BIND(h);
  launch_atomwise_gate_bwd(gz, h, 3 * (int64_t)H, true, u, b1, N, H, gh, gu, parts, err_flag, (cudaStream_t)stream);
  return launched("atomwise_gate_bwd_f16x3");
}

int fuma_coef_to_node_blocked(const float* src, const float* add, const float* row0, int32_t row0_per_node,
                              int64_t N, int32_t W, float* out, void* stream) {
  REQUIRE(N >= 0 && W > 0 && W % 4 == 0, "coef_to_node_blocked: W=%d must be a positive multiple of 4", W);
  if (N == 0) return FUMA_OK;
  REQUIRE(src && out, "coef_to_node_blocked: null pointer");
  REQUIRE_ALIGNED(src, "src"); REQUIRE_ALIGNED(out, "out");
  if (add) REQUIRE_ALIGNED(add, "add");
  if (row0) REQUIRE_ALIGNED(row0, "row0");
  BIND(src);
  launch_coef_to_node(src, 3 * (int64_t)W, true, add, row0, row0_per_node != 0, N, W, out, (cudaStream_t)stream);
  return launched("coef_to_node_blocked");
}

int64_t fuma_morton_scratch_bytes(int64_t N) { return N < 0 ? 0 : morton_scratch_bytes(N); }

int fuma_morton_reorder(const float* pos, const int64_t* Z, const int64_t* batch, const int64_t* idx_i,
                        const int64_t* idx_j, int64_t N, int64_t E, int64_t* perm, int64_t* inv_perm, float* pos_s,
                        int64_t* Z_s, int64_t* batch_s, int64_t* ii, int64_t* jj, void* scratch,
                        int64_t scratch_bytes, int* err_flag, void* stream) {
  REQUIRE(N >= 0 && N < (int64_t(1) << 31), "morton_reorder: bad N=%lld", (long long)N);
  REQUIRE(E >= 0, "morton_reorder: bad E");
  if (N == 0 && E == 0) return FUMA_OK;
  REQUIRE(pos && Z && batch && perm && inv_perm && Z_s && batch_s, "morton_reorder: null atom pointer");
  REQUIRE(E == 0 || (idx_i && idx_j && ii && jj), "morton_reorder: null edge pointer");
  const int64_t need = morton_scratch_bytes(N);
  REQUIRE(scratch_bytes >= need && (need == 0 || scratch),
          "morton_reorder: N=%lld needs %lld bytes of scratch (fuma_morton_scratch_bytes), got %lld",
          (long long)N, (long long)need, (long long)scratch_bytes);
  REQUIRE(need == 0 || (reinterpret_cast<uintptr_t>(scratch) & 255u) == 0,
          "morton_reorder: scratch must be 256-byte aligned");
  BIND(pos);
  const cudaError_t st = launch_morton_reorder(pos, Z, batch, idx_i, idx_j, N, E, perm, inv_perm, pos_s, Z_s,
                                               batch_s, ii, jj, scratch, err_flag, (cudaStream_t)stream);
  if (st != cudaSuccess) return fail((int)st, "morton_reorder: launch failed: %s", cudaGetErrorString(st));
  return launched("morton_reorder");
}

int64_t fuma_neighbor_scratch_bytes(int64_t N, const int32_t* grid) {
  if (N < 0 || !grid || grid[0] < 1 || grid[1] < 1 || grid[2] < 1) return 0;
  return neighbor_scratch_bytes(N, (int64_t)grid[0] * grid[1] * grid[2]);
}

int fuma_neighbor_list(const double* pos, int64_t N, const double* geom, const int32_t* grid, double cutoff,
                       int32_t max_neighbors, void* scratch, int64_t scratch_bytes, int32_t* counts, int64_t* src,
                       int64_t* offsets, double* dist, int* err_flag, void* stream) {
  REQUIRE(N >= 0 && N < (int64_t(1) << 31), "neighbor_list: bad N=%lld", (long long)N);
  REQUIRE(geom && grid, "neighbor_list: null geometry / grid (host arrays)");
  REQUIRE(cutoff > 0 && max_neighbors > 0, "neighbor_list: cutoff and max_neighbors must be positive");
  for (int k = 0; k < 3; ++k)
    REQUIRE(grid[k] >= 1 && grid[3 + k] <= grid[6 + k], "neighbor_list: bad bin grid / image range on axis %d", k);
  if (N == 0) return FUMA_OK;
  REQUIRE(pos && counts && src && offsets && dist && scratch, "neighbor_list: null pointer");
  const int64_t need = neighbor_scratch_bytes(N, (int64_t)grid[0] * grid[1] * grid[2]);
  REQUIRE(scratch_bytes >= need, "neighbor_list: needs %lld bytes of scratch, got %lld", (long long)need,
          (long long)scratch_bytes);
  REQUIRE((reinterpret_cast<uintptr_t>(scratch) & 255u) == 0, "neighbor_list: scratch must be 256-byte aligned");
  BIND(pos);
  const cudaError_t st = launch_neighbor_list(pos, N, geom, geom + 9, grid, grid + 3, grid + 6, grid + 9, cutoff,
                                              max_neighbors, scratch, counts, src, offsets, dist, err_flag,
                                              (cudaStream_t)stream);
  if (st != cudaSuccess) return fail((int)st, "neighbor_list: launch failed: %s", cudaGetErrorString(st));
  return launched("neighbor_list");
}

int fuma_csr_permute(const int32_t* dst_row_ptr, const int32_t* dst_col, const int32_t* src_row_ptr,
                     const int32_t* src_col, const int64_t* perm, int64_t N, int64_t E, int32_t* new_dst_row_ptr,
                     int32_t* new_dst_col, int32_t* new_src_row_ptr, int32_t* new_src_col, void* stream) {
  REQUIRE(N >= 0 && E >= 0 && E < (int64_t(1) << 31), "csr_permute: bad sizes N=%lld E=%lld", (long long)N,
          (long long)E);
  REQUIRE(dst_row_ptr && new_dst_row_ptr, "csr_permute: null row pointer");
  REQUIRE(E == 0 || (dst_col && new_dst_col), "csr_permute: null column pointer");
  const bool two = src_row_ptr != nullptr;
  REQUIRE(!two || (new_src_row_ptr && (E == 0 || (src_col && new_src_col))),
          "csr_permute: the source CSR needs all four of its pointers");
  REQUIRE(N == 0 || perm, "csr_permute: null permutation");
  BIND(dst_row_ptr);
  const int32_t* rp[2] = {dst_row_ptr, src_row_ptr};
  const int32_t* cl[2] = {dst_col, src_col};
  int32_t* nrp[2] = {new_dst_row_ptr, new_src_row_ptr};
  int32_t* ncl[2] = {new_dst_col, new_src_col};
  launch_csr_permute(two ? 2 : 1, rp, cl, perm, N, nrp, ncl, (cudaStream_t)stream);
  return launched("csr_permute");
}

int fuma_split_f16(const float* x, int64_t n, float scale, void* hi, void* lo, void* stream) {
  REQUIRE(n >= 0, "split_f16: bad n");
  REQUIRE(scale > 0.0f, "split_f16: scale must be positive");
  if (n == 0) return FUMA_OK;
  REQUIRE(x && hi && lo, "split_f16: null pointer");
  BIND(x);
  launch_split_f16(x, hi, lo, scale, n, (cudaStream_t)stream);
  return launched("split_f16");
}

}  // extern "C"
