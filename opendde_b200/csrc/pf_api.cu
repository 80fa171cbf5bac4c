// pf_api.cu -- the extern "C" entry points declared in include/pairformer_b200.h.
//
// Host-side validation (shapes, dtypes, pointers, workspace size) happens here, before any
// launch; failures return a status code and leave a message in a thread-local buffer.
// Dispatch: bf16 requests with the tuned channel counts go to the fused tcgen05 kernels
// (pf_tc_*.cu, path "tc"), other bf16 widths to the general-width tcgen05 path (pf_tc_rows.cu,
// path "tc.rows"); fp32 requests and shapes neither covers go to the SIMT kernels (pf_simt.cu).

#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "pf_common.cuh"
#include "pf_simt.h"
#include "pf_tc.h"
#include "pf_tmap.h"

namespace pf {

static thread_local char g_err[1024] = "";
static thread_local const char* g_path = "none";
static int g_force_simt = 0;

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return status;
}

void set_path(const char* p) { g_path = p; }
bool force_simt() { return g_force_simt != 0; }

static int check_dtype(int dtype) {
  if (dtype != PF_F32 && dtype != PF_BF16) return fail(PF_EINVAL_DTYPE, "unknown dtype %d", dtype);
  return PF_OK;
}

static int check_ws(void* ws, size_t have, size_t need, const char* what) {
  if (need == 0) return PF_OK;
  if (ws == nullptr) return fail(PF_EWORKSPACE, "%s: workspace is NULL (need %zu bytes)", what, need);
  if (have < need)
    return fail(PF_EWORKSPACE, "%s: workspace too small (%zu < %zu bytes)", what, have, need);
  if (((uintptr_t)ws) % 256 != 0) return fail(PF_EWORKSPACE, "%s: workspace not 256-byte aligned", what);
  return PF_OK;
}

static bool view_ok(const pf_pair_view& v) { return v.ptr != nullptr && v.row_stride >= 0 && v.col_stride >= 0; }

}  // namespace pf

using namespace pf;

extern "C" {

int pf_abi_version(void) { return PF_ABI_VERSION; }
const char* pf_last_error_string(void) { return g_err; }
const char* pf_last_path(void) { return g_path; }

int pf_set_option(int option, int64_t value) {
  if (option == PF_OPT_FORCE_SIMT) {
    g_force_simt = value ? 1 : 0;
    return PF_OK;
  }
  if (option == PF_OPT_SM_RESERVE) {
    if (value < 0 || value > 64) return fail(PF_EINVAL_ARG, "SM reserve %lld outside [0, 64]", (long long)value);
    set_sm_reserve((int)value);
    return PF_OK;
  }
  return fail(PF_EINVAL_ARG, "unknown option %d", option);
}

// ------------------------------------------------------------------ LayerNorm
int pf_layernorm_fwd(const void* x, void* y, const float* gamma, const float* beta, int64_t rows,
                     int32_t c, float eps, int32_t dtype, void* stream) {
  PF_TRY(check_dtype(dtype));
  if (!x || !y) return fail(PF_EINVAL_ARG, "layernorm: null input/output");
  if (rows < 0 || c <= 0 || c > 1024) return fail(PF_EINVAL_SHAPE, "layernorm: rows=%lld c=%d", (long long)rows, c);
  if (rows == 0) return PF_OK;
  // LayerNorm is fused into every producing tensor-core kernel; the standalone entry point runs
  // a row kernel with 128-bit loads and stores in both dtypes (HBM-bound, no MMA to feed), or
  // the scalar warp-per-row kernel when rows are not whole 16-byte vectors.
  set_path("simt");
  return simt::layernorm(x, y, gamma, beta, rows, c, eps, dtype, (cudaStream_t)stream);
}

// ------------------------------------------------------------------ triangle multiplication
static bool trimul_tc(int64_t n_i, int64_t n_j, int64_t n_k, int c_z, int c_h, int dtype) {
  return dtype == PF_BF16 && !force_simt() && tc::trimul_supported(n_i, n_j, n_k, c_z, c_h);
}
// the general-width tensor-core path (every bf16 width the fused c = 128 kernels do not take)
static bool trimul_rows(int64_t n_i, int64_t n_j, int64_t n_k, int c_z, int c_h, int dtype) {
  return dtype == PF_BF16 && !force_simt() && !tc::trimul_supported(n_i, n_j, n_k, c_z, c_h) &&
         tc::rows_trimul_supported(c_z, c_h) && n_i >= 1 && n_j >= 1 && n_k >= 1 && n_i < (1ll << 31) &&
         n_j < (1ll << 31) && n_k < (1ll << 31);
}

int pf_trimul_workspace_size(int64_t n_i, int64_t n_j, int64_t n_k, int32_t c_z, int32_t c_h,
                             int32_t dtype, size_t* bytes) {
  PF_TRY(check_dtype(dtype));
  if (!bytes) return fail(PF_EINVAL_ARG, "bytes is NULL");
  if (n_i < 0 || n_j < 0 || n_k < 0 || c_z <= 0 || c_h <= 0)
    return fail(PF_EINVAL_SHAPE, "trimul: bad sizes");
  *bytes = trimul_tc(n_i, n_j, n_k, c_z, c_h, dtype)     ? tc::trimul_ws_bytes(n_i, n_j, n_k, c_z, c_h)
           : trimul_rows(n_i, n_j, n_k, c_z, c_h, dtype) ? tc::rows_trimul_ws_bytes(n_i, n_j, n_k, c_z, c_h)
                                                         : simt::trimul_ws_bytes(n_i, n_j, n_k, c_z, c_h);
  return PF_OK;
}

int pf_trimul_fwd(const pf_trimul_params* w, pf_pair_view za, pf_pair_view zb, pf_mask_view ma,
                  pf_mask_view mb, pf_pair_view zg, pf_pair_view zo, int64_t n_i, int64_t n_j, int64_t n_k,
                  int32_t c_z, int32_t c_h, int32_t accumulate, int32_t dtype, void* workspace,
                  size_t workspace_bytes, void* stream) {
  PF_TRY(check_dtype(dtype));
  if (!w || !w->w_ap || !w->w_ag || !w->w_bp || !w->w_bg || !w->w_z || !w->w_g)
    return fail(PF_EINVAL_ARG, "trimul: null weight pointer");
  if (!view_ok(za) || !view_ok(zb) || !view_ok(zg) || !view_ok(zo))
    return fail(PF_EINVAL_ARG, "trimul: bad pair view");
  if (n_i < 0 || n_j < 0 || n_k < 0 || c_z <= 0 || c_h <= 0 || c_z > 1024 || c_h > 1024)
    return fail(PF_EINVAL_SHAPE, "trimul: bad sizes n_i=%lld n_j=%lld n_k=%lld c_z=%d c_h=%d",
                (long long)n_i, (long long)n_j, (long long)n_k, c_z, c_h);
  if (n_i == 0 || n_j == 0) return PF_OK;
  size_t need;
  PF_TRY(pf_trimul_workspace_size(n_i, n_j, n_k, c_z, c_h, dtype, &need));
  PF_TRY(check_ws(workspace, workspace_bytes, need, "trimul"));
  cudaStream_t st = (cudaStream_t)stream;
  if (trimul_tc(n_i, n_j, n_k, c_z, c_h, dtype)) {
    set_path("tc");
    return tc::trimul(w, za, zb, ma, mb, zg, zo, n_i, n_j, n_k, c_z, c_h, accumulate, workspace,
                      workspace_bytes, st);
  }
  if (trimul_rows(n_i, n_j, n_k, c_z, c_h, dtype)) {
    set_path("tc.rows");
    return tc::rows_trimul(w, za, zb, ma, mb, zg, zo, n_i, n_j, n_k, c_z, c_h, accumulate, workspace,
                           workspace_bytes, st);
  }
  set_path("simt");
  return simt::trimul(w, za, zb, ma, mb, zg, zo, n_i, n_j, n_k, c_z, c_h, accumulate, dtype, workspace,
                      workspace_bytes, st);
}

// Split stages of the same computation (Fold-CP exchanges the projections between them).
int pf_trimul_project_workspace_size(int64_t n_rows, int64_t n_cols, int32_t c_z, int32_t c_h, int32_t dtype,
                                     size_t* bytes) {
  PF_TRY(check_dtype(dtype));
  if (!bytes) return fail(PF_EINVAL_ARG, "bytes is NULL");
  if (n_rows < 0 || n_cols < 0 || c_z <= 0 || c_h <= 0) return fail(PF_EINVAL_SHAPE, "trimul project: bad sizes");
  *bytes = trimul_tc(n_rows, n_rows, n_cols, c_z, c_h, dtype) ? 0
           : trimul_rows(n_rows, n_rows, n_cols, c_z, c_h, dtype)
               ? tc::rows_trimul_project_ws_bytes(n_rows, n_cols, c_z, c_h)
               : simt::trimul_project_ws_bytes(n_rows, n_cols, c_z, c_h);
  return PF_OK;
}

int pf_trimul_project(const pf_trimul_params* w, pf_pair_view z, pf_mask_view m, int64_t n_rows, int64_t n_cols,
                      int32_t c_z, int32_t c_h, int32_t dtype, void* a_out, void* b_out, int64_t ld,
                      void* workspace, size_t workspace_bytes, void* stream) {
  PF_TRY(check_dtype(dtype));
  if (!w || !w->w_ap || !w->w_ag || !w->w_bp || !w->w_bg) return fail(PF_EINVAL_ARG, "trimul project: null weight");
  if (!view_ok(z) || !a_out || !b_out) return fail(PF_EINVAL_ARG, "trimul project: bad view or output pointer");
  if (n_rows < 0 || n_cols < 0 || c_z <= 0 || c_h <= 0 || c_z > 1024 || c_h > 1024 || ld < n_cols)
    return fail(PF_EINVAL_SHAPE, "trimul project: bad sizes n_rows=%lld n_cols=%lld ld=%lld c_z=%d c_h=%d",
                (long long)n_rows, (long long)n_cols, (long long)ld, c_z, c_h);
  if (n_rows == 0 || n_cols == 0) return PF_OK;
  size_t need;
  PF_TRY(pf_trimul_project_workspace_size(n_rows, n_cols, c_z, c_h, dtype, &need));
  if (need) PF_TRY(check_ws(workspace, workspace_bytes, need, "trimul project"));
  cudaStream_t st = (cudaStream_t)stream;
  if (trimul_tc(n_rows, n_rows, n_cols, c_z, c_h, dtype)) {
    set_path("tc");
    return tc::trimul_project(w, z, m, n_rows, n_cols, a_out, b_out, ld, st);
  }
  if (trimul_rows(n_rows, n_rows, n_cols, c_z, c_h, dtype)) {
    set_path("tc.rows");
    return tc::rows_trimul_project(w, z, m, n_rows, n_cols, c_z, c_h, a_out, b_out, ld, workspace, workspace_bytes,
                                   st);
  }
  set_path("simt");
  return simt::trimul_project(w, z, m, n_rows, n_cols, c_z, c_h, dtype, a_out, b_out, ld, workspace,
                              workspace_bytes, st);
}

int pf_trimul_combine_workspace_size(int64_t n_i, int64_t n_j, int64_t n_k, int32_t c_z, int32_t c_h,
                                     int32_t dtype, size_t* bytes) {
  PF_TRY(check_dtype(dtype));
  if (!bytes) return fail(PF_EINVAL_ARG, "bytes is NULL");
  if (n_i < 0 || n_j < 0 || n_k < 0 || c_z <= 0 || c_h <= 0) return fail(PF_EINVAL_SHAPE, "trimul combine: bad sizes");
  *bytes = trimul_tc(n_i, n_j, n_k, c_z, c_h, dtype)     ? tc::trimul_combine_ws_bytes(n_i, n_j)
           : trimul_rows(n_i, n_j, n_k, c_z, c_h, dtype) ? tc::rows_trimul_combine_ws_bytes(n_i, n_j, c_z, c_h)
                                                         : simt::trimul_combine_ws_bytes(n_i, n_j, c_z, c_h);
  return PF_OK;
}

int pf_trimul_combine(const pf_trimul_params* w, const void* a, const void* b, int64_t ld, int64_t n_i,
                      int64_t n_j, int64_t n_k, pf_pair_view zg, pf_pair_view zo, int32_t c_z, int32_t c_h,
                      int32_t accumulate, int32_t dtype, void* workspace, size_t workspace_bytes, void* stream) {
  PF_TRY(check_dtype(dtype));
  if (!w || !w->w_z || !w->w_g) return fail(PF_EINVAL_ARG, "trimul combine: null weight pointer");
  if (!view_ok(zg) || !view_ok(zo) || !a || !b) return fail(PF_EINVAL_ARG, "trimul combine: bad view or operand");
  if (n_i < 0 || n_j < 0 || n_k < 0 || c_z <= 0 || c_h <= 0 || c_z > 1024 || c_h > 1024 || ld < n_k)
    return fail(PF_EINVAL_SHAPE, "trimul combine: bad sizes n_i=%lld n_j=%lld n_k=%lld ld=%lld",
                (long long)n_i, (long long)n_j, (long long)n_k, (long long)ld);
  if (n_i == 0 || n_j == 0) return PF_OK;
  size_t need;
  PF_TRY(pf_trimul_combine_workspace_size(n_i, n_j, n_k, c_z, c_h, dtype, &need));
  PF_TRY(check_ws(workspace, workspace_bytes, need, "trimul combine"));
  cudaStream_t st = (cudaStream_t)stream;
  if (trimul_tc(n_i, n_j, n_k, c_z, c_h, dtype)) {
    set_path("tc");
    return tc::trimul_combine(w, a, b, ld, n_i, n_j, n_k, zg, zo, accumulate, workspace, workspace_bytes, st);
  }
  if (trimul_rows(n_i, n_j, n_k, c_z, c_h, dtype)) {
    set_path("tc.rows");
    return tc::rows_trimul_combine(w, a, b, ld, n_i, n_j, n_k, zg, zo, c_z, c_h, accumulate, workspace,
                                   workspace_bytes, st);
  }
  set_path("simt");
  return simt::trimul_combine(w, a, b, ld, n_i, n_j, n_k, zg, zo, c_z, c_h, accumulate, dtype, workspace,
                              workspace_bytes, st);
}

// ------------------------------------------------------------------ triangle attention
static bool triatt_tc(int c, int H, int d, int dtype) {
  return dtype == PF_BF16 && !force_simt() && tc::triatt_supported(c, H, d);
}
static bool triatt_rows(int c, int H, int d, int dtype) {
  return dtype == PF_BF16 && !force_simt() && !tc::triatt_supported(c, H, d) && tc::rows_triatt_supported(c, H, d);
}
static bool triatt_bias_tc(int c, int H, int dtype) {
  return dtype == PF_BF16 && !force_simt() && tc::triatt_bias_supported(c, H);
}
static bool triatt_bias_rows(int c, int H, int dtype) {
  return dtype == PF_BF16 && !force_simt() && !tc::triatt_bias_supported(c, H) && tc::rows_bias_supported(c, H);
}

int pf_triatt_bias_workspace_size(int64_t n_rows, int64_t n_cols, int32_t c, int32_t heads,
                                  int32_t dtype, size_t* bytes) {
  PF_TRY(check_dtype(dtype));
  if (!bytes) return fail(PF_EINVAL_ARG, "bytes is NULL");
  *bytes = triatt_bias_tc(c, heads, dtype)     ? 0
           : triatt_bias_rows(c, heads, dtype) ? tc::rows_bias_ws_bytes(n_rows, n_cols, c)
                                               : simt::triatt_bias_ws_bytes(n_rows, n_cols, c, heads);
  return PF_OK;
}

int pf_triatt_bias(const pf_triatt_params* w, pf_pair_view z, int64_t n_rows, int64_t n_cols,
                   void* bias, int64_t hs, int64_t rs, int32_t c, int32_t heads, int32_t dtype,
                   void* workspace, size_t workspace_bytes, void* stream) {
  PF_TRY(check_dtype(dtype));
  if (!w || !w->w_bias || !bias || !view_ok(z)) return fail(PF_EINVAL_ARG, "triatt_bias: null pointer");
  if (n_rows < 0 || n_cols < 0 || c <= 0 || c > 1024 || heads <= 0)
    return fail(PF_EINVAL_SHAPE, "triatt_bias: bad sizes");
  if (n_rows == 0 || n_cols == 0) return PF_OK;
  size_t need;
  PF_TRY(pf_triatt_bias_workspace_size(n_rows, n_cols, c, heads, dtype, &need));
  PF_TRY(check_ws(workspace, workspace_bytes, need, "triatt_bias"));
  cudaStream_t st = (cudaStream_t)stream;
  if (triatt_bias_tc(c, heads, dtype)) {
    set_path("tc");
    return tc::triatt_bias(w, z, n_rows, n_cols, bias, hs, rs, c, heads, st);
  }
  if (triatt_bias_rows(c, heads, dtype)) {
    set_path("tc.rows");
    return tc::rows_head_bias(w->ln_w, w->ln_b, w->w_bias, z, n_rows, n_cols, c, heads, bias, hs, rs, true,
                              workspace, workspace_bytes, st);
  }
  set_path("simt");
  return simt::triatt_bias(w, z, n_rows, n_cols, bias, hs, rs, c, heads, dtype, workspace,
                           workspace_bytes, st);
}

int pf_triatt_workspace_size(int64_t n_rows, int64_t n_keys, int64_t n_q, int32_t c, int32_t heads,
                             int32_t head_dim, int32_t dtype, size_t* bytes) {
  PF_TRY(check_dtype(dtype));
  if (!bytes) return fail(PF_EINVAL_ARG, "bytes is NULL");
  *bytes = triatt_tc(c, heads, head_dim, dtype)     ? tc::triatt_ws_bytes(n_rows, n_keys, n_q, c, heads, head_dim)
           : triatt_rows(c, heads, head_dim, dtype) ? tc::rows_triatt_ws_bytes(n_rows, n_keys, n_q, c, heads)
                                                    : simt::triatt_ws_bytes(n_rows, n_keys, n_q, c, heads, head_dim);
  return PF_OK;
}

int pf_triatt_fwd(const pf_triatt_params* w, pf_pair_view zs, pf_mask_view m, const void* bias,
                  int64_t b_hs, int64_t b_rs, pf_pair_view zo, int64_t n_rows, int64_t n_keys,
                  int64_t n_valid_keys, int64_t q_col0, int64_t n_q, int32_t c, int32_t heads,
                  int32_t head_dim, float inf, int32_t accumulate, int32_t dtype, void* workspace,
                  size_t workspace_bytes, void* stream) {
  PF_TRY(check_dtype(dtype));
  if (!w || !w->w_q || !w->w_k || !w->w_v || !w->w_g || !w->w_o || !w->w_bias)
    return fail(PF_EINVAL_ARG, "triatt: null weight pointer");
  if (!view_ok(zs) || !view_ok(zo)) return fail(PF_EINVAL_ARG, "triatt: bad pair view");
  if (n_rows < 0 || n_keys < 0 || n_q < 0 || c <= 0 || c > 1024 || heads <= 0 || head_dim <= 0)
    return fail(PF_EINVAL_SHAPE, "triatt: bad sizes");
  if (n_valid_keys < 0 || n_valid_keys > n_keys)
    return fail(PF_EINVAL_SHAPE, "triatt: n_valid_keys=%lld outside [0, n_keys=%lld]",
                (long long)n_valid_keys, (long long)n_keys);
  if (q_col0 < 0 || q_col0 + n_q > n_keys)
    return fail(PF_EINVAL_SHAPE, "triatt: query columns [%lld, %lld) outside the slab",
                (long long)q_col0, (long long)(q_col0 + n_q));
  if (bias == nullptr && !(q_col0 == 0 && n_q == n_keys && n_rows == n_keys))
    return fail(PF_EINVAL_ARG, "triatt: bias may be NULL only for the square single-device case");
  if (n_rows == 0 || n_q == 0) return PF_OK;
  size_t need;
  PF_TRY(pf_triatt_workspace_size(n_rows, n_keys, n_q, c, heads, head_dim, dtype, &need));
  PF_TRY(check_ws(workspace, workspace_bytes, need, "triatt"));
  cudaStream_t st = (cudaStream_t)stream;
  if (triatt_tc(c, heads, head_dim, dtype)) {
    set_path("tc");
    return tc::triatt(w, zs, m, bias, b_hs, b_rs, zo, n_rows, n_keys, n_valid_keys, q_col0, n_q,
                      c, heads, head_dim, inf, accumulate, workspace, workspace_bytes, st);
  }
  if (triatt_rows(c, heads, head_dim, dtype)) {
    set_path("tc.rows");
    return tc::rows_triatt(w, zs, m, bias, b_hs, b_rs, zo, n_rows, n_keys, n_valid_keys, q_col0, n_q, c, heads, inf,
                           accumulate, workspace, workspace_bytes, st);
  }
  set_path("simt");
  return simt::triatt(w, zs, m, bias, b_hs, b_rs, zo, n_rows, n_keys, n_valid_keys, q_col0, n_q, c,
                      heads, head_dim, inf, accumulate, dtype, workspace, workspace_bytes, st);
}

// ------------------------------------------------------------------ transition
static bool transition_tc(int c, int nm, int dtype) {
  return dtype == PF_BF16 && !force_simt() && tc::transition_supported(c, nm);
}
static bool transition_rows(int c, int nm, int dtype) {
  return dtype == PF_BF16 && !force_simt() && !tc::transition_supported(c, nm) && tc::rows_transition_supported(c, nm);
}

int pf_transition_workspace_size(int64_t rows, int32_t c, int32_t n_mult, int32_t dtype,
                                 size_t* bytes) {
  PF_TRY(check_dtype(dtype));
  if (!bytes) return fail(PF_EINVAL_ARG, "bytes is NULL");
  *bytes = transition_tc(c, n_mult, dtype)     ? 0
           : transition_rows(c, n_mult, dtype) ? tc::rows_transition_ws_bytes(rows, c, n_mult)
                                               : simt::transition_ws_bytes(rows, c, n_mult);
  return PF_OK;
}

int pf_transition_fwd(const pf_transition_params* w, const void* x, int64_t x_stride, void* out,
                      int64_t out_stride, int64_t rows, int32_t c, int32_t n_mult,
                      int32_t accumulate, int32_t dtype, void* workspace, size_t workspace_bytes,
                      void* stream) {
  PF_TRY(check_dtype(dtype));
  if (!w || !w->w_a || !w->w_b || !w->w_o || !x || !out) return fail(PF_EINVAL_ARG, "transition: null pointer");
  if (rows < 0 || c <= 0 || c > 1024 || n_mult <= 0 || x_stride < c || out_stride < c)
    return fail(PF_EINVAL_SHAPE, "transition: bad sizes");
  if (rows == 0) return PF_OK;
  size_t need;
  PF_TRY(pf_transition_workspace_size(rows, c, n_mult, dtype, &need));
  PF_TRY(check_ws(workspace, workspace_bytes, need, "transition"));
  cudaStream_t st = (cudaStream_t)stream;
  if (transition_tc(c, n_mult, dtype)) {
    set_path("tc");
    return tc::transition(w, x, x_stride, out, out_stride, rows, c, n_mult, accumulate, st);
  }
  if (transition_rows(c, n_mult, dtype)) {
    set_path("tc.rows");
    return tc::rows_transition(w, x, x_stride, out, out_stride, rows, c, n_mult, accumulate, workspace,
                               workspace_bytes, st);
  }
  set_path("simt");
  return simt::transition(w, x, x_stride, out, out_stride, rows, c, n_mult, accumulate, dtype,
                          workspace, workspace_bytes, st);
}

// ------------------------------------------------------------------ AttentionPairBias
static bool apb_bias_tc(int c_z, int heads, int dtype) {
  return dtype == PF_BF16 && !force_simt() && tc::apb_pair_bias_supported(c_z, heads);
}
static bool apb_bias_rows(int c_z, int heads, int dtype) {
  return dtype == PF_BF16 && !force_simt() && !tc::apb_pair_bias_supported(c_z, heads) &&
         tc::rows_bias_supported(c_z, heads);
}

int pf_apb_pair_bias_workspace_size(int64_t n_rows, int64_t n_cols, int32_t c_z, int32_t heads,
                                    int32_t dtype, size_t* bytes) {
  PF_TRY(check_dtype(dtype));
  if (!bytes) return fail(PF_EINVAL_ARG, "bytes is NULL");
  *bytes = apb_bias_tc(c_z, heads, dtype)     ? 0
           : apb_bias_rows(c_z, heads, dtype) ? tc::rows_bias_ws_bytes(n_rows, n_cols, c_z)
                                              : simt::apb_pair_bias_ws_bytes(n_rows * n_cols, c_z, heads);
  return PF_OK;
}

int pf_apb_pair_bias(const pf_apb_params* w, pf_pair_view z, int64_t n_rows, int64_t n_cols,
                     float* bias, int64_t hs, int64_t rs, int32_t c_z, int32_t heads, int32_t dtype,
                     void* workspace, size_t workspace_bytes, void* stream) {
  PF_TRY(check_dtype(dtype));
  if (!w || !w->w_z || !bias || !view_ok(z)) return fail(PF_EINVAL_ARG, "apb_pair_bias: null pointer");
  if (n_rows < 0 || n_cols < 0 || c_z <= 0 || c_z > 1024 || heads <= 0)
    return fail(PF_EINVAL_SHAPE, "apb_pair_bias: bad sizes");
  if (n_rows == 0 || n_cols == 0) return PF_OK;
  size_t need;
  PF_TRY(pf_apb_pair_bias_workspace_size(n_rows, n_cols, c_z, heads, dtype, &need));
  PF_TRY(check_ws(workspace, workspace_bytes, need, "apb_pair_bias"));
  if (apb_bias_tc(c_z, heads, dtype)) {
    set_path("tc");
    return tc::apb_pair_bias(w, z, n_rows, n_cols, bias, hs, rs, (cudaStream_t)stream);
  }
  if (apb_bias_rows(c_z, heads, dtype)) {
    set_path("tc.rows");
    return tc::rows_head_bias(w->ln_z_w, w->ln_z_b, w->w_z, z, n_rows, n_cols, c_z, heads, bias, hs, rs, false,
                              workspace, workspace_bytes, (cudaStream_t)stream);
  }
  set_path("simt");
  return simt::apb_pair_bias(w, z, n_rows, n_cols, bias, hs, rs, c_z, heads, dtype, workspace,
                             workspace_bytes, (cudaStream_t)stream);
}

// the single path's projections on tcgen05 (bf16); the attention itself stays on the fp32 split kernel
static bool apb_single_rows(int c_s, int heads, int dtype) {
  return dtype == PF_BF16 && !force_simt() && heads > 0 && tc::rows_apb_supported(c_s, heads);
}

// workspace of pf_apb_fwd: [own pair bias (only when bias == NULL)] [pair-bias scratch | attention]
static size_t apb_own_bias_bytes(int64_t n, int heads) { return align_up((size_t)heads * n * n * 4, 256); }

int pf_apb_workspace_size(int64_t n, int32_t c_s, int32_t c_z, int32_t heads, int32_t dtype,
                          size_t* bytes) {
  PF_TRY(check_dtype(dtype));
  if (!bytes) return fail(PF_EINVAL_ARG, "bytes is NULL");
  size_t pb = 0;
  PF_TRY(pf_apb_pair_bias_workspace_size(n, n, c_z > 0 ? c_z : 1, heads, dtype, &pb));
  const size_t att = apb_single_rows(c_s, heads, dtype) ? tc::rows_apb_ws_bytes(n, n, c_s, heads)
                                                        : simt::apb_rows_ws_bytes(n, n, c_s, heads > 0 ? heads : 1);
  *bytes = apb_own_bias_bytes(n, heads) + (pb > att ? pb : att);
  return PF_OK;
}

int pf_apb_fwd(const pf_apb_params* w, const void* s_in, void* s_out, pf_pair_view z,
               const float* bias, int64_t n, int32_t c_s, int32_t c_z, int32_t heads,
               int32_t accumulate, int32_t dtype, void* workspace, size_t workspace_bytes,
               void* stream) {
  PF_TRY(check_dtype(dtype));
  if (!w || !w->w_q || !w->w_k || !w->w_v || !w->w_g || !w->w_o || !s_in || !s_out)
    return fail(PF_EINVAL_ARG, "apb: null pointer");
  if (bias == nullptr && (!view_ok(z) || !w->w_z)) return fail(PF_EINVAL_ARG, "apb: need z or bias");
  if (n < 0 || c_s <= 0 || c_s > 1024 || heads <= 0 || c_s % heads != 0)
    return fail(PF_EINVAL_SHAPE, "apb: bad sizes n=%lld c_s=%d heads=%d", (long long)n, c_s, heads);
  if (n == 0) return PF_OK;
  size_t need;
  PF_TRY(pf_apb_workspace_size(n, c_s, c_z, heads, dtype, &need));
  PF_TRY(check_ws(workspace, workspace_bytes, need, "apb"));
  char* ws = (char*)workspace;
  const size_t own = apb_own_bias_bytes(n, heads);
  bool bias_tc = false;
  if (bias == nullptr) {
    float* own_bias = (float*)ws;
    PF_TRY(pf_apb_pair_bias(w, z, n, n, own_bias, n * n, n, c_z, heads, dtype, ws + own,
                            workspace_bytes - own, stream));
    bias = own_bias;
    bias_tc = apb_bias_tc(c_z, heads, dtype) || apb_bias_rows(c_z, heads, dtype);
  }
  // The pair bias (one pass over the N x N x c_z pair tensor) dominates; the single-row
  // attention over N tokens is SIMT in both modes, its projections tensor-core in bf16.
  if (apb_single_rows(c_s, heads, dtype)) {
    set_path(bias_tc ? "tc+simt" : "simt");
    return tc::rows_apb(w, s_in, s_out, bias, n * n, n, n, 0, n, c_s, heads, accumulate, ws + own,
                        workspace_bytes - own, (cudaStream_t)stream);
  }
  set_path(bias_tc ? "tc+simt" : "simt");
  return simt::apb_rows(w, s_in, s_out, bias, n * n, n, n, 0, n, c_s, heads, accumulate, dtype, ws + own,
                        workspace_bytes - own, (cudaStream_t)stream);
}

int pf_apb_rows_workspace_size(int64_t n, int64_t n_q, int32_t c_s, int32_t heads, int32_t dtype,
                               size_t* bytes) {
  PF_TRY(check_dtype(dtype));
  if (!bytes) return fail(PF_EINVAL_ARG, "bytes is NULL");
  if (n < 0 || n_q < 0 || c_s <= 0 || heads <= 0 || c_s % heads) return fail(PF_EINVAL_SHAPE, "apb rows: bad sizes");
  *bytes = apb_single_rows(c_s, heads, dtype) ? tc::rows_apb_ws_bytes(n, n_q, c_s, heads)
                                              : simt::apb_rows_ws_bytes(n, n_q, c_s, heads);
  return PF_OK;
}

int pf_apb_rows_fwd(const pf_apb_params* w, const void* s_in, void* s_out, const float* bias,
                    int64_t head_stride, int64_t row_stride, int64_t n, int64_t q_row0, int64_t n_q,
                    int32_t c_s, int32_t heads, int32_t accumulate, int32_t dtype, void* workspace,
                    size_t workspace_bytes, void* stream) {
  PF_TRY(check_dtype(dtype));
  if (!w || !w->w_q || !w->w_k || !w->w_v || !w->w_g || !w->w_o || !s_in || !s_out || !bias)
    return fail(PF_EINVAL_ARG, "apb_rows: null pointer");
  if (n < 0 || n_q < 0 || q_row0 < 0 || q_row0 + n_q > n || c_s <= 0 || c_s > 1024 || heads <= 0 ||
      c_s % heads != 0)
    return fail(PF_EINVAL_SHAPE, "apb_rows: bad sizes n=%lld q_row0=%lld n_q=%lld c_s=%d heads=%d",
                (long long)n, (long long)q_row0, (long long)n_q, c_s, heads);
  if (n_q == 0) return PF_OK;
  size_t need;
  PF_TRY(pf_apb_rows_workspace_size(n, n_q, c_s, heads, dtype, &need));
  PF_TRY(check_ws(workspace, workspace_bytes, need, "apb_rows"));
  if (apb_single_rows(c_s, heads, dtype)) {
    set_path("tc.rows+simt");
    return tc::rows_apb(w, s_in, s_out, bias, head_stride, row_stride, n, q_row0, n_q, c_s, heads, accumulate,
                        workspace, workspace_bytes, (cudaStream_t)stream);
  }
  set_path("simt");
  return simt::apb_rows(w, s_in, s_out, bias, head_stride, row_stride, n, q_row0, n_q, c_s, heads,
                        accumulate, dtype, workspace, workspace_bytes, (cudaStream_t)stream);
}

// ------------------------------------------------------------------ OuterProductMean
static bool opm_rows(int c_m, int c_hidden, int c_z, int dtype) {
  return dtype == PF_BF16 && !force_simt() && tc::rows_opm_supported(c_m, c_hidden, c_z);
}

int pf_opm_workspace_size(int64_t n_seq, int64_t n_res, int64_t n_rows, int64_t n_cols, int32_t c_m,
                          int32_t c_hidden, int32_t c_z, int32_t dtype, size_t* bytes) {
  PF_TRY(check_dtype(dtype));
  if (!bytes) return fail(PF_EINVAL_ARG, "bytes is NULL");
  if (n_seq < 0 || n_res < 0 || n_rows < 0 || n_cols < 0 || c_m <= 0 || c_hidden <= 0 || c_z <= 0)
    return fail(PF_EINVAL_SHAPE, "opm: bad sizes");
  *bytes = opm_rows(c_m, c_hidden, c_z, dtype)
               ? tc::rows_opm_ws_bytes(n_seq, n_res, n_rows, n_cols, c_m, c_hidden)
               : simt::opm_ws_bytes(n_seq, n_res, n_rows, n_cols, c_m, c_hidden, c_z);
  return PF_OK;
}

int pf_opm_fwd(const pf_opm_params* w, pf_pair_view m, pf_mask_view mask, pf_pair_view z_out, int64_t n_seq,
               int64_t n_res, int64_t row0, int64_t n_rows, int64_t col0, int64_t n_cols, int32_t c_m,
               int32_t c_hidden, int32_t c_z, float eps, int32_t accumulate, int32_t dtype, void* workspace,
               size_t workspace_bytes, void* stream) {
  PF_TRY(check_dtype(dtype));
  if (!w || !w->w_1 || !w->w_2 || !w->w_out || !w->ln_w) return fail(PF_EINVAL_ARG, "opm: null weight pointer");
  if (!view_ok(m) || !view_ok(z_out)) return fail(PF_EINVAL_ARG, "opm: bad view");
  if (n_seq < 0 || n_res < 0 || c_m <= 0 || c_m > 1024 || c_hidden <= 0 || c_hidden > 64 || c_z <= 0 ||
      c_z > 1024)
    return fail(PF_EINVAL_SHAPE, "opm: bad sizes n_seq=%lld n_res=%lld c_m=%d c_hidden=%d c_z=%d",
                (long long)n_seq, (long long)n_res, c_m, c_hidden, c_z);
  if (row0 < 0 || n_rows < 0 || row0 + n_rows > n_res || col0 < 0 || n_cols < 0 || col0 + n_cols > n_res)
    return fail(PF_EINVAL_SHAPE, "opm: tile rows [%lld, %lld) x cols [%lld, %lld) outside the %lld residues",
                (long long)row0, (long long)(row0 + n_rows), (long long)col0, (long long)(col0 + n_cols),
                (long long)n_res);
  if (n_rows == 0 || n_cols == 0) return PF_OK;
  size_t need;
  PF_TRY(pf_opm_workspace_size(n_seq, n_res, n_rows, n_cols, c_m, c_hidden, c_z, dtype, &need));
  PF_TRY(check_ws(workspace, workspace_bytes, need, "opm"));
  cudaStream_t st = (cudaStream_t)stream;
  if (n_seq == 0) return fail(PF_EINVAL_SHAPE, "opm: the MSA representation has no sequences (n_seq = 0)");
  if (opm_rows(c_m, c_hidden, c_z, dtype)) {
    set_path("tc.rows");
    return tc::rows_opm(w, m, mask, z_out, n_seq, n_res, row0, n_rows, col0, n_cols, c_m, c_hidden, c_z, eps,
                        accumulate, workspace, workspace_bytes, st);
  }
  set_path("simt");
  return simt::opm(w, m, mask, z_out, n_seq, n_res, row0, n_rows, col0, n_cols, c_m, c_hidden, c_z, eps, accumulate,
                   dtype, workspace, workspace_bytes, st);
}

// ------------------------------------------------------------------ trunk pair input, recycling
int pf_trunk_init_workspace_size(int64_t n_rows, int64_t n_cols, int32_t c_s, int32_t c_z, int32_t r_max,
                                 int32_t s_max, int32_t dtype, size_t* bytes) {
  PF_TRY(check_dtype(dtype));
  if (!bytes) return fail(PF_EINVAL_ARG, "bytes is NULL");
  if (n_rows < 0 || n_cols < 0 || c_s <= 0 || c_z <= 0 || r_max < 0 || s_max < 0)
    return fail(PF_EINVAL_SHAPE, "trunk init: bad sizes");
  *bytes = trunk::init_ws_bytes(n_rows, n_cols, c_z, r_max, s_max);
  return PF_OK;
}

int pf_trunk_init_fwd(const pf_trunk_init_params* w, const void* s_init, int64_t s_stride, pf_token_ids ids,
                      pf_mask_view token_bonds, pf_pair_view z_out, int64_t n_token, int64_t row0, int64_t n_rows,
                      int64_t col0, int64_t n_cols, int32_t c_s, int32_t c_z, int32_t r_max, int32_t s_max,
                      int32_t dtype, void* workspace, size_t workspace_bytes, void* stream) {
  PF_TRY(check_dtype(dtype));
  if (!w || !w->w_zinit1 || !w->w_zinit2 || !w->w_relp || !w->w_bond || !s_init)
    return fail(PF_EINVAL_ARG, "trunk init: null weight or s_init");
  if (!ids.asym_id || !ids.residue_index || !ids.entity_id || !ids.token_index || !ids.sym_id)
    return fail(PF_EINVAL_ARG, "trunk init: null token id array");
  if (!view_ok(z_out)) return fail(PF_EINVAL_ARG, "trunk init: bad output view");
  if (n_token < 0 || c_s <= 0 || c_s > 4096 || c_z <= 0 || c_z > 1024 || c_z % 8 || r_max < 0 || r_max > 1024 ||
      s_max < 0 || s_max > 1024 || s_stride < c_s)
    return fail(PF_EINVAL_SHAPE, "trunk init: bad sizes c_s=%d c_z=%d (c_z a multiple of 8) r_max=%d s_max=%d", c_s,
                c_z, r_max, s_max);
  if (row0 < 0 || n_rows < 0 || row0 + n_rows > n_token || col0 < 0 || n_cols < 0 || col0 + n_cols > n_token)
    return fail(PF_EINVAL_SHAPE, "trunk init: tile rows [%lld, %lld) x cols [%lld, %lld) outside %lld tokens",
                (long long)row0, (long long)(row0 + n_rows), (long long)col0, (long long)(col0 + n_cols),
                (long long)n_token);
  const size_t esz = dtype == PF_F32 ? 4 : 2;
  if (((uintptr_t)z_out.ptr) % 16 || (z_out.row_stride * esz) % 16 || (z_out.col_stride * esz) % 16)
    return fail(PF_EINVAL_SHAPE, "trunk init: the output view needs 16-byte aligned positions");
  if (n_rows == 0 || n_cols == 0) return PF_OK;
  if (n_rows > 65535) return fail(PF_EUNSUPPORTED, "trunk init: tile of %lld rows > 65535", (long long)n_rows);
  size_t need;
  PF_TRY(pf_trunk_init_workspace_size(n_rows, n_cols, c_s, c_z, r_max, s_max, dtype, &need));
  PF_TRY(check_ws(workspace, workspace_bytes, need, "trunk init"));
  set_path("simt");
  return trunk::init(w, s_init, s_stride, ids, token_bonds, z_out, row0, n_rows, col0, n_cols, c_s, c_z, r_max,
                     s_max, dtype, workspace, workspace_bytes, (cudaStream_t)stream);
}

static bool pair_ln_linear_rows(int c_in, int c_out, int dtype) {
  return dtype == PF_BF16 && !force_simt() && tc::rows_pair_ln_linear_supported(c_in, c_out);
}

int pf_pair_ln_linear_workspace_size(int64_t n_rows, int64_t n_cols, int32_t c_in, int32_t c_out, int32_t dtype,
                                     size_t* bytes) {
  PF_TRY(check_dtype(dtype));
  if (!bytes) return fail(PF_EINVAL_ARG, "bytes is NULL");
  if (n_rows < 0 || n_cols < 0 || c_in <= 0 || c_out <= 0) return fail(PF_EINVAL_SHAPE, "pair LN-linear: bad sizes");
  *bytes = pair_ln_linear_rows(c_in, c_out, dtype) ? tc::rows_pair_ln_linear_ws_bytes(n_rows, n_cols, c_in)
                                                   : simt::pair_ln_linear_ws_bytes(n_rows, n_cols, c_in, c_out);
  return PF_OK;
}

int pf_pair_ln_linear_fwd(const pf_pair_linear_params* w, pf_pair_view z_in, pf_pair_view z_out, int64_t n_rows,
                          int64_t n_cols, int32_t c_in, int32_t c_out, int32_t accumulate, int32_t dtype,
                          void* workspace, size_t workspace_bytes, void* stream) {
  PF_TRY(check_dtype(dtype));
  if (!w || !w->w || !w->ln_w) return fail(PF_EINVAL_ARG, "pair LN-linear: null weight pointer");
  if (!view_ok(z_in) || !view_ok(z_out)) return fail(PF_EINVAL_ARG, "pair LN-linear: bad view");
  if (n_rows < 0 || n_cols < 0 || c_in <= 0 || c_in > 1024 || c_out <= 0 || c_out > 1024)
    return fail(PF_EINVAL_SHAPE, "pair LN-linear: bad sizes c_in=%d c_out=%d", c_in, c_out);
  if (z_in.ptr == z_out.ptr) return fail(PF_EINVAL_ARG, "pair LN-linear: z_out must not alias z_in");
  if (n_rows == 0 || n_cols == 0) return PF_OK;
  size_t need;
  PF_TRY(pf_pair_ln_linear_workspace_size(n_rows, n_cols, c_in, c_out, dtype, &need));
  PF_TRY(check_ws(workspace, workspace_bytes, need, "pair LN-linear"));
  cudaStream_t st = (cudaStream_t)stream;
  if (pair_ln_linear_rows(c_in, c_out, dtype)) {
    set_path("tc.rows");
    return tc::rows_pair_ln_linear(w, z_in, z_out, n_rows, n_cols, c_in, c_out, accumulate, workspace,
                                   workspace_bytes, st);
  }
  set_path("simt");
  return simt::pair_ln_linear(w, z_in, z_out, n_rows, n_cols, c_in, c_out, accumulate, dtype, workspace,
                              workspace_bytes, st);
}

// ------------------------------------------------------------------ pair heads and conditioning
static bool pair_head_rows(int c_z, int n_bins, int dtype) {
  return dtype == PF_BF16 && !force_simt() && tc::rows_pair_head_supported(c_z, n_bins);
}

int pf_pair_head_workspace_size(int64_t n_rows, int64_t n_cols, int32_t c_z, int32_t n_bins, int32_t dtype,
                                size_t* bytes) {
  PF_TRY(check_dtype(dtype));
  if (!bytes) return fail(PF_EINVAL_ARG, "bytes is NULL");
  if (n_rows < 0 || n_cols < 0 || c_z <= 0 || n_bins <= 0) return fail(PF_EINVAL_SHAPE, "pair head: bad sizes");
  *bytes = pair_head_rows(c_z, n_bins, dtype) ? tc::rows_pair_head_ws_bytes(n_rows, n_cols, c_z)
                                              : simt::pair_head_ws_bytes(n_rows, n_cols, c_z, n_bins);
  return PF_OK;
}

int pf_pair_head_fwd(const pf_pair_head_params* w, int32_t mode, pf_pair_view z, pf_pair_view zt, int64_t n_rows,
                     int64_t n_cols, int32_t c_z, int32_t n_bins, pf_pair_view logits, int32_t logits_dtype,
                     float* contact, int64_t contact_rs, int64_t contact_cs, int32_t contact_bins, int32_t dtype,
                     void* workspace, size_t workspace_bytes, void* stream) {
  PF_TRY(check_dtype(dtype));
  PF_TRY(check_dtype(logits_dtype));
  if (mode != PF_HEAD_PLAIN && mode != PF_HEAD_SYM_IN && mode != PF_HEAD_SYM_OUT)
    return fail(PF_EINVAL_ARG, "pair head: unknown mode %d", mode);
  if (!w || !w->w) return fail(PF_EINVAL_ARG, "pair head: null weight pointer");
  if (!view_ok(z) || !view_ok(logits) || (mode != PF_HEAD_PLAIN && !view_ok(zt)))
    return fail(PF_EINVAL_ARG, "pair head: bad view");
  if (dtype == PF_F32 && logits_dtype != PF_F32) return fail(PF_EINVAL_DTYPE, "pair head: fp32 input needs fp32 logits");
  if (n_rows < 0 || n_cols < 0 || c_z <= 0 || c_z > 1024 || n_bins <= 0 || n_bins > 256)
    return fail(PF_EINVAL_SHAPE, "pair head: bad sizes c_z=%d n_bins=%d (1..256 bins)", c_z, n_bins);
  if (contact && (contact_bins < 0 || contact_bins > n_bins || contact_rs < 0 || contact_cs < 0))
    return fail(PF_EINVAL_ARG, "pair head: contact_bins %d outside [0, %d] or bad contact strides", contact_bins,
                n_bins);
  const size_t lsz = logits_dtype == PF_F32 ? 4 : 2;
  if (((uintptr_t)logits.ptr) % lsz) return fail(PF_EINVAL_ARG, "pair head: misaligned logits");
  if (n_rows == 0 || n_cols == 0) return PF_OK;
  size_t need;
  PF_TRY(pf_pair_head_workspace_size(n_rows, n_cols, c_z, n_bins, dtype, &need));
  PF_TRY(check_ws(workspace, workspace_bytes, need, "pair head"));
  cudaStream_t st = (cudaStream_t)stream;
  if (pair_head_rows(c_z, n_bins, dtype)) {
    set_path("tc.rows");
    return tc::rows_pair_head(w, mode, z, zt, n_rows, n_cols, c_z, n_bins, logits, logits_dtype == PF_F32, contact,
                              contact_rs, contact_cs, contact_bins, workspace, workspace_bytes, st);
  }
  set_path("simt");
  return simt::pair_head(w, mode, z, zt, n_rows, n_cols, c_z, n_bins, logits, logits_dtype == PF_F32, contact,
                         contact_rs, contact_cs, contact_bins, dtype, workspace, workspace_bytes, st);
}

int pf_confidence_pair_init_workspace_size(int64_t n_rows, int64_t n_cols, int32_t c_s_inputs, int32_t c_z,
                                           int32_t n_dist_bins, int32_t dtype, size_t* bytes) {
  PF_TRY(check_dtype(dtype));
  if (!bytes) return fail(PF_EINVAL_ARG, "bytes is NULL");
  if (n_rows < 0 || n_cols < 0 || c_s_inputs <= 0 || c_z <= 0 || n_dist_bins < 0)
    return fail(PF_EINVAL_SHAPE, "confidence pair init: bad sizes");
  *bytes = heads::conf_init_ws_bytes(n_rows, n_cols, c_z, n_dist_bins);
  return PF_OK;
}

static int check_pair_io(const pf_pair_view& a, const pf_pair_view& b, int dtype, const char* what) {
  const size_t esz = dtype == PF_F32 ? 4 : 2;
  for (const pf_pair_view* v : {&a, &b})
    if (((uintptr_t)v->ptr) % 16 || (v->row_stride * esz) % 16 || (v->col_stride * esz) % 16)
      return fail(PF_EINVAL_SHAPE, "%s: pair views need 16-byte aligned positions", what);
  return PF_OK;
}

static int check_tile(int64_t n_token, int64_t row0, int64_t n_rows, int64_t col0, int64_t n_cols, const char* what) {
  if (row0 < 0 || n_rows < 0 || row0 + n_rows > n_token || col0 < 0 || n_cols < 0 || col0 + n_cols > n_token)
    return fail(PF_EINVAL_SHAPE, "%s: tile rows [%lld, %lld) x cols [%lld, %lld) outside %lld tokens", what,
                (long long)row0, (long long)(row0 + n_rows), (long long)col0, (long long)(col0 + n_cols),
                (long long)n_token);
  return PF_OK;
}

int pf_confidence_pair_init_fwd(const pf_confidence_init_params* w, const void* s_inputs, int64_t s_stride,
                                const float* coords, pf_pair_view z_trunk, pf_pair_view z_out, int64_t n_token,
                                int64_t row0, int64_t n_rows, int64_t col0, int64_t n_cols, int32_t c_s_inputs,
                                int32_t c_z, int32_t n_dist_bins, int32_t dtype, void* workspace,
                                size_t workspace_bytes, void* stream) {
  PF_TRY(check_dtype(dtype));
  if (!w || !w->w_s1 || !w->w_s2 || !w->w_d || !w->w_d0 || !w->lower_bins || !w->upper_bins || !s_inputs || !coords)
    return fail(PF_EINVAL_ARG, "confidence pair init: null weight, bins, s_inputs or coords");
  if (!view_ok(z_trunk) || !view_ok(z_out)) return fail(PF_EINVAL_ARG, "confidence pair init: bad view");
  if (n_token < 0 || c_s_inputs <= 0 || c_s_inputs > 4096 || c_z <= 0 || c_z > 1024 || c_z % 8 || n_dist_bins < 1 ||
      n_dist_bins > 64 || s_stride < c_s_inputs)
    return fail(PF_EINVAL_SHAPE,
                "confidence pair init: bad sizes c_s_inputs=%d c_z=%d (a multiple of 8) bins=%d (1..64)", c_s_inputs,
                c_z, n_dist_bins);
  PF_TRY(check_tile(n_token, row0, n_rows, col0, n_cols, "confidence pair init"));
  PF_TRY(check_pair_io(z_trunk, z_out, dtype, "confidence pair init"));
  if (n_rows == 0 || n_cols == 0) return PF_OK;
  size_t need;
  PF_TRY(pf_confidence_pair_init_workspace_size(n_rows, n_cols, c_s_inputs, c_z, n_dist_bins, dtype, &need));
  PF_TRY(check_ws(workspace, workspace_bytes, need, "confidence pair init"));
  set_path("simt");
  return heads::conf_init(w, s_inputs, s_stride, coords, z_trunk, z_out, row0, n_rows, col0, n_cols, c_s_inputs, c_z,
                          n_dist_bins, dtype, workspace, workspace_bytes, (cudaStream_t)stream);
}

int pf_diffusion_pair_cond_workspace_size(int64_t n_rows, int64_t n_cols, int32_t c_z, int32_t c_zd, int32_t r_max,
                                          int32_t s_max, int32_t dtype, size_t* bytes) {
  PF_TRY(check_dtype(dtype));
  if (!bytes) return fail(PF_EINVAL_ARG, "bytes is NULL");
  if (n_rows < 0 || n_cols < 0 || c_z <= 0 || c_zd <= 0 || r_max < 0 || s_max < 0)
    return fail(PF_EINVAL_SHAPE, "diffusion pair: bad sizes");
  *bytes = heads::diffusion_ws_bytes(n_rows, n_cols, c_z, c_zd, r_max, s_max, dtype);
  return PF_OK;
}

int pf_diffusion_pair_cond_fwd(const pf_diffusion_pair_params* w, pf_pair_view z_trunk, pf_token_ids ids,
                               pf_pair_view z_out, int64_t n_token, int64_t row0, int64_t n_rows, int64_t col0,
                               int64_t n_cols, int32_t c_z, int32_t c_zd, int32_t r_max, int32_t s_max, int32_t dtype,
                               void* workspace, size_t workspace_bytes, void* stream) {
  PF_TRY(check_dtype(dtype));
  if (!w || !w->w_relp || !w->ln_z_w || !w->w_z || !w->t1.w_a || !w->t1.w_b || !w->t1.w_o || !w->t2.w_a ||
      !w->t2.w_b || !w->t2.w_o)
    return fail(PF_EINVAL_ARG, "diffusion pair: null weight pointer");
  if (c_z != c_zd && (!w->ln_zt_w || !w->w_zt))
    return fail(PF_EINVAL_ARG, "diffusion pair: c_z %d != c_zd %d needs layernorm_z_trunk and linear_no_bias_z_trunk",
                c_z, c_zd);
  if (!ids.asym_id || !ids.residue_index || !ids.entity_id || !ids.token_index || !ids.sym_id)
    return fail(PF_EINVAL_ARG, "diffusion pair: null token id array");
  if (!view_ok(z_trunk) || !view_ok(z_out)) return fail(PF_EINVAL_ARG, "diffusion pair: bad view");
  if (n_token < 0 || c_z <= 0 || c_z > 1024 || c_z % 8 || c_zd <= 0 || c_zd > 512 || c_zd % 8 || r_max < 0 ||
      r_max > 1024 || s_max < 0 || s_max > 1024)
    return fail(PF_EINVAL_SHAPE,
                "diffusion pair: bad sizes c_z=%d c_zd=%d (multiples of 8, c_zd <= 512) r_max=%d s_max=%d", c_z, c_zd,
                r_max, s_max);
  PF_TRY(check_tile(n_token, row0, n_rows, col0, n_cols, "diffusion pair"));
  PF_TRY(check_pair_io(z_trunk, z_out, dtype, "diffusion pair"));
  if (n_rows == 0 || n_cols == 0) return PF_OK;
  const size_t need = heads::diffusion_ws_bytes(n_rows, n_cols, c_z, c_zd, r_max, s_max, dtype);
  PF_TRY(check_ws(workspace, workspace_bytes, need, "diffusion pair"));
  PF_TRY(heads::diffusion(w, z_trunk, ids, z_out, row0, n_rows, col0, n_cols, c_z, c_zd, r_max, s_max, dtype,
                          workspace, workspace_bytes, (cudaStream_t)stream));
  set_path(dtype == PF_BF16 && !force_simt() ? "tc.rows" : "simt");
  return PF_OK;
}

}  // extern "C"
