// pf_simt.h -- generic SIMT path (fp32 arithmetic), see pf_simt.cu.
#pragma once
#include <cuda_runtime.h>
#include "../../include/pairformer_b200.h"

namespace pf {
namespace simt {

int layernorm(const void* x, void* y, const float* g, const float* b, int64_t rows, int c,
              float eps, int dtype, cudaStream_t st);

size_t trimul_ws_bytes(int64_t n_i, int64_t n_j, int64_t n_k, int c_z, int c_h);
int trimul(const pf_trimul_params* p, pf_pair_view za, pf_pair_view zb, pf_mask_view ma,
           pf_mask_view mb, pf_pair_view zg, pf_pair_view zo, int64_t n_i, int64_t n_j, int64_t n_k, int c_z,
           int c_h, int acc, int dtype, void* ws, size_t ws_bytes, cudaStream_t st);
size_t trimul_project_ws_bytes(int64_t n_rows, int64_t n_cols, int c_z, int c_h);
int trimul_project(const pf_trimul_params* p, pf_pair_view z, pf_mask_view m, int64_t n_rows, int64_t n_cols,
                   int c_z, int c_h, int dtype, void* a, void* b, int64_t ld, void* ws, size_t ws_bytes,
                   cudaStream_t st);
size_t trimul_combine_ws_bytes(int64_t n_i, int64_t n_j, int c_z, int c_h);
int trimul_combine(const pf_trimul_params* p, const void* a, const void* b, int64_t ld, int64_t n_i, int64_t n_j,
                   int64_t n_k, pf_pair_view zg, pf_pair_view zo, int c_z, int c_h, int acc, int dtype, void* ws,
                   size_t ws_bytes, cudaStream_t st);

size_t triatt_ws_bytes(int64_t n_rows, int64_t n_keys, int64_t n_q, int c, int H, int d);
int triatt(const pf_triatt_params* p, pf_pair_view zs, pf_mask_view m, const void* bias,
           int64_t b_hs, int64_t b_rs, pf_pair_view zo, int64_t n_rows, int64_t n_keys,
           int64_t n_valid, int64_t q_col0, int64_t n_q, int c, int H, int d, float inf, int acc,
           int dtype, void* ws, size_t ws_bytes, cudaStream_t st);
size_t triatt_bias_ws_bytes(int64_t n_rows, int64_t n_cols, int c, int H);
int triatt_bias(const pf_triatt_params* p, pf_pair_view z, int64_t n_rows, int64_t n_cols,
                void* bias, int64_t hs, int64_t rs, int c, int H, int dtype, void* ws,
                size_t ws_bytes, cudaStream_t st);

size_t transition_ws_bytes(int64_t rows, int c, int nm);
int transition(const pf_transition_params* p, const void* x, int64_t xs, void* out, int64_t os,
               int64_t rows, int c, int nm, int acc, int dtype, void* ws, size_t ws_bytes,
               cudaStream_t st);

size_t apb_pair_bias_ws_bytes(int64_t P, int c_z, int H);
int apb_pair_bias(const pf_apb_params* p, pf_pair_view z, int64_t n_rows, int64_t n_cols,
                  float* bias, int64_t hs, int64_t rs, int c_z, int H, int dtype, void* ws,
                  size_t ws_bytes, cudaStream_t st);
size_t apb_rows_ws_bytes(int64_t n, int64_t nq, int c_s, int H);
int apb_rows(const pf_apb_params* p, const void* s_in, void* s_out, const float* bias, int64_t b_hs,
             int64_t b_rs, int64_t n, int64_t q0, int64_t nq, int c_s, int H, int acc, int dtype, void* ws,
             size_t ws_bytes, cudaStream_t st);

// Single-representation attention with a pair bias (fp32), split over the keys and merged:
// o(j, h*d + e) for queries j < n_q over keys < n; q(j) at q + j*q_ps, k/v(key) at + key*kv_ps,
// bias(h, j, key) at bias + h*b_hs + j*b_rs + key; `part` holds attn_split_part_floats floats.
size_t attn_split_part_floats(int64_t n, int64_t nq, int c_s, int H);
int attn_split(int d, const float* q, int64_t q_ps, const float* k, const float* v, int64_t kv_ps, const float* bias,
               int64_t b_hs, int64_t b_rs, int64_t n_q, int64_t n, int H, float* part, float* o, int64_t o_ps,
               cudaStream_t st);

// OuterProductMean (fp32 arithmetic) of the rows [row0, row0 + n_rows) x cols [col0, col0 + n_cols),
// and the norm tile sum_s mask(s, i) mask(s, j) + eps it divides by (shared with the bf16 path).
size_t opm_ws_bytes(int64_t n_seq, int64_t n_res, int64_t n_rows, int64_t n_cols, int c_m, int C, int c_z);
int opm(const pf_opm_params* p, pf_pair_view m, pf_mask_view mask, pf_pair_view z_out, int64_t n_seq, int64_t n_res,
        int64_t row0, int64_t n_rows, int64_t col0, int64_t n_cols, int c_m, int C, int c_z, float eps, int acc,
        int dtype, void* ws, size_t ws_bytes, cudaStream_t st);
int opm_norm(pf_mask_view m, int64_t n_seq, int64_t row0, int64_t n_rows, int64_t col0, int64_t n_cols, float eps,
             float* norm, cudaStream_t st);

// c[m][n] = sum_k a[m*lda + k] w[n*k + k'] (fp32 result; a and w in the storage type)
template <class T>
int gemm_rows(const T* a, int64_t lda, const T* w, float* c, int64_t m, int n, int k, cudaStream_t st);
// z_out (+)= W LN(z_in) on pair views (fp32 arithmetic)
size_t pair_ln_linear_ws_bytes(int64_t n_rows, int64_t n_cols, int c_in, int c_out);
int pair_ln_linear(const pf_pair_linear_params* p, pf_pair_view zi, pf_pair_view zo, int64_t n_rows, int64_t n_cols,
                   int c_in, int c_out, int acc, int dtype, void* ws, size_t ws_bytes, cudaStream_t st);

// bin logits of a pair tile (pf_pair_head_fwd), fp32 arithmetic
size_t pair_head_ws_bytes(int64_t n_rows, int64_t n_cols, int c_z, int n_bins);
int pair_head(const pf_pair_head_params* p, int mode, pf_pair_view z, pf_pair_view zt, int64_t n_rows, int64_t n_cols,
              int c_z, int n_bins, pf_pair_view lo, int lo_f32, float* contact, int64_t crs, int64_t ccs, int cbins,
              int dtype, void* ws, size_t ws_bytes, cudaStream_t st);

}  // namespace simt

namespace heads {
// the confidence head's pair input and the diffusion pair conditioning on a tile (pf_heads.cu)
size_t conf_init_ws_bytes(int64_t n_rows, int64_t n_cols, int c_z, int n_bins);
int conf_init(const pf_confidence_init_params* p, const void* s, int64_t s_stride, const float* coords,
              pf_pair_view zi, pf_pair_view zo, int64_t row0, int64_t n_rows, int64_t col0, int64_t n_cols, int c_s,
              int c_z, int n_bins, int dtype, void* ws, size_t ws_bytes, cudaStream_t st);
size_t diffusion_ws_bytes(int64_t n_rows, int64_t n_cols, int c_z, int c_zd, int r_max, int s_max, int dtype);
int diffusion(const pf_diffusion_pair_params* p, pf_pair_view zt, pf_token_ids ids, pf_pair_view zo, int64_t row0,
              int64_t n_rows, int64_t col0, int64_t n_cols, int c_z, int c_zd, int r_max, int s_max, int dtype,
              void* ws, size_t ws_bytes, cudaStream_t st);
}  // namespace heads

namespace trunk {
// the trunk's pair input on a tile (pf_trunk.cu)
size_t init_ws_bytes(int64_t n_rows, int64_t n_cols, int c_z, int r_max, int s_max);
int init(const pf_trunk_init_params* p, const void* s, int64_t s_stride, pf_token_ids ids, pf_mask_view bonds,
         pf_pair_view zo, int64_t row0, int64_t n_rows, int64_t col0, int64_t n_cols, int c_s, int c_z, int r_max,
         int s_max, int dtype, void* ws, size_t ws_bytes, cudaStream_t st);
}  // namespace trunk
}  // namespace pf
