// pf_tc.h -- tcgen05 / TMA (sm_100a) kernels of the bf16 path. Each *_supported() says
// whether the shape is covered: the fused c = 128 kernels first, then the general-width
// path; the API layer routes what neither covers (and every fp32 request) to the SIMT path.
#pragma once
#include <cuda_runtime.h>
#include "../../include/pairformer_b200.h"

namespace pf {
namespace tc {

bool trimul_supported(int64_t n_i, int64_t n_j, int64_t n_k, int c_z, int c_h);
size_t trimul_ws_bytes(int64_t n_i, int64_t n_j, int64_t n_k, int c_z, int c_h);
int trimul(const pf_trimul_params* p, pf_pair_view za, pf_pair_view zb, pf_mask_view ma,
           pf_mask_view mb, pf_pair_view zg, pf_pair_view zo, int64_t n_i, int64_t n_j, int64_t n_k, int c_z,
           int c_h, int acc, void* ws, size_t ws_bytes, cudaStream_t st);
int trimul_project(const pf_trimul_params* p, pf_pair_view z, pf_mask_view m, int64_t n_rows,
                   int64_t n_cols, void* a, void* b, int64_t ld, cudaStream_t st);
size_t trimul_combine_ws_bytes(int64_t n_i, int64_t n_j);
int trimul_combine(const pf_trimul_params* p, const void* a, const void* b, int64_t ld, int64_t n_i,
                   int64_t n_j, int64_t n_k, pf_pair_view zg, pf_pair_view zo, int acc, void* ws,
                   size_t ws_bytes, cudaStream_t st);

bool triatt_bias_supported(int c, int H);
int triatt_bias(const pf_triatt_params* p, pf_pair_view z, int64_t n_rows, int64_t n_cols,
                void* bias, int64_t hs, int64_t rs, int c, int H, cudaStream_t st);
bool triatt_supported(int c, int H, int d);
size_t triatt_ws_bytes(int64_t n_rows, int64_t n_keys, int64_t n_q, int c, int H, int d);
int triatt(const pf_triatt_params* p, pf_pair_view zs, pf_mask_view m, const void* bias,
           int64_t b_hs, int64_t b_rs, pf_pair_view zo, int64_t n_rows, int64_t n_keys,
           int64_t n_valid, int64_t q_col0, int64_t n_q, int c, int H, int d, float inf, int acc,
           void* ws, size_t ws_bytes, cudaStream_t st);

bool apb_pair_bias_supported(int c_z, int heads);
int apb_pair_bias(const pf_apb_params* p, pf_pair_view z, int64_t n_rows, int64_t n_cols, float* bias,
                  int64_t hs, int64_t rs, cudaStream_t st);

bool transition_supported(int c, int nm);
int transition(const pf_transition_params* p, const void* x, int64_t xs, void* out, int64_t os,
               int64_t rows, int c, int nm, int acc, cudaStream_t st);


// General-width path (pf_tc_rows.cu): every width with c % 8 == 0 (and c_h % 64 == 0 for the
// triangle update, H * 32 % 128 == 0 with d = 32 for triangle attention), on tcgen05 GEMMs with
// LayerNorm passes between them and the width-independent contraction and attention core.
bool rows_trimul_supported(int c_z, int c_h);
size_t rows_trimul_ws_bytes(int64_t n_i, int64_t n_j, int64_t n_k, int c_z, int c_h);
int rows_trimul(const pf_trimul_params* p, pf_pair_view za, pf_pair_view zb, pf_mask_view ma, pf_mask_view mb,
                pf_pair_view zg, pf_pair_view zo, int64_t n_i, int64_t n_j, int64_t n_k, int c_z, int c_h, int acc,
                void* ws, size_t ws_bytes, cudaStream_t st);
size_t rows_trimul_project_ws_bytes(int64_t n_rows, int64_t n_cols, int c_z, int c_h);
int rows_trimul_project(const pf_trimul_params* p, pf_pair_view z, pf_mask_view m, int64_t n_rows, int64_t n_cols,
                        int c_z, int c_h, void* a, void* b, int64_t ld, void* ws, size_t ws_bytes, cudaStream_t st);
size_t rows_trimul_combine_ws_bytes(int64_t n_i, int64_t n_j, int c_z, int c_h);
int rows_trimul_combine(const pf_trimul_params* p, const void* a, const void* b, int64_t ld, int64_t n_i,
                        int64_t n_j, int64_t n_k, pf_pair_view zg, pf_pair_view zo, int c_z, int c_h, int acc,
                        void* ws, size_t ws_bytes, cudaStream_t st);
bool rows_triatt_supported(int c, int H, int d);
size_t rows_triatt_ws_bytes(int64_t n_rows, int64_t n_keys, int64_t n_q, int c, int H);
int rows_triatt(const pf_triatt_params* p, pf_pair_view zs, pf_mask_view m, const void* bias, int64_t b_hs,
                int64_t b_rs, pf_pair_view zo, int64_t n_rows, int64_t n_keys, int64_t n_valid, int64_t q_col0,
                int64_t n_q, int c, int H, float inf, int acc, void* ws, size_t ws_bytes, cudaStream_t st);
bool rows_bias_supported(int c, int H);
size_t rows_bias_ws_bytes(int64_t n_rows, int64_t n_cols, int c);
// bias(h, r, s) = W LN(z(r, s)): f16 in log2 units (triangle attention) or fp32 (pair bias)
int rows_head_bias(const float* ln_w, const float* ln_b, const void* w_bias, pf_pair_view z, int64_t n_rows,
                   int64_t n_cols, int c, int H, void* bias, int64_t hs, int64_t rs, bool f16_log2, void* ws,
                   size_t ws_bytes, cudaStream_t st);
bool rows_transition_supported(int c, int nm);
size_t rows_transition_ws_bytes(int64_t rows, int c, int nm);
int rows_transition(const pf_transition_params* p, const void* x, int64_t xs, void* out, int64_t os, int64_t rows,
                    int c, int nm, int acc, void* ws, size_t ws_bytes, cudaStream_t st);

// AttentionPairBias single path (bf16): LN_a and the q / k / v / g / o projections on tcgen05,
// the pair-biased attention itself on the fp32 split kernel; rows [q0, q0 + nq) of s_out.
bool rows_apb_supported(int c_s, int H);
size_t rows_apb_ws_bytes(int64_t n, int64_t nq, int c_s, int H);
int rows_apb(const pf_apb_params* p, const void* s_in, void* s_out, const float* bias, int64_t b_hs, int64_t b_rs,
             int64_t n, int64_t q0, int64_t nq, int c_s, int H, int acc, void* ws, size_t ws_bytes, cudaStream_t st);

// OuterProductMean (bf16, c_hidden = 32): projections, the outer product over the sequences and
// W_out on tcgen05; see pf_opm_fwd.
bool rows_opm_supported(int c_m, int c_hidden, int c_z);
size_t rows_opm_ws_bytes(int64_t n_seq, int64_t n_res, int64_t n_rows, int64_t n_cols, int c_m, int C);
int rows_opm(const pf_opm_params* p, pf_pair_view m, pf_mask_view mask, pf_pair_view z_out, int64_t S, int64_t N,
             int64_t row0, int64_t nr, int64_t col0, int64_t nc, int c_m, int C, int c_z, float eps, int acc,
             void* ws, size_t ws_bytes, cudaStream_t st);

// z_out (+)= W LN(z_in) on pair views (bf16): a LayerNorm pass and one row GEMM
bool rows_pair_ln_linear_supported(int c_in, int c_out);
size_t rows_pair_ln_linear_ws_bytes(int64_t n_rows, int64_t n_cols, int c_in);
int rows_pair_ln_linear(const pf_pair_linear_params* p, pf_pair_view zi, pf_pair_view zo, int64_t n_rows,
                        int64_t n_cols, int c_in, int c_out, int acc, void* ws, size_t ws_bytes, cudaStream_t st);

// bin logits of a pair tile (pf_pair_head_fwd, bf16): one LayerNorm / transposed-sum pass and one
// row GEMM whose epilogue adds the bias and forms the softmax contact sum
bool rows_pair_head_supported(int c_z, int n_bins);
size_t rows_pair_head_ws_bytes(int64_t n_rows, int64_t n_cols, int c_z);
int rows_pair_head(const pf_pair_head_params* p, int mode, pf_pair_view z, pf_pair_view zt, int64_t n_rows,
                   int64_t n_cols, int c_z, int n_bins, pf_pair_view lo, int lo_f32, float* contact,
                   int64_t contact_rs, int64_t contact_cs, int contact_bins, void* ws, size_t ws_bytes,
                   cudaStream_t st);

}  // namespace tc
}  // namespace pf
