/*
 * pairformer_b200.h -- C ABI of the B200-native (sm_100a) Pairformer pair stack.
 *
 * Plain C: device pointers, sizes, element strides, dtype enums and a cudaStream_t passed
 * as void*. Every entry point returns a pf_status code; a human-readable message for the
 * last failure on the calling thread is available from pf_last_error_string(). No compute
 * entry point allocates or frees device memory (only the peer-window calls of the Fold-CP
 * exchange, whose purpose it is): the caller owns inputs, outputs and workspace
 * (size it with the matching *_workspace_size call). All work is enqueued on the stream
 * passed in; no entry point synchronises the host.
 *
 * Each entry point replaces one reference interface (OpenDDE 1.0.2, package `opendde`);
 * the replaced function is cited beside it. Pair tensors are addressed through
 * pf_pair_view so that the ending-node / incoming variants and the Fold-CP slabs are the
 * same kernels on transposed or offset views (no physical transposes).
 */
#ifndef PAIRFORMER_B200_H
#define PAIRFORMER_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PF_ABI_VERSION 1

#if defined(__GNUC__)
#define PF_API __attribute__((visibility("default")))
#else
#define PF_API
#endif

typedef enum {
  PF_OK = 0,
  PF_EINVAL_SHAPE = 1,   /* sizes / strides / alignment rejected by host-side validation */
  PF_EINVAL_DTYPE = 2,   /* unknown dtype enum */
  PF_EUNSUPPORTED = 3,   /* valid request that this build does not implement */
  PF_ECUDA = 4,          /* a CUDA runtime/driver call failed (message has the CUDA error) */
  PF_ENCCL = 5,          /* reserved for collective entry points */
  PF_ETIMEOUT = 6,       /* a bounded device-side wait gave up (status word set by a kernel) */
  PF_EINVAL_ARG = 7,     /* null pointer or out-of-range scalar argument */
  PF_EWORKSPACE = 8      /* workspace pointer null or smaller than *_workspace_size */
} pf_status;

typedef enum {
  PF_F32 = 0,   /* fp32 storage, fp32 arithmetic (SIMT FFMA; the tolerance-1e-4 mode)        */
  PF_BF16 = 1   /* bf16 storage, fp32 accumulation on tcgen05 tensor cores where shapes allow */
} pf_dtype;

/* A view of a pair tensor: element (r, s, ch) lives at ptr + r*row_stride + s*col_stride + ch
 * (strides in elements; the channel dim is contiguous). A transposed view swaps the strides. */
typedef struct {
  void* ptr;
  int64_t row_stride;
  int64_t col_stride;
} pf_pair_view;

/* A view of an fp32 pair mask: mask(r, s) = ptr[r*row_stride + s*col_stride]. */
typedef struct {
  const float* ptr;
  int64_t row_stride;
  int64_t col_stride;
} pf_mask_view;

/* ---- library ------------------------------------------------------------------------ */

PF_API int pf_abi_version(void);
PF_API const char* pf_last_error_string(void);
/* Options: PF_OPT_FORCE_SIMT=1 routes bf16 requests to the generic SIMT kernels (testing).
 * PF_OPT_SM_RESERVE=r (0..64, per calling thread; 0 = default): the persistent tensor-core kernels
 * this thread launches afterwards use r fewer CTAs than the device has SMs, and pf_copy_regions
 * launches at most 8 r CTAs, so that a band copy enqueued on another stream runs on the r free
 * SMs beside them (the Fold-CP overlapped band exchange). No reference counterpart. */
#define PF_OPT_FORCE_SIMT 1
#define PF_OPT_SM_RESERVE 2
PF_API int pf_set_option(int option, int64_t value);
/* Name of the kernel family the last call on this thread dispatched to ("tc" or "simt"). */
PF_API const char* pf_last_path(void);
/* Device status word of the current device: bit 0 = a bounded device-side wait (mbarrier
 * pipeline wait) gave up; the kernel then drained instead of hanging. Bit 1 = a bf16
 * triangle-attention logit exceeded the f16 range of the logit accumulator (the affected rows
 * are invalid). Bit 2 = a kernel's shared-memory layout did not fit the dynamic shared memory it
 * was given (it returned without writing its outputs). The word is sticky: while it is non-zero every later tensor-core kernel drains
 * at once and leaves its outputs unwritten, so callers must check it. Synchronises with the
 * device (it copies the word to the host); clear != 0 resets it. No reference counterpart
 * (the reference has no device-side waits). */
PF_API int pf_device_status(int* status_out, int clear);
/* Stream-ordered copy of the same word into dst (pinned host or device memory, 4 bytes) on
 * `stream`, without synchronising: a caller checks dst once the copy has completed (e.g. at its
 * next call), so a timed-out wait is reported without adding a device synchronisation to every
 * forward. No reference counterpart. */
PF_API int pf_device_status_async(unsigned int* dst, void* stream);
/* Measurement hooks (no reference counterpart; the reference times whole stages with
 * host wall clocks, opendde/distributed/foldcp/metrics.py:136-234):
 * pf_launch_count  -- number of kernels this library has launched in the process;
 * pf_profile_enable -- when on, every launch is bracketed by a CUDA event pair on its stream;
 * pf_profile_report -- resolves the pairs into JSON {"kernel": [launches, total_ms], ...}
 *                      (waits for the last recorded event) and clears them. */
PF_API long long pf_launch_count(void);
PF_API int pf_profile_enable(int on);
PF_API int pf_profile_report(char* buf, size_t len);
/* Self-test of the failure path of the bounded device-side waits (no reference counterpart):
 * one thread waits on an mbarrier that nothing arrives on, gives up after limit_ns
 * (1 ms .. 10 s), sets bit 0 of the device status word and returns; no fault, the context stays
 * usable. Read and clear the word with pf_device_status before the next library call (a set
 * word makes every other bounded wait give up at once). */
PF_API int pf_selftest_bounded_wait(int64_t limit_ns, void* stream);

/* ---- LayerNorm ------------------------------------------------------------------------
 * y[r, :] = (x[r, :] - mean) / sqrt(var + eps) * gamma + beta over the last dim c.
 * Replaces OpenFoldLayerNorm.forward (opendde/model/triangular/layers.py:255-269) and the
 * fused extension FusedLayerNorm (opendde/model/layer_norm/layer_norm.py:233-288), launched
 * on the caller's stream (the reference launches on the legacy default stream,
 * layer_norm_cuda_kernel.cu:271). gamma/beta may be NULL (no scale / no offset). */
PF_API int pf_layernorm_fwd(const void* x, void* y, const float* gamma, const float* beta,
                     int64_t rows, int32_t c, float eps, int32_t dtype, void* stream);

/* ---- Triangle multiplicative update -----------------------------------------------------
 * Replaces TriangleMultiplicativeUpdate.forward (opendde/model/triangular/triangular.py:458-567,
 * _combine_projections :112-139) and its Fold-CP adapter
 * distributed_triangle_multiplication_update (opendde/distributed/foldcp/real_pairformer.py:1226).
 *
 *   a(i,k) = ma(i,k) * sigmoid(W_ag LN_in(za(i,k))) * (W_ap LN_in(za(i,k)))      i<n_i, k<n_k
 *   b(j,k) = mb(j,k) * sigmoid(W_bg LN_in(zb(j,k))) * (W_bp LN_in(zb(j,k)))      j<n_j
 *   x(i,j) = LN_out( sum_k a(i,k) * b(j,k) )
 *   u(i,j) = (W_z x(i,j)) * sigmoid(W_g LN_in(zg(i,j)))
 *   zo(i,j) = (accumulate ? zo(i,j) : 0) + u(i,j)
 * Outgoing: za = zb = zg = z, ma = mb = mask. Incoming: za, zb, ma, mb are the transposed
 * views of z and the mask, zg = z. All weights are [out, in] row-major in `dtype`; LayerNorm
 * parameters are fp32. zo may alias za, zb and zg (each position of zg is read before the
 * same position of zo is written, and the projections finish before zo is touched). */
typedef struct {
  const float* ln_in_w;  const float* ln_in_b;    /* [c_z] */
  const void* w_ap; const void* w_ag;             /* [c_h, c_z] */
  const void* w_bp; const void* w_bg;             /* [c_h, c_z] */
  const float* ln_out_w; const float* ln_out_b;   /* [c_h] */
  const void* w_z;                                /* [c_z, c_h] */
  const void* w_g;                                /* [c_z, c_z] */
} pf_trimul_params;

PF_API int pf_trimul_workspace_size(int64_t n_i, int64_t n_j, int64_t n_k, int32_t c_z, int32_t c_h,
                             int32_t dtype, size_t* bytes);
PF_API int pf_trimul_fwd(const pf_trimul_params* w, pf_pair_view za, pf_pair_view zb,
                  pf_mask_view ma, pf_mask_view mb, pf_pair_view zg, pf_pair_view zo,
                  int64_t n_i, int64_t n_j, int64_t n_k, int32_t c_z, int32_t c_h,
                  int32_t accumulate, int32_t dtype, void* workspace, size_t workspace_bytes,
                  void* stream);

/* The same update in two stages, for callers that move the projections between them (the
 * Fold-CP ring of real_pairformer.py:1226-1404 exchanges a_local / b_local, :1308-1384):
 * pf_trimul_project: a(ch, r, s) and b(ch, r, s) of one pair view z (with mask m), r < n_rows,
 *   s < n_cols, stored channel-major at a_out[(ch*n_rows + r)*ld + s] (same for b_out) in the
 *   storage dtype (fp32 for PF_F32, bf16 for PF_BF16; bf16 needs 16-byte aligned outputs and
 *   ld a multiple of 8);
 * pf_trimul_combine: x(i, j) = LN_out(sum_{k<n_k} a(ch, i, k) b(ch, j, k)) from a [c_h][n_i][ld]
 *   and b [c_h][n_j][ld] in that layout, then zo (+)= (W_z x) * sigmoid(W_g LN_in(zg)). */
PF_API int pf_trimul_project_workspace_size(int64_t n_rows, int64_t n_cols, int32_t c_z, int32_t c_h,
                                            int32_t dtype, size_t* bytes);
PF_API int pf_trimul_project(const pf_trimul_params* w, pf_pair_view z, pf_mask_view m, int64_t n_rows,
                             int64_t n_cols, int32_t c_z, int32_t c_h, int32_t dtype, void* a_out, void* b_out,
                             int64_t ld, void* workspace, size_t workspace_bytes, void* stream);
PF_API int pf_trimul_combine_workspace_size(int64_t n_i, int64_t n_j, int64_t n_k, int32_t c_z, int32_t c_h,
                                            int32_t dtype, size_t* bytes);
PF_API int pf_trimul_combine(const pf_trimul_params* w, const void* a, const void* b, int64_t ld, int64_t n_i,
                             int64_t n_j, int64_t n_k, pf_pair_view zg, pf_pair_view zo, int32_t c_z,
                             int32_t c_h, int32_t accumulate, int32_t dtype, void* workspace,
                             size_t workspace_bytes, void* stream);

/* Allocation-free variant of pf_trimul_fwd (no counterpart in the reference). For callers
 * that cannot allocate device memory or pass a workspace (a plugin inside a runtime that owns
 * every allocation, a foreign-language binding that only holds its input/output pointers):
 * the scratch comes from a fixed array of PF_STATIC_SCRATCH_BYTES compiled into the library,
 * reserved on every GPU that loads it until the process exits (48 MiB: a square bf16 problem
 * up to n = 256 with c_z = c_h = 128). Larger requests return PF_EINVAL_SHAPE with a message
 * naming the limit. The first call on a device looks up the array's device address (make it
 * before any stream capture begins); no call allocates or frees memory. Calls share the
 * array: calls whose GPU work overlaps race and must be serialised by the caller. */
#define PF_STATIC_SCRATCH_BYTES (48u * 1024u * 1024u)
PF_API size_t pf_static_scratch_bytes(void);
PF_API int pf_trimul_fwd_static_scratch(const pf_trimul_params* w, pf_pair_view za, pf_pair_view zb,
                                        pf_mask_view ma, pf_mask_view mb, pf_pair_view zg,
                                        pf_pair_view zo, int64_t n_i, int64_t n_j, int64_t n_k,
                                        int32_t c_z, int32_t c_h, int32_t accumulate, int32_t dtype,
                                        void* stream);

/* ---- Triangle attention (starting node; ending node = transposed views) ------------------
 * Replaces TriangleAttention.forward (opendde/model/triangular/triangular.py:648-706) with
 * Attention._prep_qkv/_attention/_wrap_up (opendde/model/triangular/layers.py:302-424), and
 * the Fold-CP adapter distributed_triangle_attention_update (real_pairformer.py:2633).
 *
 * Rows i < n_rows of the slab zs attend over keys k < n_keys of the same row:
 *   x = LN(zs(i,k));  q,k,v,g from x;  bias(h,j,k) = W_b LN(z(j,k))
 *   logits(h,i,j,k) = q(i,j).k(i,k)/sqrt(d) + inf*(m(i,k)-1) + bias(h,j,k)
 *   o(i,j) = W_o[ sigmoid(W_g x(i,j)) * softmax_k(logits) v(i,k) ]
 * Queries are the slab columns j = q_col0 .. q_col0+n_q-1; the output goes to zo(i, j-q_col0).
 * Keys with index >= n_valid_keys do not exist (Fold-CP padding); n_valid_keys <= n_keys.
 * bias: NULL => computed from zs itself (requires q_col0==0 and n_q==n_keys==n_rows, the
 * single-device case); otherwise a buffer written by pf_triatt_bias for the query rows,
 * addressed bias + h*bias_head_stride + j*bias_row_stride + k.
 * ending node: pass transposed views of z and the mask. */
typedef struct {
  const float* ln_w; const float* ln_b;   /* [c]          layer_norm           */
  const void* w_bias;                     /* [H, c]       linear (triangle bias) */
  const void* w_q; const void* w_k; const void* w_v;  /* [H*d, c]  mha.linear_{q,k,v} */
  const void* w_g;                        /* [H*d, c]     mha.linear_g          */
  const void* w_o;                        /* [c, H*d]     mha.linear_o          */
} pf_triatt_params;

/* bias(h, r, s) for positions r < n_rows, s < n_cols of z, written to
 * bias + h*bias_head_stride + r*bias_row_stride + s. Format: fp32 natural units for PF_F32;
 * f16 (IEEE half) scaled by log2(e) for PF_BF16 (the tensor-core attention works in base 2). */
PF_API int pf_triatt_bias_workspace_size(int64_t n_rows, int64_t n_cols, int32_t c, int32_t heads,
                                  int32_t dtype, size_t* bytes);
PF_API int pf_triatt_bias(const pf_triatt_params* w, pf_pair_view z, int64_t n_rows, int64_t n_cols,
                   void* bias, int64_t bias_head_stride, int64_t bias_row_stride,
                   int32_t c, int32_t heads, int32_t dtype, void* workspace,
                   size_t workspace_bytes, void* stream);
PF_API int pf_triatt_workspace_size(int64_t n_rows, int64_t n_keys, int64_t n_q, int32_t c,
                             int32_t heads, int32_t head_dim, int32_t dtype, size_t* bytes);
PF_API int pf_triatt_fwd(const pf_triatt_params* w, pf_pair_view zs, pf_mask_view m,
                  const void* bias, int64_t bias_head_stride, int64_t bias_row_stride,
                  pf_pair_view zo, int64_t n_rows, int64_t n_keys, int64_t n_valid_keys,
                  int64_t q_col0, int64_t n_q, int32_t c, int32_t heads, int32_t head_dim,
                  float inf, int32_t accumulate, int32_t dtype,
                  void* workspace, size_t workspace_bytes, void* stream);

/* ---- Transition (LN -> SiLU(W_a y) * (W_b y) -> W_out) ------------------------------------
 * Replaces Transition.forward (opendde/model/modules/primitives.py:182-217) and the Fold-CP
 * distributed_pair_transition_update (real_pairformer.py:1405, local in inference).
 * x and out are [rows, c] with row strides x_stride/out_stride (elements); out may be x itself
 * (same pointer and stride: the in-place update) or disjoint from it, not partly overlapping.
 * out = (accumulate ? out : 0) + Transition(x). */
typedef struct {
  const float* ln_w; const float* ln_b;   /* [c]        layernorm1        */
  const void* w_a; const void* w_b;       /* [n*c, c]   linear_no_bias_a/b */
  const void* w_o;                        /* [c, n*c]   linear_no_bias     */
} pf_transition_params;

PF_API int pf_transition_workspace_size(int64_t rows, int32_t c, int32_t n_mult, int32_t dtype,
                                 size_t* bytes);
PF_API int pf_transition_fwd(const pf_transition_params* w, const void* x, int64_t x_stride,
                      void* out, int64_t out_stride, int64_t rows, int32_t c, int32_t n_mult,
                      int32_t accumulate, int32_t dtype, void* workspace,
                      size_t workspace_bytes, void* stream);

/* ---- AttentionPairBias, single representation (has_s = False) -----------------------------
 * Replaces AttentionPairBias.forward with standard_multihead_attention
 * (opendde/model/modules/transformer.py:550-671) and Attention (primitives.py:645-857),
 * and the Fold-CP distributed_attention_pair_bias_update (real_pairformer.py:1714).
 * pf_apb_pair_bias: bias(h, r, s) = W_z LN_z(z(r, s)) for r < n_rows, s < n_cols, written
 * to bias + h*head_stride + r*row_stride + s (fp32).
 * pf_apb_fwd: s_out = (accumulate ? s_out : 0) + APB(s_in, bias) with the full [H, n, n]
 * bias (bias == NULL => computed from z, which must then be given). */
typedef struct {
  const float* ln_a_w; const float* ln_a_b;   /* [c_s]   layernorm_a            */
  const void* w_q; const float* b_q;          /* [c_s, c_s], [c_s] attention.linear_q */
  const void* w_k; const void* w_v;           /* [c_s, c_s]                    */
  const void* w_g; const void* w_o;           /* [c_s, c_s]                    */
  const float* ln_z_w; const float* ln_z_b;   /* [c_z]   layernorm_z (b may be NULL) */
  const void* w_z;                            /* [H, c_z] linear_nobias_z     */
} pf_apb_params;

PF_API int pf_apb_pair_bias_workspace_size(int64_t n_rows, int64_t n_cols, int32_t c_z, int32_t heads,
                                    int32_t dtype, size_t* bytes);
PF_API int pf_apb_pair_bias(const pf_apb_params* w, pf_pair_view z, int64_t n_rows, int64_t n_cols,
                     float* bias, int64_t head_stride, int64_t row_stride,
                     int32_t c_z, int32_t heads, int32_t dtype, void* workspace,
                     size_t workspace_bytes, void* stream);
PF_API int pf_apb_workspace_size(int64_t n, int32_t c_s, int32_t c_z, int32_t heads, int32_t dtype,
                          size_t* bytes);
PF_API int pf_apb_fwd(const pf_apb_params* w, const void* s_in, void* s_out, pf_pair_view z,
               const float* bias, int64_t n, int32_t c_s, int32_t c_z, int32_t heads,
               int32_t accumulate, int32_t dtype, void* workspace, size_t workspace_bytes,
               void* stream);

/* pf_apb_rows_fwd: the query rows [q_row0, q_row0 + n_q) of pf_apb_fwd, as the Fold-CP single
 * bridge runs them on one rank (real_pairformer.py:1714-1810, _single_update_rank_range):
 * keys and values come from all n rows of s_in; s_out holds n_q rows (row r = query
 * q_row0 + r, row stride c_s); bias(h, r, k) = bias[h*head_stride + r*row_stride + k] (fp32)
 * for local query r and key k < n. s_out = (accumulate ? s_out : 0) + APB rows. */
PF_API int pf_apb_rows_workspace_size(int64_t n, int64_t n_q, int32_t c_s, int32_t heads, int32_t dtype,
                                      size_t* bytes);
PF_API int pf_apb_rows_fwd(const pf_apb_params* w, const void* s_in, void* s_out, const float* bias,
                           int64_t head_stride, int64_t row_stride, int64_t n, int64_t q_row0,
                           int64_t n_q, int32_t c_s, int32_t heads, int32_t accumulate, int32_t dtype,
                           void* workspace, size_t workspace_bytes, void* stream);

/* ---- OuterProductMean (Algorithm 10) ---------------------------------------------------------
 * Replaces OuterProductMean.forward (opendde/model/triangular/layers.py:497-627) and the Fold-CP
 * pair-tile update (opendde/model/modules/pairformer.py:979-1046). For i in
 * [row0, row0 + n_rows), j in [col0, col0 + n_cols):
 *   z_out(i - row0, j - col0) = (accumulate ? z_out : 0)
 *       + (W_out vec_{c,e}(sum_s a(s, i, c) b(s, j, e)) + b_out) / (sum_s mask(s, i) mask(s, j) + eps)
 * with a = linear_1(LN(m)) * mask, b = linear_2(LN(m)) * mask; m(s, i) = m.ptr + s*m.row_stride
 * + i*m.col_stride (n_seq x n_res positions, c_m contiguous channels), mask(s, i) the MSA mask
 * (ptr NULL = ones). z_out is an n_rows x n_cols view of c_z channels. bf16 runs the
 * projections, the outer product (K = n_seq) and W_out (K = c_hidden^2) on tcgen05 when
 * c_hidden = 32; fp32 (and other c_hidden) on the SIMT kernels. */
typedef struct {
  const float* ln_w; const float* ln_b;   /* [c_m]              layer_norm      */
  const void* w_1; const void* w_2;       /* [c_hidden, c_m]    linear_1, linear_2 (no bias) */
  const void* w_out;                      /* [c_z, c_hidden^2]  linear_out      */
  const float* b_out;                     /* [c_z]              linear_out.bias */
} pf_opm_params;

PF_API int pf_opm_workspace_size(int64_t n_seq, int64_t n_res, int64_t n_rows, int64_t n_cols, int32_t c_m,
                                 int32_t c_hidden, int32_t c_z, int32_t dtype, size_t* bytes);
PF_API int pf_opm_fwd(const pf_opm_params* w, pf_pair_view m, pf_mask_view mask, pf_pair_view z_out,
                      int64_t n_seq, int64_t n_res, int64_t row0, int64_t n_rows, int64_t col0, int64_t n_cols,
                      int32_t c_m, int32_t c_hidden, int32_t c_z, float eps, int32_t accumulate, int32_t dtype,
                      void* workspace, size_t workspace_bytes, void* stream);

/* ---- Trunk pair initialisation and recycling ------------------------------------------------
 * Replaces the trunk's pair input, opendde/model/opendde.py:812-835, and its Fold-CP local
 * construction (opendde/distributed/foldcp/trunk_init.py:90-178). For i in [row0, row0 + n_rows),
 * j in [col0, col0 + n_cols):
 *   z_out(i - row0, j - col0) = W_1 s(i) + W_2 s(j) + W_relp relp(i, j) + W_bond bond(i, j)
 * with relp(i, j) the one-hot relative-position features of RelativePositionEncoding
 * (opendde/model/modules/embedders.py:87-302; 4 r_max + 2 s_max + 7 of them) computed from the
 * per-token ids, so W_relp relp is a sum of four weight columns (no feature tensor is formed),
 * and bond(i, j) = token_bonds(i, j) (ptr NULL: no bonds). s_init rows are s_stride elements
 * apart in the storage dtype; the ids are int32 [n_token]. */
typedef struct {
  const void* w_zinit1; const void* w_zinit2;  /* [c_z, c_s] linear_no_bias_zinit1 / 2        */
  const void* w_relp;                          /* [c_z, 4 r_max + 2 s_max + 7]                 */
  const void* w_bond;                          /* [c_z, 1]    linear_no_bias_token_bond          */
} pf_trunk_init_params;
typedef struct {
  const int32_t* asym_id; const int32_t* residue_index; const int32_t* entity_id;
  const int32_t* token_index; const int32_t* sym_id;
} pf_token_ids;

PF_API int pf_trunk_init_workspace_size(int64_t n_rows, int64_t n_cols, int32_t c_s, int32_t c_z, int32_t r_max,
                                        int32_t s_max, int32_t dtype, size_t* bytes);
PF_API int pf_trunk_init_fwd(const pf_trunk_init_params* w, const void* s_init, int64_t s_stride, pf_token_ids ids,
                             pf_mask_view token_bonds, pf_pair_view z_out, int64_t n_token, int64_t row0,
                             int64_t n_rows, int64_t col0, int64_t n_cols, int32_t c_s, int32_t c_z, int32_t r_max,
                             int32_t s_max, int32_t dtype, void* workspace, size_t workspace_bytes, void* stream);

/* z_out (+)= W LN(z_in) over the positions of two pair views (c_in -> c_out channels): the
 * recycling update z = z_init + linear_no_bias_z_cycle(layernorm_z_cycle(z)) of opendde.py:835
 * with z_out holding z_init and accumulate = 1 (z_out must not alias z_in). bf16 on tcgen05. */
typedef struct {
  const float* ln_w; const float* ln_b;  /* [c_in] */
  const void* w;                         /* [c_out, c_in] */
} pf_pair_linear_params;

PF_API int pf_pair_ln_linear_workspace_size(int64_t n_rows, int64_t n_cols, int32_t c_in, int32_t c_out,
                                            int32_t dtype, size_t* bytes);
PF_API int pf_pair_ln_linear_fwd(const pf_pair_linear_params* w, pf_pair_view z_in, pf_pair_view z_out, int64_t n_rows,
                                 int64_t n_cols, int32_t c_in, int32_t c_out, int32_t accumulate, int32_t dtype,
                                 void* workspace, size_t workspace_bytes, void* stream);

/* ---- Pair heads and pair conditioning downstream of the stack ----------------------------
 * pf_pair_head_fwd: per-position bin logits of a pair tile (n_rows x n_cols positions of c_z
 * channels, n_bins outputs), in one of three forms:
 *   PF_HEAD_PLAIN    logits = W LN(z) + b               ConfidenceHead pae (confidence.py:599-601)
 *   PF_HEAD_SYM_IN   logits = W LN(z + z^T) + b         ConfidenceHead pde (confidence.py:602-606)
 *   PF_HEAD_SYM_OUT  logits = (W z + b) + (W z^T + b)   DistogramHead.forward (head.py:33-46)
 * zt is the view whose (r, s) element is z^T at the tile's position (r, s), i.e. z(col, row):
 * the transposed view of the plane on one GPU, or the reciprocal rectangle (viewed transposed)
 * under Fold-CP (distogram.py:22-50, foldcp/confidence.py:22-29); unused by PLAIN. ln_w / ln_b:
 * the LayerNorm's affine parameters (PLAIN, SYM_IN; NULL = 1 / 0), unused by SYM_OUT; b NULL =
 * no bias. logits is a pair view of n_bins (<= 256) channels stored as logits_dtype (PF_F32: the
 * confidence heads' fp32 outputs; or the stack dtype). contact (optional, fp32 at
 * contact + r*contact_rs + s*contact_cs) = the sum of softmax(logits) over the first contact_bins
 * bins (the bins whose top <= thres, foldcp/distogram.py:159-166). bf16 on tcgen05 (LayerNorm /
 * transposed-sum pass + row GEMM with the bias and the softmax in its epilogue); fp32 on the SIMT
 * kernels. */
enum { PF_HEAD_PLAIN = 0, PF_HEAD_SYM_IN = 1, PF_HEAD_SYM_OUT = 2 };
typedef struct {
  const float* ln_w; const float* ln_b;  /* [c_z] LayerNorm parameters, or NULL              */
  const void* w;                         /* [n_bins, c_z]                                    */
  const float* b;                        /* [n_bins] bias, or NULL                           */
} pf_pair_head_params;

PF_API int pf_pair_head_workspace_size(int64_t n_rows, int64_t n_cols, int32_t c_z, int32_t n_bins, int32_t dtype,
                                       size_t* bytes);
PF_API int pf_pair_head_fwd(const pf_pair_head_params* w, int32_t mode, pf_pair_view z, pf_pair_view zt,
                            int64_t n_rows, int64_t n_cols, int32_t c_z, int32_t n_bins, pf_pair_view logits,
                            int32_t logits_dtype, float* contact, int64_t contact_rs, int64_t contact_cs,
                            int32_t contact_bins, int32_t dtype, void* workspace, size_t workspace_bytes,
                            void* stream);

/* pf_confidence_pair_init_fwd: the ConfidenceHead's pair input on a tile, rows
 * [row0, row0 + n_rows) x cols [col0, col0 + n_cols) of n_token:
 *   z_out(i, j) = z_trunk(i, j) + W_s2 s_inputs(i) + W_s1 s_inputs(j)
 *                 + W_d one_hot(d_ij) + W_d0 d_ij,  d_ij = |x_i - x_j|,
 *   one_hot_b(d) = (d > lower_b) * (d < upper_b)
 * (confidence.py:289-296, 540-572; the Fold-CP local form foldcp/confidence.py:81-148 and
 * confidence.py:177-202). coords: fp32 [n_token][3] representative-atom positions; 1..64 distance
 * bins. z_out may alias z_trunk. */
typedef struct {
  const void* w_s1; const void* w_s2;    /* [c_z, c_s_inputs] linear_no_bias_s1 / s2         */
  const void* w_d;                       /* [c_z, n_dist_bins] linear_no_bias_d               */
  const void* w_d0;                      /* [c_z, 1] linear_no_bias_d_wo_onehot               */
  const float* lower_bins; const float* upper_bins;  /* [n_dist_bins]                         */
} pf_confidence_init_params;

PF_API int pf_confidence_pair_init_workspace_size(int64_t n_rows, int64_t n_cols, int32_t c_s_inputs, int32_t c_z,
                                                  int32_t n_dist_bins, int32_t dtype, size_t* bytes);
PF_API int pf_confidence_pair_init_fwd(const pf_confidence_init_params* w, const void* s_inputs, int64_t s_stride,
                                       const float* coords, pf_pair_view z_trunk, pf_pair_view z_out, int64_t n_token,
                                       int64_t row0, int64_t n_rows, int64_t col0, int64_t n_cols,
                                       int32_t c_s_inputs, int32_t c_z, int32_t n_dist_bins, int32_t dtype,
                                       void* workspace, size_t workspace_bytes, void* stream);

/* pf_diffusion_pair_cond_fwd: the pair half of DiffusionConditioning on a tile (prepare_cache and
 * _apply_pair_z_transitions, diffusion.py:828-847, 1019-1040; the Fold-CP local form
 * prepare_cache_foldcp_local, :906-1017):
 *   x    = c_z == c_zd ? z_trunk : W_zt LN_zt(z_trunk)        (layernorm_z_trunk has no offset)
 *   pair = W_z LN_z([x | relpe(i, j)])                         (relpe from the token ids, as in
 *                                                               pf_trunk_init_fwd; no offset)
 *   pair += transition_z1(pair); pair += transition_z2(pair)   (n = 2)
 * z_out: the tile of c_zd channels (16-byte aligned positions); it may alias z_trunk when
 * c_z == c_zd (z_trunk is consumed before z_out is written). */
typedef struct {
  const float* ln_zt_w;                  /* [c_z]  layernorm_z_trunk.weight (c_z != c_zd)     */
  const void* w_zt;                      /* [c_zd, c_z] linear_no_bias_z_trunk (c_z != c_zd)  */
  const void* w_relp;                    /* [c_zd, 4 r_max + 2 s_max + 7] relpe.linear_no_bias */
  const float* ln_z_w;                   /* [2 c_zd] layernorm_z.weight                        */
  const void* w_z;                       /* [c_zd, 2 c_zd] linear_no_bias_z                    */
  pf_transition_params t1, t2;           /* transition_z1 / transition_z2                      */
} pf_diffusion_pair_params;

PF_API int pf_diffusion_pair_cond_workspace_size(int64_t n_rows, int64_t n_cols, int32_t c_z, int32_t c_zd,
                                                 int32_t r_max, int32_t s_max, int32_t dtype, size_t* bytes);
PF_API int pf_diffusion_pair_cond_fwd(const pf_diffusion_pair_params* w, pf_pair_view z_trunk, pf_token_ids ids,
                                      pf_pair_view z_out, int64_t n_token, int64_t row0, int64_t n_rows, int64_t col0,
                                      int64_t n_cols, int32_t c_z, int32_t c_zd, int32_t r_max, int32_t s_max,
                                      int32_t dtype, void* workspace, size_t workspace_bytes, void* stream);

/* ---- Fold-CP band exchange through peer memory ------------------------------------------
 * Replace the reference's ring / transpose band exchanges over NCCL send/receive
 * (opendde/distributed/foldcp/comm.py:26-184, used by real_pairformer.py:1226-1404 and
 * :2633-2756) for ranks on one NVLink node: each rank publishes its pair tile into a window
 * exported with a CUDA IPC handle; the peers open the handle once and, after a stream-ordered
 * barrier, copy the rectangles their bands need straight out of the window.
 *
 * pf_peer_window_alloc is the one entry point that allocates device memory (cudaMalloc of
 * `bytes` on the current device); it writes the window's pointer and its IPC handle
 * (pf_peer_handle_bytes() bytes) for the peers. pf_peer_window_open maps a peer's handle into
 * this process (not valid on the process that allocated it); pf_peer_window_close unmaps it;
 * pf_peer_window_free releases an own window once no peer reads it any more. */
PF_API size_t pf_peer_handle_bytes(void);
PF_API int pf_peer_window_alloc(size_t bytes, void** ptr_out, void* handle_out);
PF_API int pf_peer_window_free(void* ptr);
PF_API int pf_peer_window_open(const void* handle, void** ptr_out);
PF_API int pf_peer_window_close(void* ptr);

/* One 3D byte box: planes x rows x row_bytes from src (row pitch src_pitch, plane pitch
 * src_plane_pitch bytes) to dst (dst_pitch, dst_plane_pitch). src may be a peer's window. A
 * band of a pair tile is one plane; a band of a channel-major projection has one plane per
 * channel. */
typedef struct {
  const void* src;
  void* dst;
  int64_t planes;
  int64_t rows;
  int64_t row_bytes;
  int64_t src_pitch;
  int64_t dst_pitch;
  int64_t src_plane_pitch;
  int64_t dst_plane_pitch;
} pf_copy_region;
#define PF_MAX_COPY_REGIONS 32
/* Copies up to PF_MAX_COPY_REGIONS boxes with one kernel launch on `stream` (16-byte vectors
 * when every pointer, pitch and row length allows). The caller orders it after the peers'
 * writes (the barrier) and before anything overwrites the sources. */
PF_API int pf_copy_regions(const pf_copy_region* regions, int32_t n_regions, void* stream);
/* The same copies by the GPU's copy engines (any number of regions; one 2-D or 3-D copy per
 * region, no SMs), so a band copied on a side stream overlaps kernels on another stream. */
PF_API int pf_copy_regions_dma(const pf_copy_region* regions, int32_t n_regions, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PAIRFORMER_B200_H */
