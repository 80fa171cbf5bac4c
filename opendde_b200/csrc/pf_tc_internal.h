// pf_tc_internal.h -- pieces of the c = 128 tensor-core kernels that the general-width path
// (pf_tc_rows.cu) reuses: the per-channel contraction of the triangle update and the
// mask preparation + core of triangle attention. Both are width-independent: the contraction
// is batched over channels, and the attention core works on one (row pair, head) of d = 32 at
// a time.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/pairformer_b200.h"

namespace pf {
namespace tc {

// x(ch, i, j) = sum_k a(ch, i, k) b(ch, j, k) for ch < channels: a, b channel-major bf16 with
// row pitches lda / ldb (elements, multiples of 8) and plane pitches n_i * lda / n_j * ldb;
// x channel-major with row pitch ld_j, plane pitch n_i * ld_j. tcgen05, fp32 accumulate.
int trimul_contract(const __nv_bfloat16* a, int64_t lda, const __nv_bfloat16* b, int64_t ldb, int64_t n_i,
                    int64_t n_j, int64_t n_k, int channels, __nv_bfloat16* x, int64_t ld_j, unsigned int* status,
                    cudaStream_t st);

// Buffers of the triangle-attention core (d = 32, `heads` heads):
//   q  [(i*heads + h)*n_q + j][32]      f16, pre-scaled by log2(e)/sqrt(32)
//   k  [(i*heads + h)*ld_keys + key][32] f16
//   vt [(i*heads + h)*32 + d][ld_keys]  f16
//   bias(h, j, key) at bias + h*b_hs + j*b_rs + key, f16 in log2 units
//   o  [(i*n_q + j)][heads*32]          bf16 (written)
//   mb, flags, rowflags: per-row key bias and tile flags (written by triatt_masks)
struct CoreIO {
  const __half* q;
  const __half* k;
  const __half* vt;
  const void* bias;
  int64_t b_hs, b_rs;
  __nv_bfloat16* o;
  __half* mb;
  uint8_t* flags;
  uint8_t* rowflags;
  int64_t ld_keys, ld_mb, n_tiles_k;
};

int triatt_masks(pf_mask_view m, int64_t n_rows, int64_t n_keys, int64_t n_valid, float inf, const CoreIO& io,
                 cudaStream_t st);
int triatt_core(const CoreIO& io, int64_t n_rows, int64_t n_keys, int64_t n_valid, int64_t n_q, int heads,
                unsigned int* status, cudaStream_t st);

}  // namespace tc
}  // namespace pf
