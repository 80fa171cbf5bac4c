// pf_relp.cuh -- the relative-position feature of a token pair as the indices of its one-hot
// entries (RelativePositionEncoding, opendde/model/modules/embedders.py:124-179, 226-290), shared
// by the trunk's pair input (pf_trunk.cu) and the diffusion pair conditioning (pf_heads.cu), with
// the 4-channel vector accesses of their one-warp-per-position kernels.
//
// The feature vector is [residue offset (2R + 2) | token offset (2R + 2) | same entity (1) |
// symmetry-copy offset (2S + 2)], R = r_max, S = s_max: three one-hots and one bit. Its product
// with a weight matrix is therefore the sum of three columns, plus the same-entity column when the
// bit is set; the [N, N, 4R + 2S + 7] feature tensor is never formed.
#pragma once
#include <stdint.h>

#include "../../include/pairformer_b200.h"
#include "pf_common.cuh"

namespace pf {

struct RelpIndex {
  int res, tok, ent, chn;  // feature columns; ent is used only when same_ent
  bool same_ent;
};

__host__ __device__ __forceinline__ int relp_n_feat(int r_max, int s_max) { return 4 * r_max + 2 * s_max + 7; }

__device__ __forceinline__ int relp_clip(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

// Residue offset clipped to [0, 2R] within a chain (2R + 1 across chains); token offset clipped
// the same way within one residue of one chain (2R + 1 otherwise); symmetry-copy offset clipped to
// [0, 2S] within an entity (2S + 1 across entities).
__device__ __forceinline__ RelpIndex relp_index(const pf_token_ids& ids, int64_t i, int64_t j, int R, int S) {
  const bool same_chain = ids.asym_id[i] == ids.asym_id[j];
  const int res_i = ids.residue_index[i], res_j = ids.residue_index[j];
  const bool same_res = res_i == res_j;
  RelpIndex x;
  x.same_ent = ids.entity_id[i] == ids.entity_id[j];
  x.res = same_chain ? relp_clip(res_i - res_j + R, 0, 2 * R) : 2 * R + 1;
  x.tok = 2 * R + 2 +
          ((same_chain && same_res) ? relp_clip(ids.token_index[i] - ids.token_index[j] + R, 0, 2 * R) : 2 * R + 1);
  x.ent = 4 * R + 4;
  x.chn = 4 * R + 5 + (x.same_ent ? relp_clip(ids.sym_id[i] - ids.sym_id[j] + S, 0, 2 * S) : 2 * S + 1);
  return x;
}

// Four consecutive channels as fp32, from / to the storage type (8-byte bf16 or 16-byte fp32
// accesses: with one warp per position, a warp moves 128 channels in one coalesced access).
template <class T>
__device__ __forceinline__ void load4(const T* p, float* f);
template <>
__device__ __forceinline__ void load4<float>(const float* p, float* f) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  f[0] = a.x, f[1] = a.y, f[2] = a.z, f[3] = a.w;
}
template <>
__device__ __forceinline__ void load4<__nv_bfloat16>(const __nv_bfloat16* p, float* f) {
  const uint2 q = *reinterpret_cast<const uint2*>(p);
  f[0] = __uint_as_float(q.x << 16), f[1] = __uint_as_float(q.x & 0xffff0000u);
  f[2] = __uint_as_float(q.y << 16), f[3] = __uint_as_float(q.y & 0xffff0000u);
}
template <class T>
__device__ __forceinline__ void store4(T* p, const float* f);
template <>
__device__ __forceinline__ void store4<float>(float* p, const float* f) {
  *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
}
template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* p, const float* f) {
  const __nv_bfloat162 a = __floats2bfloat162_rn(f[0], f[1]), b = __floats2bfloat162_rn(f[2], f[3]);
  *reinterpret_cast<uint2*>(p) =
      make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
}

__device__ __forceinline__ float4 ldf4(const float* p) { return *reinterpret_cast<const float4*>(p); }

// wt[f*c + ch] = w[ch*n_feat + f] (fp32): a [c, n_feat] weight as rows of contiguous channels
template <class T>
__global__ void k_cols_to_rows(const T* __restrict__ w, int n_feat, int c, float* __restrict__ wt) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n_feat * c) return;
  const int f = idx / c, ch = idx - f * c;
  wt[idx] = to_f(w[(int64_t)ch * n_feat + f]);
}

}  // namespace pf
