// pf_trunk.cu -- the trunk's pair input (opendde/model/opendde.py:812-835) and its Fold-CP
// local construction (opendde/distributed/foldcp/trunk_init.py:90-178), for any tile of the
// pair plane, in both storage dtypes.
//
//   1. the per-token projections W_1 s(i) (tile rows) and W_2 s(j) (tile columns), fp32, by the
//      SIMT GEMM (n_token x c_s x c_z: small next to the plane);
//   2. k_relp_weights: W_relp^T and W_bond as fp32 rows [feature][c_z] (contiguous channels);
//   3. k_trunk_init: one thread per position (i, j): the relative-position feature indices from
//      the five per-token ids (the one-hot rules of RelativePositionEncoding,
//      opendde/model/modules/embedders.py:124-179), then per 8 channels
//      (W_1 s(i) + W_2 s(j)) + (sum of the four selected W_relp columns) + bond(i, j) W_bond,
//      written as 16-byte (bf16) or 32-byte (fp32) stores. HBM-bound on the tile it writes.
// The recycling update z_init + W LN(z) is pf_pair_ln_linear_fwd (pf_api.cu).

#include "pf_common.cuh"
#include "pf_prof.h"
#include "pf_simt.h"

namespace pf {
namespace trunk {

namespace {

// wt[f*c_z + c] = w_relp[c*n_feat + f]; wt[n_feat*c_z + c] = w_bond[c]  (fp32)
template <class T>
__global__ void k_relp_weights(const T* __restrict__ w_relp, const T* __restrict__ w_bond, int n_feat, int c_z,
                               float* __restrict__ wt) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (n_feat + 1) * c_z) return;
  const int f = idx / c_z, c = idx - f * c_z;
  wt[idx] = f < n_feat ? to_f(w_relp[(int64_t)c * n_feat + f]) : to_f(w_bond[c]);
}

struct TrunkArgs {
  const float* zr;  // [n_rows][c_z]  W_1 s(row0 + i)
  const float* zc;  // [n_cols][c_z]  W_2 s(col0 + j)
  const float* wt;  // [n_feat + 1][c_z]
  pf_token_ids ids;
  pf_mask_view bonds;
  int64_t row0, n_rows, col0, n_cols;
  int c_z, r_max, s_max;
  int64_t zo_rs, zo_cs;
};

__device__ __forceinline__ int clip_i(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

template <class T>
__global__ void __launch_bounds__(128) k_trunk_init(TrunkArgs a, T* __restrict__ zo) {
  const int64_t li = blockIdx.y;
  const int64_t lj = (int64_t)blockIdx.x * 128 + threadIdx.x;
  if (lj >= a.n_cols) return;
  const int64_t i = a.row0 + li, j = a.col0 + lj;
  const int asym_i = a.ids.asym_id[i], asym_j = a.ids.asym_id[j];
  const int res_i = a.ids.residue_index[i], res_j = a.ids.residue_index[j];
  const int ent_i = a.ids.entity_id[i], ent_j = a.ids.entity_id[j];
  const int tok_i = a.ids.token_index[i], tok_j = a.ids.token_index[j];
  const int sym_i = a.ids.sym_id[i], sym_j = a.ids.sym_id[j];
  const int R = a.r_max, S = a.s_max;
  const bool same_chain = asym_i == asym_j, same_res = res_i == res_j, same_ent = ent_i == ent_j;
  // feature indices: [residue offset (2R + 2) | token offset (2R + 2) | same entity | chain offset (2S + 2)]
  const int f_res = same_chain ? clip_i(res_i - res_j + R, 0, 2 * R) : 2 * R + 1;
  const int f_tok = 2 * R + 2 + ((same_chain && same_res) ? clip_i(tok_i - tok_j + R, 0, 2 * R) : 2 * R + 1);
  const int f_ent = 4 * R + 4;
  const int f_chn = 4 * R + 5 + (same_ent ? clip_i(sym_i - sym_j + S, 0, 2 * S) : 2 * S + 1);
  const int n_feat = 4 * R + 2 * S + 7;
  const float bond = a.bonds.ptr ? a.bonds.ptr[i * a.bonds.row_stride + j * a.bonds.col_stride] : 0.f;
  const int C = a.c_z;
  const float* zr = a.zr + li * C;
  const float* zc = a.zc + lj * C;
  const float* w_res = a.wt + (int64_t)f_res * C;
  const float* w_tok = a.wt + (int64_t)f_tok * C;
  const float* w_ent = a.wt + (int64_t)f_ent * C;
  const float* w_chn = a.wt + (int64_t)f_chn * C;
  const float* w_bond = a.wt + (int64_t)n_feat * C;
  T* out = zo + li * a.zo_rs + lj * a.zo_cs;
  for (int c = 0; c < C; c += 8) {
    float y[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float relp = w_res[c + e] + w_tok[c + e] + w_chn[c + e];
      if (same_ent) relp += w_ent[c + e];
      y[e] = (zr[c + e] + zc[c + e]) + relp + bond * w_bond[c + e];
    }
    if constexpr (sizeof(T) == 2) {
      uint4 q;
      uint32_t* qw = &q.x;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(y[2 * e], y[2 * e + 1]);
        qw[e] = *reinterpret_cast<const uint32_t*>(&h);
      }
      *reinterpret_cast<uint4*>(out + c) = q;
    } else {
      reinterpret_cast<float4*>(out + c)[0] = make_float4(y[0], y[1], y[2], y[3]);
      reinterpret_cast<float4*>(out + c)[1] = make_float4(y[4], y[5], y[6], y[7]);
    }
  }
}

}  // namespace

size_t init_ws_bytes(int64_t n_rows, int64_t n_cols, int c_z, int r_max, int s_max) {
  Arena ar(nullptr, 0);
  ar.take<float>((size_t)n_rows * c_z);
  ar.take<float>((size_t)n_cols * c_z);
  ar.take<float>((size_t)(4 * r_max + 2 * s_max + 8) * c_z);
  return ar.used;
}

template <class T>
static int init_t(const pf_trunk_init_params* p, const T* s, int64_t s_stride, pf_token_ids ids, pf_mask_view bonds,
                  pf_pair_view zo, int64_t row0, int64_t n_rows, int64_t col0, int64_t n_cols, int c_s, int c_z,
                  int r_max, int s_max, Arena& ar, cudaStream_t st) {
  float* zr = ar.take<float>((size_t)n_rows * c_z);
  float* zc = ar.take<float>((size_t)n_cols * c_z);
  const int n_feat = 4 * r_max + 2 * s_max + 7;
  float* wt = ar.take<float>((size_t)(n_feat + 1) * c_z);
  if (!ar.ok()) return fail(PF_EWORKSPACE, "trunk init workspace too small");
  PF_TRY(simt::gemm_rows<T>(s + row0 * s_stride, s_stride, (const T*)p->w_zinit1, zr, n_rows, c_z, c_s, st));
  PF_TRY(simt::gemm_rows<T>(s + col0 * s_stride, s_stride, (const T*)p->w_zinit2, zc, n_cols, c_z, c_s, st));
  {
    PF_LAUNCH_SCOPE(st, "k_relp_weights");
    const int n = (n_feat + 1) * c_z;
    k_relp_weights<T><<<(n + 255) / 256, 256, 0, st>>>((const T*)p->w_relp, (const T*)p->w_bond, n_feat, c_z, wt);
  }
  PF_CHECK_LAUNCH();
  TrunkArgs a{zr, zc, wt, ids, bonds, row0, n_rows, col0, n_cols, c_z, r_max, s_max, zo.row_stride, zo.col_stride};
  dim3 grid((unsigned)((n_cols + 127) / 128), (unsigned)n_rows);
  {
    PF_LAUNCH_SCOPE_WORK(st, "k_trunk_init", (double)n_rows * n_cols * c_z * sizeof(T), 'b');
    k_trunk_init<T><<<grid, 128, 0, st>>>(a, (T*)zo.ptr);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

int init(const pf_trunk_init_params* p, const void* s, int64_t s_stride, pf_token_ids ids, pf_mask_view bonds,
         pf_pair_view zo, int64_t row0, int64_t n_rows, int64_t col0, int64_t n_cols, int c_s, int c_z, int r_max,
         int s_max, int dtype, void* ws, size_t ws_bytes, cudaStream_t st) {
  Arena ar(ws, ws_bytes);
  if (dtype == PF_F32)
    return init_t<float>(p, (const float*)s, s_stride, ids, bonds, zo, row0, n_rows, col0, n_cols, c_s, c_z, r_max,
                         s_max, ar, st);
  return init_t<__nv_bfloat16>(p, (const __nv_bfloat16*)s, s_stride, ids, bonds, zo, row0, n_rows, col0, n_cols, c_s,
                               c_z, r_max, s_max, ar, st);
}

}  // namespace trunk
}  // namespace pf
