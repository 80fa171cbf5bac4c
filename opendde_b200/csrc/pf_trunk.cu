// pf_trunk.cu -- the trunk's pair input (opendde/model/opendde.py:812-835) and its Fold-CP
// local construction (opendde/distributed/foldcp/trunk_init.py:90-178), for any tile of the
// pair plane, in both storage dtypes.
//
//   1. the per-token projections W_1 s(i) (tile rows) and W_2 s(j) (tile columns), fp32, by the
//      SIMT GEMM (n_token x c_s x c_z: small next to the plane);
//   2. k_cols_to_rows: W_relp^T and W_bond as fp32 rows [feature][c_z] (contiguous channels);
//   3. k_trunk_init: one warp per position (i, j): the relative-position feature indices from
//      the five per-token ids (relp_index, pf_relp.cuh), then per 4 channels of each lane
//      (W_1 s(i) + W_2 s(j)) + (sum of the four selected W_relp columns) + bond(i, j) W_bond,
//      each lane storing 8 (bf16) or 16 (fp32) bytes, a warp 128 channels at once (coalesced;
//      one thread per position made every weight-row read touch 32 lines per warp). HBM-bound on
//      the tile it writes.
// The recycling update z_init + W LN(z) is pf_pair_ln_linear_fwd (pf_api.cu).

#include "pf_common.cuh"
#include "pf_prof.h"
#include "pf_relp.cuh"
#include "pf_simt.h"

namespace pf {
namespace trunk {

namespace {

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

// One warp per position (i, j); lane l owns channels 4l + 128k.
template <class T>
__global__ void __launch_bounds__(256) k_trunk_init(TrunkArgs a, T* __restrict__ zo) {
  const int lane = threadIdx.x & 31;
  const int64_t pos = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (pos >= a.n_rows * a.n_cols) return;
  const int64_t li = pos / a.n_cols, lj = pos - li * a.n_cols;
  const int64_t i = a.row0 + li, j = a.col0 + lj;
  const RelpIndex f = relp_index(a.ids, i, j, a.r_max, a.s_max);
  const int n_feat = relp_n_feat(a.r_max, a.s_max);
  const float bond = a.bonds.ptr ? a.bonds.ptr[i * a.bonds.row_stride + j * a.bonds.col_stride] : 0.f;
  const int C = a.c_z;
  const float* zr = a.zr + li * C;
  const float* zc = a.zc + lj * C;
  const float* w_res = a.wt + (int64_t)f.res * C;
  const float* w_tok = a.wt + (int64_t)f.tok * C;
  const float* w_ent = a.wt + (int64_t)f.ent * C;
  const float* w_chn = a.wt + (int64_t)f.chn * C;
  const float* w_bond = a.wt + (int64_t)n_feat * C;
  T* out = zo + li * a.zo_rs + lj * a.zo_cs;
  for (int c = 4 * lane; c < C; c += 128) {
    const float4 r4 = ldf4(zr + c), c4 = ldf4(zc + c), a4 = ldf4(w_res + c), t4 = ldf4(w_tok + c),
                 h4 = ldf4(w_chn + c), b4 = ldf4(w_bond + c);
    float4 e4 = make_float4(0.f, 0.f, 0.f, 0.f);
    if (f.same_ent) e4 = ldf4(w_ent + c);
    const float y[4] = {(r4.x + c4.x) + (a4.x + t4.x + h4.x + e4.x) + bond * b4.x,
                        (r4.y + c4.y) + (a4.y + t4.y + h4.y + e4.y) + bond * b4.y,
                        (r4.z + c4.z) + (a4.z + t4.z + h4.z + e4.z) + bond * b4.z,
                        (r4.w + c4.w) + (a4.w + t4.w + h4.w + e4.w) + bond * b4.w};
    store4<T>(out + c, y);
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
    // W_relp^T rows, then the bond column as row n_feat
    PF_LAUNCH_SCOPE(st, "k_cols_to_rows");
    k_cols_to_rows<T><<<(n_feat * c_z + 255) / 256, 256, 0, st>>>((const T*)p->w_relp, n_feat, c_z, wt);
    k_cols_to_rows<T><<<(c_z + 255) / 256, 256, 0, st>>>((const T*)p->w_bond, 1, c_z, wt + (size_t)n_feat * c_z);
  }
  PF_CHECK_LAUNCH();
  TrunkArgs a{zr, zc, wt, ids, bonds, row0, n_rows, col0, n_cols, c_z, r_max, s_max, zo.row_stride, zo.col_stride};
  const int64_t blocks = (n_rows * n_cols + 7) / 8;
  if (blocks > 0x7fffffffll) return fail(PF_EUNSUPPORTED, "trunk init: tile too large");
  {
    PF_LAUNCH_SCOPE_WORK(st, "k_trunk_init", (double)n_rows * n_cols * c_z * sizeof(T), 'b');
    k_trunk_init<T><<<(unsigned)blocks, 256, 0, st>>>(a, (T*)zo.ptr);
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
