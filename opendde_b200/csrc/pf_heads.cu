// pf_heads.cu -- pair work downstream of the stack, on any tile of the pair plane:
//
//   confidence pair input (opendde/model/modules/confidence.py:289-296, 540-572):
//     1. W_s2 s_inputs(i) for the tile rows and W_s1 s_inputs(j) for its columns (SIMT GEMM, fp32);
//     2. k_cols_to_rows: W_d^T and W_d0 as fp32 rows [bin][c_z];
//     3. k_conf_init: one warp per position: d = |x_i - x_j|, its distance bins (the strict
//        lower < d < upper test of one_hot, opendde/model/utils.py:212-228), then per 4 channels
//        of each lane z_trunk + row + column + W_d[bin] + d W_d0 in fp32, one rounding to the
//        storage type, coalesced 128-channel accesses per warp. HBM-bound: 2 x c_z x sizeof(T)
//        bytes per position.
//
//   diffusion pair conditioning (DiffusionConditioning.prepare_cache + _apply_pair_z_transitions,
//   opendde/model/modules/diffusion.py:828-847, 1019-1040):
//     1. c_z != c_zd: x = W_zt LN(z_trunk) into the first half of a [P][2 c_zd] buffer
//        (pf_pair_ln_linear_fwd: LayerNorm pass + tcgen05 row GEMM in bf16);
//     2. k_relp_cat: the relative-position term (four weight columns, relp_index) into the second
//        half, and z_trunk into the first when it is not compressed;
//     3. pair = W_z LN([x | relp]) (pf_pair_ln_linear_fwd), then two residual transitions
//        (pf_transition_fwd, n = 2) in place; a final copy when the output view is not dense.
//
// The bin logits of the distogram and confidence heads are pf_pair_head_fwd (pf_tc_rows.cu for
// bf16, pf_simt.cu for fp32).

#include "pf_common.cuh"
#include "pf_prof.h"
#include "pf_relp.cuh"
#include "pf_simt.h"

namespace pf {
namespace heads {

namespace {

inline unsigned nblk(int64_t n, int t) { return (unsigned)((n + t - 1) / t); }

struct ConfArgs {
  const float* zr;      // [n_rows][c_z]  W_s2 s_inputs(row0 + i)
  const float* zc;      // [n_cols][c_z]  W_s1 s_inputs(col0 + j)
  const float* wt;      // [n_bins + 1][c_z]  W_d^T, then W_d0
  const float* coords;  // [n_token][3]
  const float* lower;
  const float* upper;
  int n_bins;           // <= 64
  int64_t row0, n_rows, col0, n_cols;
  int c_z;
  int64_t zi_rs, zi_cs, zo_rs, zo_cs;
};

// One warp per position (i, j); lane l owns channels 4l + 128k. The distance bins are tested 32 at
// a time (lane b tests bin b0 + b) and the one-hot's set bits gathered by ballot, so bins that
// overlapped would add every matching column, as the reference's one_hot would.
template <class T>
__global__ void __launch_bounds__(256) k_conf_init(ConfArgs a, const T* __restrict__ zi, T* __restrict__ zo) {
  const int lane = threadIdx.x & 31;
  const int64_t pos = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (pos >= a.n_rows * a.n_cols) return;
  const int64_t li = pos / a.n_cols, lj = pos - li * a.n_cols;
  const int64_t i = a.row0 + li, j = a.col0 + lj;
  // the direct form of the distance: differences, squares, sum in coordinate order, sqrt
  const float dx = a.coords[3 * i] - a.coords[3 * j];
  const float dy = a.coords[3 * i + 1] - a.coords[3 * j + 1];
  const float dz = a.coords[3 * i + 2] - a.coords[3 * j + 2];
  const float d = sqrtf(__fadd_rn(__fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy)), __fmul_rn(dz, dz)));
  unsigned hits[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int b = 32 * h + lane;
    const bool in = b < a.n_bins && d > a.lower[b] && d < a.upper[b];
    hits[h] = __ballot_sync(0xffffffffu, in);
  }
  const int C = a.c_z;
  const float* zr = a.zr + li * C;
  const float* zc = a.zc + lj * C;
  const float* w0 = a.wt + (int64_t)a.n_bins * C;
  const T* src = zi + li * a.zi_rs + lj * a.zi_cs;
  T* out = zo + li * a.zo_rs + lj * a.zo_cs;
  for (int c = 4 * lane; c < C; c += 128) {
    float y[4];
    load4<T>(src + c, y);
    const float4 r4 = ldf4(zr + c), c4 = ldf4(zc + c), d4 = ldf4(w0 + c);
    float4 b4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      for (unsigned m = hits[h]; m; m &= m - 1) {
        const float4 w = ldf4(a.wt + (int64_t)(32 * h + __ffs(m) - 1) * C + c);
        b4.x += w.x, b4.y += w.y, b4.z += w.z, b4.w += w.w;
      }
    }
    y[0] = fmaf(d, d4.x, ((r4.x + c4.x) + y[0]) + b4.x);
    y[1] = fmaf(d, d4.y, ((r4.y + c4.y) + y[1]) + b4.y);
    y[2] = fmaf(d, d4.z, ((r4.z + c4.z) + y[2]) + b4.z);
    y[3] = fmaf(d, d4.w, ((r4.w + c4.w) + y[3]) + b4.w);
    store4<T>(out + c, y);
  }
}

// cat[p*ld + c_zd + ch] = relpe(i, j)[ch]; with x: cat[p*ld + ch] = x(i, j)[ch] (ld = 2 c_zd). One
// warp per position, lane l owning channels 4l + 128k.
template <class T>
__global__ void __launch_bounds__(256) k_relp_cat(const float* __restrict__ wt, pf_token_ids ids, int64_t row0,
                                                  int64_t n_rows, int64_t col0, int64_t n_cols, int c_zd, int r_max,
                                                  int s_max, const T* __restrict__ x, int64_t x_rs, int64_t x_cs,
                                                  T* __restrict__ cat) {
  const int lane = threadIdx.x & 31;
  const int64_t pos = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (pos >= n_rows * n_cols) return;
  const int64_t li = pos / n_cols, lj = pos - li * n_cols;
  const RelpIndex f = relp_index(ids, row0 + li, col0 + lj, r_max, s_max);
  const int C = c_zd;
  const float* w_res = wt + (int64_t)f.res * C;
  const float* w_tok = wt + (int64_t)f.tok * C;
  const float* w_ent = wt + (int64_t)f.ent * C;
  const float* w_chn = wt + (int64_t)f.chn * C;
  T* dst = cat + pos * (2 * C);
  const T* src = x ? x + li * x_rs + lj * x_cs : nullptr;
  for (int c = 4 * lane; c < C; c += 128) {
    const float4 a4 = ldf4(w_res + c), t4 = ldf4(w_tok + c), h4 = ldf4(w_chn + c);
    float4 e4 = make_float4(0.f, 0.f, 0.f, 0.f);
    if (f.same_ent) e4 = ldf4(w_ent + c);
    const float y[4] = {a4.x + t4.x + h4.x + e4.x, a4.y + t4.y + h4.y + e4.y, a4.z + t4.z + h4.z + e4.z,
                        a4.w + t4.w + h4.w + e4.w};
    store4<T>(dst + C + c, y);
    if (src) {
      float v[4];
      load4<T>(src + c, v);
      store4<T>(dst + c, v);
    }
  }
}

// dst(r, s, :) = src[(r*n_cols + s)*c + :], one warp per position
template <class T>
__global__ void __launch_bounds__(256) k_to_view(const T* __restrict__ src, int64_t n_rows, int64_t n_cols, int c,
                                                 T* __restrict__ dst, int64_t rs, int64_t cs) {
  const int lane = threadIdx.x & 31;
  const int64_t pos = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (pos >= n_rows * n_cols) return;
  const int64_t r = pos / n_cols, s = pos - r * n_cols;
  for (int ch = 4 * lane; ch < c; ch += 128) {
    float f[4];
    load4<T>(src + pos * c + ch, f);
    store4<T>(dst + r * rs + s * cs + ch, f);
  }
}

}  // namespace

// ------------------------------------------------------------------ confidence pair input
size_t conf_init_ws_bytes(int64_t n_rows, int64_t n_cols, int c_z, int n_bins) {
  Arena ar(nullptr, 0);
  ar.take<float>((size_t)n_rows * c_z);
  ar.take<float>((size_t)n_cols * c_z);
  ar.take<float>((size_t)(n_bins + 1) * c_z);
  return ar.used;
}

template <class T>
static int conf_init_t(const pf_confidence_init_params* p, const T* s, int64_t s_stride, const float* coords,
                       pf_pair_view zi, pf_pair_view zo, int64_t row0, int64_t n_rows, int64_t col0, int64_t n_cols,
                       int c_s, int c_z, int nb, Arena& ar, cudaStream_t st) {
  float* zr = ar.take<float>((size_t)n_rows * c_z);
  float* zc = ar.take<float>((size_t)n_cols * c_z);
  float* wt = ar.take<float>((size_t)(nb + 1) * c_z);
  if (!ar.ok()) return fail(PF_EWORKSPACE, "confidence pair init workspace too small");
  PF_TRY(simt::gemm_rows<T>(s + row0 * s_stride, s_stride, (const T*)p->w_s2, zr, n_rows, c_z, c_s, st));
  PF_TRY(simt::gemm_rows<T>(s + col0 * s_stride, s_stride, (const T*)p->w_s1, zc, n_cols, c_z, c_s, st));
  {
    PF_LAUNCH_SCOPE(st, "k_cols_to_rows");
    k_cols_to_rows<T><<<nblk((int64_t)nb * c_z, 256), 256, 0, st>>>((const T*)p->w_d, nb, c_z, wt);
    k_cols_to_rows<T><<<nblk(c_z, 256), 256, 0, st>>>((const T*)p->w_d0, 1, c_z, wt + (size_t)nb * c_z);
  }
  PF_CHECK_LAUNCH();
  ConfArgs a{zr,   zc,     wt,  coords,        p->lower_bins, p->upper_bins, nb,           row0,         n_rows,
             col0, n_cols, c_z, zi.row_stride, zi.col_stride, zo.row_stride, zo.col_stride};
  const int64_t blocks = (n_rows * n_cols + 7) / 8;
  if (blocks > 0x7fffffffll) return fail(PF_EUNSUPPORTED, "confidence pair init: tile too large");
  {
    PF_LAUNCH_SCOPE_WORK(st, "k_conf_init", 2.0 * (double)n_rows * n_cols * c_z * sizeof(T), 'b');
    k_conf_init<T><<<(unsigned)blocks, 256, 0, st>>>(a, (const T*)zi.ptr, (T*)zo.ptr);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

int conf_init(const pf_confidence_init_params* p, const void* s, int64_t s_stride, const float* coords,
              pf_pair_view zi, pf_pair_view zo, int64_t row0, int64_t n_rows, int64_t col0, int64_t n_cols, int c_s,
              int c_z, int n_bins, int dtype, void* ws, size_t ws_bytes, cudaStream_t st) {
  Arena ar(ws, ws_bytes);
  if (dtype == PF_F32)
    return conf_init_t<float>(p, (const float*)s, s_stride, coords, zi, zo, row0, n_rows, col0, n_cols, c_s, c_z,
                              n_bins, ar, st);
  return conf_init_t<__nv_bfloat16>(p, (const __nv_bfloat16*)s, s_stride, coords, zi, zo, row0, n_rows, col0, n_cols,
                                    c_s, c_z, n_bins, ar, st);
}

// ------------------------------------------------------------------ diffusion pair conditioning
static size_t sub_ws_bytes(int64_t P, int c_z, int c_zd, int dtype) {
  size_t need = 0, b = 0;
  if (c_z != c_zd && pf_pair_ln_linear_workspace_size(P, 1, c_z, c_zd, dtype, &b) == PF_OK && b > need) need = b;
  if (pf_pair_ln_linear_workspace_size(P, 1, 2 * c_zd, c_zd, dtype, &b) == PF_OK && b > need) need = b;
  if (pf_transition_workspace_size(P, c_zd, 2, dtype, &b) == PF_OK && b > need) need = b;
  return need;
}

size_t diffusion_ws_bytes(int64_t n_rows, int64_t n_cols, int c_z, int c_zd, int r_max, int s_max, int dtype) {
  const int64_t P = n_rows * n_cols;
  const size_t esz = dtype == PF_F32 ? 4 : 2;
  Arena ar(nullptr, 0);
  ar.take<char>((size_t)P * 2 * c_zd * esz);  // [x | relp]
  ar.take<char>((size_t)P * c_zd * esz);      // the dense pair before the final copy
  ar.take<float>((size_t)relp_n_feat(r_max, s_max) * c_zd);
  ar.take<char>(sub_ws_bytes(P, c_z, c_zd, dtype));
  return ar.used;
}

template <class T>
static int diffusion_t(const pf_diffusion_pair_params* p, pf_pair_view zt, pf_token_ids ids, pf_pair_view zo,
                       int64_t row0, int64_t n_rows, int64_t col0, int64_t n_cols, int c_z, int c_zd, int r_max,
                       int s_max, int dtype, Arena& ar, cudaStream_t st) {
  const int64_t P = n_rows * n_cols;
  const int nf = relp_n_feat(r_max, s_max);
  T* cat = ar.take<T>((size_t)P * 2 * c_zd);
  T* dense = ar.take<T>((size_t)P * c_zd);
  float* wt = ar.take<float>((size_t)nf * c_zd);
  const size_t sub_bytes = sub_ws_bytes(P, c_z, c_zd, dtype);
  char* sub = ar.take<char>(sub_bytes);
  if (!ar.ok()) return fail(PF_EWORKSPACE, "diffusion pair conditioning workspace too small");
  // a dense output tile is the working buffer itself
  const bool out_dense = zo.col_stride == c_zd && zo.row_stride == n_cols * c_zd;
  if (out_dense) dense = (T*)zo.ptr;
  const bool compress = c_z != c_zd;
  const pf_pair_view cat_v{cat, n_cols * 2 * c_zd, 2 * c_zd};
  if (compress) {
    const pf_pair_linear_params lp{p->ln_zt_w, nullptr, p->w_zt};
    PF_TRY(pf_pair_ln_linear_fwd(&lp, zt, cat_v, n_rows, n_cols, c_z, c_zd, 0, dtype, sub, sub_bytes, st));
  }
  {
    PF_LAUNCH_SCOPE(st, "k_cols_to_rows");
    k_cols_to_rows<T><<<nblk((int64_t)nf * c_zd, 256), 256, 0, st>>>((const T*)p->w_relp, nf, c_zd, wt);
  }
  PF_CHECK_LAUNCH();
  {
    const int64_t blocks = (P + 7) / 8;
    if (blocks > 0x7fffffffll) return fail(PF_EUNSUPPORTED, "diffusion pair: tile too large");
    PF_LAUNCH_SCOPE_WORK(st, "k_relp_cat", (compress ? 1.0 : 3.0) * (double)P * c_zd * sizeof(T), 'b');
    k_relp_cat<T><<<(unsigned)blocks, 256, 0, st>>>(wt, ids, row0, n_rows, col0, n_cols, c_zd, r_max, s_max,
                                                    compress ? nullptr : (const T*)zt.ptr, zt.row_stride,
                                                    zt.col_stride, cat);
  }
  PF_CHECK_LAUNCH();
  const pf_pair_view dv{dense, n_cols * c_zd, c_zd};
  const pf_pair_linear_params lz{p->ln_z_w, nullptr, p->w_z};
  PF_TRY(pf_pair_ln_linear_fwd(&lz, cat_v, dv, n_rows, n_cols, 2 * c_zd, c_zd, 0, dtype, sub, sub_bytes, st));
  PF_TRY(pf_transition_fwd(&p->t1, dense, c_zd, dense, c_zd, P, c_zd, 2, 1, dtype, sub, sub_bytes, st));
  PF_TRY(pf_transition_fwd(&p->t2, dense, c_zd, dense, c_zd, P, c_zd, 2, 1, dtype, sub, sub_bytes, st));
  if (out_dense) return PF_OK;
  {
    PF_LAUNCH_SCOPE_WORK(st, "k_to_view", 2.0 * (double)P * c_zd * sizeof(T), 'b');
    k_to_view<T><<<(unsigned)((P + 7) / 8), 256, 0, st>>>(dense, n_rows, n_cols, c_zd, (T*)zo.ptr, zo.row_stride,
                                                          zo.col_stride);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

int diffusion(const pf_diffusion_pair_params* p, pf_pair_view zt, pf_token_ids ids, pf_pair_view zo, int64_t row0,
              int64_t n_rows, int64_t col0, int64_t n_cols, int c_z, int c_zd, int r_max, int s_max, int dtype,
              void* ws, size_t ws_bytes, cudaStream_t st) {
  Arena ar(ws, ws_bytes);
  if (dtype == PF_F32)
    return diffusion_t<float>(p, zt, ids, zo, row0, n_rows, col0, n_cols, c_z, c_zd, r_max, s_max, dtype, ar, st);
  return diffusion_t<__nv_bfloat16>(p, zt, ids, zo, row0, n_rows, col0, n_cols, c_z, c_zd, r_max, s_max, dtype, ar,
                                    st);
}

}  // namespace heads
}  // namespace pf
