// pf_tc_rows.cu -- tensor-core (tcgen05) path for the Pairformer widths outside the fused
// c = 128 kernels: the template stack (c_z = 64, c_h = 128, transition x2), the structural
// refiner (c_z = c_h = 384, 12 heads of 32, transition x2, AttentionPairBias on c_z = 384) and
// any other width with c_z % 8 == 0 and c_h % 64 == 0 (reference: opendde/config/model_base.py
// :20,30; opendde/model/modules/pairformer.py:91-93,804-808,1678-1685).
//
// Each op is a short chain of width-generic kernels over the caller's workspace:
//   k_ln_pos     LayerNorm of every position of a bf16 pair view (channels contiguous) into
//                contiguous rows; L lanes per position, 16-byte loads and stores, fp32 statistics
//                (two-pass mean / centred variance, eps inside the root, as layers.py:226-269).
//   k_ln_cmajor  the same over the channel-major contraction output x[ch][i][j]: a tile of
//                128 positions x c_h channels staged in shared memory, rows written out.
//   k_pack_w     the weights of one GEMM in its B-operand row order: 64-row halves of two
//                matrices interleaved per 128 rows (p | g of a projection side, a | b of the
//                SwiGLU), or up to four matrices concatenated (q | k | v | g).
//   k_rowgemm<E> persistent GEMM D[p, n] = sum_k A[p, k] W[n, k] over 128-position tiles of a
//                contiguous bf16 row buffer: K streamed in 64-channel blocks by TMA through a
//                4-stage ring, tiles of 128 x BN (BN <= 256) accumulated in TMEM (two
//                accumulators, so the epilogue of one tile overlaps the MMAs of the next), then
//                the op's epilogue E from TMEM: gated projection stored channel-major (trimul
//                a / b), q / k / v^T / gate for the attention core, head-major bias, SwiGLU
//                hidden rows, or the residual update of a pair view (optionally gated).
//   k_gate_mul   o *= g (the attention output gate).
// The per-channel contraction of the triangle update and the attention core are the c = 128
// path's own kernels (pf_tc_internal.h); both are width-independent.

#include "pf_common.cuh"
#include "pf_prof.h"
#include "pf_sm100.cuh"
#include "pf_tc.h"
#include "pf_simt.h"
#include "pf_tc_internal.h"
#include "pf_tmap.h"

namespace pf {
namespace tc {
using namespace sm100;

namespace {

constexpr float LOG2E_R = 1.4426950408889634f;
constexpr int RD = 32;  // attention head dimension

// ------------------------------------------------------------------ LayerNorm of pair views
// out[p*c + ch] = LN(x(r, s))[ch], p = r*n_cols + s; x(r, s) = x + r*rs + s*cs (elements),
// channels contiguous. With a second view y: LN(x(r, s) + y(r, s)) (the sum held in bf16
// between the passes); norm = 0: the plain x (+ y), no LayerNorm. L lanes per position (a power
// of two <= 16), each lane holding up to MAXV 16-byte vectors (8 channels each) between the passes.
template <int L, int MAXV>
__global__ void __launch_bounds__(256) k_ln_pos(const __nv_bfloat16* __restrict__ x, int64_t rs, int64_t cs,
                                                const __nv_bfloat16* __restrict__ y, int64_t yrs, int64_t ycs,
                                                int norm, int64_t n_rows, int64_t n_cols, int c,
                                                const float* __restrict__ gamma, const float* __restrict__ beta,
                                                __nv_bfloat16* __restrict__ out) {
  const int64_t per_block = 256 / L;
  const int64_t p = (int64_t)blockIdx.x * per_block + threadIdx.x / L;
  const int sub = threadIdx.x % L;
  const bool live = p < n_rows * n_cols;
  const int nvec = c >> 3;
  uint4 v[MAXV];
  float sum = 0.f;
  const __nv_bfloat16* src = x;
  const __nv_bfloat16* src2 = y;
  if (live) {
    const int64_t r = p / n_cols, s = p - r * n_cols;
    src = x + r * rs + s * cs;
    if (y) src2 = y + r * yrs + s * ycs;
  }
#pragma unroll
  for (int t = 0; t < MAXV; ++t) {
    const int vi = t * L + sub;
    v[t] = make_uint4(0u, 0u, 0u, 0u);
    if (live && vi < nvec) {
      v[t] = *reinterpret_cast<const uint4*>(src + vi * 8);
      if (y) {
        const uint4 u = *reinterpret_cast<const uint4*>(src2 + vi * 8);
        const uint32_t wx[4] = {v[t].x, v[t].y, v[t].z, v[t].w}, wy[4] = {u.x, u.y, u.z, u.w};
        uint32_t ws[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) ws[e] = pack_bf16(bf16lo(wx[e]) + bf16lo(wy[e]), bf16hi(wx[e]) + bf16hi(wy[e]));
        v[t] = make_uint4(ws[0], ws[1], ws[2], ws[3]);
      }
      const uint32_t w[4] = {v[t].x, v[t].y, v[t].z, v[t].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) sum += bf16lo(w[e]) + bf16hi(w[e]);
    }
  }
  if (!norm) {  // uniform over the block: no lane reaches the shuffles below
    if (!live) return;
#pragma unroll
    for (int t = 0; t < MAXV; ++t) {
      const int vi = t * L + sub;
      if (vi < nvec) *reinterpret_cast<uint4*>(out + p * c + vi * 8) = v[t];
    }
    return;
  }
#pragma unroll
  for (int o = L / 2; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float mean = sum / (float)c;
  float sq = 0.f;
#pragma unroll
  for (int t = 0; t < MAXV; ++t) {
    const int vi = t * L + sub;
    if (live && vi < nvec) {
      const uint32_t w[4] = {v[t].x, v[t].y, v[t].z, v[t].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float d0 = bf16lo(w[e]) - mean, d1 = bf16hi(w[e]) - mean;
        sq = fmaf(d0, d0, sq);
        sq = fmaf(d1, d1, sq);
      }
    }
  }
#pragma unroll
  for (int o = L / 2; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  const float rstd = rsqrtf(sq / (float)c + 1e-5f);
  if (!live) return;
#pragma unroll
  for (int t = 0; t < MAXV; ++t) {
    const int vi = t * L + sub;
    if (vi < nvec) {
      const uint32_t w[4] = {v[t].x, v[t].y, v[t].z, v[t].w};
      uint32_t o4[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ch = vi * 8 + e * 2;
        float y0 = (bf16lo(w[e]) - mean) * rstd, y1 = (bf16hi(w[e]) - mean) * rstd;
        if (gamma) {
          y0 *= gamma[ch];
          y1 *= gamma[ch + 1];
        }
        if (beta) {
          y0 += beta[ch];
          y1 += beta[ch + 1];
        }
        o4[e] = pack_bf16(y0, y1);
      }
      *reinterpret_cast<uint4*>(out + p * c + vi * 8) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
    }
  }
}

// out[(i*n_j + j)*c + ch] = LN over ch of x[(ch*n_i + i)*ld + j]. One CTA of 256 threads per
// (i, 64 j): the [ch][64] bf16 tile is loaded into shared memory one 128-byte channel row per
// warp instruction, then four threads per position each sum a quarter of the channels; the four
// partial sums (then the four partial squared deviations) are combined through shared memory. A thread per position over all c channels (the previous form) left a c-long dependent
// chain and, with c * 256 B of shared memory per 128 positions, two CTAs per SM at c = 384.
constexpr int CM_J = 64;
__global__ void __launch_bounds__(256) k_ln_cmajor(const __nv_bfloat16* __restrict__ x, int64_t ld, int64_t n_i,
                                                   int64_t n_j, int c, const float* __restrict__ gamma,
                                                   const float* __restrict__ beta, __nv_bfloat16* __restrict__ out) {
  extern __shared__ __nv_bfloat16 tile[];  // [c][CM_J]
  __shared__ float red[2][4][CM_J];
  const int64_t tpr = (n_j + CM_J - 1) / CM_J;
  const int64_t i = blockIdx.x / tpr;
  const int64_t j0 = (blockIdx.x % tpr) * CM_J;
  const int64_t plane = n_i * ld;
  {
    // load: warp w takes channels w, w + 8, ...; lane l the positions j0 + 2l, j0 + 2l + 1 (one
    // 128-byte row of a channel per warp instruction, bf16 pairs; ld and j0 are even)
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    const int64_t jj = j0 + 2 * l;
    const __nv_bfloat16* src = x + i * ld + jj;
    uint32_t* t32 = reinterpret_cast<uint32_t*>(tile);
    if (jj + 1 < n_j) {
#pragma unroll 8
      for (int ch = w; ch < c; ch += 8) t32[ch * (CM_J / 2) + l] = *reinterpret_cast<const uint32_t*>(src + ch * plane);
    } else {
      for (int ch = w; ch < c; ch += 8) {
        const uint32_t lo = jj < n_j ? (uint32_t)__bfloat16_as_ushort(src[ch * plane]) : 0u;
        t32[ch * (CM_J / 2) + l] = lo;
      }
    }
  }
  __syncthreads();
  const int jl = threadIdx.x & (CM_J - 1), part = threadIdx.x >> 6;
  const int64_t j = j0 + jl;
  const bool live = j < n_j;
  const int cq = c >> 2, ch0 = part * cq;
  float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
  for (int k = 0; k < cq; ++k) s4[k & 3] += __bfloat162float(tile[(ch0 + k) * CM_J + jl]);
  red[0][part][jl] = (s4[0] + s4[1]) + (s4[2] + s4[3]);
  __syncthreads();
  const float mean = ((red[0][0][jl] + red[0][1][jl]) + (red[0][2][jl] + red[0][3][jl])) / (float)c;
  float q4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
  for (int k = 0; k < cq; ++k) {
    const float d = __bfloat162float(tile[(ch0 + k) * CM_J + jl]) - mean;
    q4[k & 3] = fmaf(d, d, q4[k & 3]);
  }
  red[1][part][jl] = (q4[0] + q4[1]) + (q4[2] + q4[3]);
  __syncthreads();
  if (!live) return;  // no barrier follows
  const float var = ((red[1][0][jl] + red[1][1][jl]) + (red[1][2][jl] + red[1][3][jl])) / (float)c;
  const float rstd = rsqrtf(var + 1e-5f);
  __nv_bfloat16* dst = out + (i * n_j + j) * c + ch0;
  auto y_of = [&](int ch) {
    float y = (__bfloat162float(tile[ch * CM_J + jl]) - mean) * rstd;
    if (gamma) y *= gamma[ch];
    if (beta) y += beta[ch];
    return y;
  };
  if ((cq & 7) == 0) {  // 16-byte stores (the part's start is 16-byte aligned)
    for (int k = 0; k < cq; k += 8) {
      uint32_t o4[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) o4[e] = pack_bf16(y_of(ch0 + k + 2 * e), y_of(ch0 + k + 2 * e + 1));
      *reinterpret_cast<uint4*>(dst + k) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
    }
  } else {  // c % 8 == 0 makes cq even: 4-byte stores
    for (int k = 0; k < cq; k += 2)
      *reinterpret_cast<uint32_t*>(dst + k) = pack_bf16(y_of(ch0 + k), y_of(ch0 + k + 1));
  }
}

// ------------------------------------------------------------------ weight packing
struct PackSrc {
  const __nv_bfloat16* m[4];
};
// mode 0 (interleave): output row n: 128-row group G = n / 128, half = (n % 128) / 64,
//   side = G / groups, source m[2*side + half], source row (G % groups)*64 + n % 64.
// mode 1 (concatenate): source m[n / rows_per_src], source row n % rows_per_src.
__global__ void k_pack_w(PackSrc src, int mode, int groups, int rows_per_src, int k, int64_t n_rows,
                         __nv_bfloat16* __restrict__ dst) {
  const int64_t n = blockIdx.x;
  if (n >= n_rows) return;
  const __nv_bfloat16* s;
  if (mode == 0) {
    const int G = (int)(n / 128), half = (int)((n % 128) / 64), side = G / groups;
    s = src.m[2 * side + half] + ((int64_t)(G % groups) * 64 + n % 64) * k;
  } else {
    s = src.m[n / rows_per_src] + (n % rows_per_src) * (int64_t)k;
  }
  const uint4* sv = reinterpret_cast<const uint4*>(s);
  uint4* dv = reinterpret_cast<uint4*>(dst + n * k);
  for (int v = threadIdx.x; v < k / 8; v += blockDim.x) dv[v] = sv[v];
}

// o[i] = o[i] * g[i] (bf16), 8 elements per thread
__global__ void k_gate_mul(__nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ g, int64_t n8) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  uint4 a = reinterpret_cast<uint4*>(o)[i];
  const uint4 b = reinterpret_cast<const uint4*>(g)[i];
  uint32_t* aw = &a.x;
  const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
  uint32_t r[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) r[e] = pack_bf16(bf16lo(aw[e]) * bf16lo(bw[e]), bf16hi(aw[e]) * bf16hi(bw[e]));
  reinterpret_cast<uint4*>(o)[i] = make_uint4(r[0], r[1], r[2], r[3]);
}

// ob[j*c + ch] = bf16(o[j*c + ch] * sigmoid(g[j*g_ps + ch])) (the gate of the single attention,
// accurate exp as in the fp32 path)
__global__ void k_gate_f32_bf16(const float* __restrict__ o, const float* __restrict__ g, int64_t g_ps, int64_t nq,
                                int c, __nv_bfloat16* __restrict__ ob) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nq * c) return;
  const int64_t j = i / c;
  const int ch = (int)(i - j * c);
  ob[i] = __float2bfloat16_rn(o[i] * (1.0f / (1.0f + expf(-g[j * g_ps + ch]))));
}

// ------------------------------------------------------------------ the row GEMM
constexpr int RB_M = 128, RB_K = 64, R_STAGES = 4, RB_NMAX = 256;
constexpr uint32_t R_A_BYTES = RB_M * RB_K * 2;    // 16 KB
constexpr uint32_t R_B_BYTES = RB_NMAX * RB_K * 2;  // 32 KB
constexpr uint32_t R_STAGE = R_A_BYTES + R_B_BYTES;
constexpr uint32_t R_SMEM = R_STAGES * R_STAGE + 256;

enum Epi : int {
  E_STORE = 0, E_AB = 1, E_RESID = 2, E_SWIGLU = 3, E_QKVG = 4, E_HBIAS = 5, E_STOREF = 6, E_OPMAB = 7, E_HEAD = 8
};
// A operand: contiguous rows (A_ROWS), or the outer products X[(i, c)][(j, e)] of
// OuterProductMean read as rows (i, j) of K = (c, e) through a 4-D tensor map (A_OUTER)
enum AMode : int { A_ROWS = 0, A_OUTER = 1 };

struct RowArgs {
  int64_t n_pos;          // rows of A (positions)
  int64_t m_tiles;
  int n_tiles, bn, kb;    // output tiles of bn columns; K blocks of 64 channels
  int64_t n_work;         // m_tiles * n_tiles
  int n_out;              // logical output columns that exist
  unsigned int* status;
  int64_t e_cols;         // position p -> (r, c) = (p / e_cols, p % e_cols) in the epilogue's view
  // E_STORE (act 1: sigmoid) and E_SWIGLU: out[p*ldo + n]
  __nv_bfloat16* out;
  int64_t ldo;
  int act;
  // E_STOREF: outf[p*ldo + n] = acc + (n < n_colbias ? colbias[n] : 0), fp32
  float* outf;
  const float* colbias;
  int n_colbias;
  // E_AB: dst[side][(ch*e_rows + r)*ld + c] = mask(r, c) * sigmoid(g) * p; 64-channel groups
  __nv_bfloat16* dst[2];
  int64_t e_rows, ld;
  int ch_groups;
  pf_mask_view mask;
  // E_RESID: out[r*rs + c*cs + n] = (accumulate ? out : 0) + acc * (gate ? gate[p*ldg + n] : 1)
  int64_t rs, cs;
  int accumulate;
  const __nv_bfloat16* gate;
  int64_t ldg;
  //   (E_RESID, optional) acc + colbias[n], divided by rownorm[p] (or norm_const if rownorm is null)
  const float* rownorm;
  float norm_const;
  int divide;
  // A_OUTER: position tiles are (i, 128 j) of an a_rows x e_cols grid, a_tpr tiles per i
  int64_t a_tpr;
  // E_OPMAB: dst[0][(r*C + ch)*ld + c] = mask(r, c) * acc  (the a^T / b^T operands of the outer
  // product, C = n_out channels)
  // E_QKVG: columns [q | k | v | g], heads x 32 each; queries are the columns
  // [q_col0, q_col0 + n_q) of the view
  __half* q;
  __half* k;
  __half* vt;
  __nv_bfloat16* g;
  int heads;
  int64_t n_q, q_col0, ld_keys;
  float q_scale;
  // E_HBIAS: bias[h*hs + r*bias_rs + c] = acc_h * scale (fp32, or f16 if bias_f16)
  void* bias;
  int64_t hs, bias_rs;
  int bias_f16;
  float bias_scale;
  // E_HEAD: y = acc + bias_scale * colbias[n] (colbias may be null) stored at
  // (outf or out) + r*rs + c*cs + n; contact[r*contact_rs + c*contact_cs] = sum over n <
  // contact_bins of softmax(y) (one output tile: bn >= n_out)
  float* contact;
  int64_t contact_rs, contact_cs;
  int contact_bins;
};

__device__ __forceinline__ uint4 pack8_bf16(const float* f) {
  return make_uint4(pack_bf16(f[0], f[1]), pack_bf16(f[2], f[3]), pack_bf16(f[4], f[5]), pack_bf16(f[6], f[7]));
}
__device__ __forceinline__ uint4 pack8_f16(const float* f) {
  return make_uint4(pack_f16(f[0], f[1]), pack_f16(f[2], f[3]), pack_f16(f[4], f[5]), pack_f16(f[6], f[7]));
}

// Lines the epilogue of a tile will read (the residual row and the gate row of E_RESID), sent to
// L2 before the tile's accumulator is ready. With one thread per position and every thread
// reading its own row, the reads otherwise reach DRAM with only a few 16-byte loads in flight
// per SM: the accumulating epilogue ran 20x slower than the storing one (6.7 vs 0.32 ms for
// 2.36M rows of 128 channels).
template <int E>
__device__ __forceinline__ void row_prefetch(const RowArgs& a, bool valid, int64_t p, int64_t r, int64_t c, int n0) {
  if constexpr (E == E_RESID) {
    if (!valid || n0 >= a.n_out) return;
    const int bytes = (a.n_out - n0 < a.bn ? a.n_out - n0 : a.bn) * 2;
    if (a.accumulate) {
      const char* o = reinterpret_cast<const char*>(a.out + r * a.rs + c * a.cs + n0);
      for (int b = 0; b < bytes; b += 128) prefetch_l2(o + b);
    }
    if (a.gate) {
      const char* g = reinterpret_cast<const char*>(a.gate + p * a.ldg + n0);
      for (int b = 0; b < bytes; b += 128) prefetch_l2(g + b);
    }
  }
}

// Epilogue of one 128 x bn accumulator: thread = one position (TMEM lane), taddr = its lane's
// address at column 0 of the accumulator. Every tcgen05.ld is executed by all 32 lanes.
template <int E>
__device__ __forceinline__ void row_epilogue(const RowArgs& a, uint32_t taddr, bool valid, int64_t p, int64_t r,
                                             int64_t c, int n0) {
  if constexpr (E == E_STOREF) {
    for (int cc = 0; cc < a.bn; cc += 16) {
      uint32_t v[16];
      tmem_ld16(taddr + cc, v);
      tmem_ld_wait();
      const int n = n0 + cc;
      if (!valid || n >= a.n_out) continue;
      float* o = a.outf + p * a.ldo + n;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        if (n + e < a.n_out) {
          float y = __uint_as_float(v[e]);
          if (n + e < a.n_colbias) y += a.colbias[n + e];
          o[e] = y;
        }
      }
    }
  } else if constexpr (E == E_STORE || E == E_RESID) {
    for (int cc = 0; cc < a.bn; cc += 32) {
      const int n = n0 + cc;
      // columns of this tile (bn is a multiple of 16, not of 32) that exist
      int cnt = a.n_out - n < 32 ? a.n_out - n : 32;
      if (a.bn - cc < cnt) cnt = a.bn - cc;
      // E_RESID: the chunk's residual and gate vectors, all in flight before the TMEM load
      uint4 oq[4], gq[4];
      if constexpr (E == E_RESID) {
        if (valid && cnt == 32) {
          const uint4* o4 = reinterpret_cast<const uint4*>(a.out + r * a.rs + c * a.cs + n);
          const uint4* g4 = a.gate ? reinterpret_cast<const uint4*>(a.gate + p * a.ldg + n) : nullptr;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            oq[e] = a.accumulate ? o4[e] : make_uint4(0u, 0u, 0u, 0u);
            gq[e] = g4 ? g4[e] : make_uint4(0u, 0u, 0u, 0u);
          }
        }
      }
      uint32_t v[32];
      tmem_ld32(taddr + cc, v);
      tmem_ld_wait();
      if (!valid || n >= a.n_out) continue;
      float f[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) f[e] = __uint_as_float(v[e]);
      if constexpr (E == E_STORE) {
        if (a.act == 1) {
#pragma unroll
          for (int e = 0; e < 32; ++e) f[e] = fast_sigmoid(f[e]);
        }
        __nv_bfloat16* o = a.out + p * a.ldo + n;
        if (cnt == 32) {
#pragma unroll
          for (int e = 0; e < 4; ++e) reinterpret_cast<uint4*>(o)[e] = pack8_bf16(f + 8 * e);
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (e < cnt) o[e] = __float2bfloat16_rn(f[e]);
        }
      } else {
        __nv_bfloat16* o = a.out + r * a.rs + c * a.cs + n;
        const __nv_bfloat16* gp = a.gate ? a.gate + p * a.ldg + n : nullptr;
        if (a.divide) {
          const float nrm = a.rownorm ? a.rownorm[p] : a.norm_const;
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float bias = (a.colbias && e < cnt) ? a.colbias[n + e] : 0.f;
            f[e] = (f[e] + bias) / nrm;
          }
        }
        if (cnt == 32) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float y[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) y[u] = f[8 * e + u];
            if (gp) {
              const uint32_t gw[4] = {gq[e].x, gq[e].y, gq[e].z, gq[e].w};
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                y[2 * u] *= bf16lo(gw[u]);
                y[2 * u + 1] *= bf16hi(gw[u]);
              }
            }
            if (a.accumulate) {
              const uint32_t ow[4] = {oq[e].x, oq[e].y, oq[e].z, oq[e].w};
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                y[2 * u] += bf16lo(ow[u]);
                y[2 * u + 1] += bf16hi(ow[u]);
              }
            }
            reinterpret_cast<uint4*>(o)[e] = pack8_bf16(y);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            if (e < cnt) {
              float y = f[e];
              if (gp) y *= __bfloat162float(gp[e]);
              if (a.accumulate) y += __bfloat162float(o[e]);
              o[e] = __float2bfloat16_rn(y);
            }
          }
        }
      }
    }
  } else if constexpr (E == E_AB || E == E_SWIGLU) {
    float mk = 0.f;
    if (E == E_AB && valid)
      mk = a.mask.ptr ? a.mask.ptr[r * a.mask.row_stride + c * a.mask.col_stride] : 1.f;
    for (int sub = 0; sub < a.bn; sub += 128) {
      const int G = (n0 + sub) >> 7;  // 128-column group: [first 64 | second 64]
#pragma unroll 1
      for (int cc = 0; cc < 64; cc += 16) {
        uint32_t x0[16], x1[16];
        tmem_ld16(taddr + sub + cc, x0);
        tmem_ld16(taddr + sub + 64 + cc, x1);
        tmem_ld_wait();
        if (!valid) continue;
        if constexpr (E == E_AB) {
          // reference order mask * sigmoid(g) * p (triangular.py:539-544)
          const int side = G / a.ch_groups;
          const int64_t ch0 = (int64_t)(G % a.ch_groups) * 64 + cc;
          __nv_bfloat16* d = a.dst[side] + (ch0 * a.e_rows + r) * a.ld + c;
          const int64_t plane = a.e_rows * a.ld;
#pragma unroll
          for (int e = 0; e < 16; ++e)
            d[e * plane] = __float2bfloat16_rn(mk * fast_sigmoid(__uint_as_float(x1[e])) * __uint_as_float(x0[e]));
        } else {
          const int h0 = G * 64 + cc;  // hidden unit; n_out counts the packed [a | b] rows
          if (h0 >= a.n_out / 2) continue;
          float y[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float u = __uint_as_float(x0[e]);
            y[e] = u * fast_sigmoid(u) * __uint_as_float(x1[e]);
          }
          uint4* o = reinterpret_cast<uint4*>(a.out + p * a.ldo + h0);
          o[0] = pack8_bf16(y);
          o[1] = pack8_bf16(y + 8);
        }
      }
    }
  } else if constexpr (E == E_OPMAB) {
    float mk = 0.f;
    if (valid) mk = a.mask.ptr ? a.mask.ptr[r * a.mask.row_stride + c * a.mask.col_stride] : 1.f;
#pragma unroll 1
    for (int cc = 0; cc < a.bn; cc += 16) {
      uint32_t v[16];
      tmem_ld16(taddr + cc, v);
      tmem_ld_wait();
      if (!valid) continue;
      __nv_bfloat16* d = a.dst[0] + (r * a.n_out + n0 + cc) * a.ld + c;
#pragma unroll
      for (int e = 0; e < 16; ++e) d[e * a.ld] = __float2bfloat16_rn(mk * __uint_as_float(v[e]));
    }
  } else if constexpr (E == E_QKVG) {
    const int hd = a.heads * RD;
    const int part = n0 / hd, w0 = n0 - part * hd;
    const int64_t j = c - a.q_col0;
    const bool is_q = valid && j >= 0 && j < a.n_q;
#pragma unroll 1
    for (int cc = 0; cc < a.bn; cc += 16) {
      uint32_t v[16];
      tmem_ld16(taddr + cc, v);
      tmem_ld_wait();
      const int within = w0 + cc, h = within >> 5, d0 = within & 31;
      float f[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) f[e] = __uint_as_float(v[e]);
      const int64_t ih = r * a.heads + h;
      if (part == 0) {
        if (!is_q) continue;
#pragma unroll
        for (int e = 0; e < 16; ++e) f[e] *= a.q_scale;
        uint4* o = reinterpret_cast<uint4*>(a.q + ((ih * a.n_q + j) * RD + d0));
        o[0] = pack8_f16(f);
        o[1] = pack8_f16(f + 8);
      } else if (part == 1) {
        if (!valid) continue;
        uint4* o = reinterpret_cast<uint4*>(a.k + ((ih * a.ld_keys + c) * RD + d0));
        o[0] = pack8_f16(f);
        o[1] = pack8_f16(f + 8);
      } else if (part == 2) {
        if (!valid) continue;
        __half* o = a.vt + (ih * RD + d0) * a.ld_keys + c;
#pragma unroll
        for (int e = 0; e < 16; ++e) o[e * a.ld_keys] = __float2half_rn(f[e]);
      } else {
        if (!is_q) continue;
#pragma unroll
        for (int e = 0; e < 16; ++e) f[e] = fast_sigmoid(f[e]);
        uint4* o = reinterpret_cast<uint4*>(a.g + ((r * a.n_q + j) * hd + within));
        o[0] = pack8_bf16(f);
        o[1] = pack8_bf16(f + 8);
      }
    }
  } else if constexpr (E == E_HEAD) {
    // one pass over the accumulator in 16-column chunks: store the logits and keep an online
    // softmax (running max, and the sums over all bins and over the contact bins, rescaled when
    // the max grows)
    float mx = -INFINITY, tot = 0.f, sel = 0.f;
#pragma unroll 1
    for (int cc = 0; cc < a.bn; cc += 16) {
      const int n = n0 + cc;
      const int cnt = a.n_out - n < 16 ? (a.n_out - n > 0 ? a.n_out - n : 0) : 16;
      // the chunk's bias values in flight before the TMEM load's wait
      float bias[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) bias[e] = (a.colbias && e < cnt) ? a.bias_scale * a.colbias[n + e] : 0.f;
      uint32_t v[16];
      tmem_ld16(taddr + cc, v);
      tmem_ld_wait();
      if (!valid || cnt == 0) continue;
      float f[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) f[e] = __uint_as_float(v[e]) + bias[e];
      const int64_t off = r * a.rs + c * a.cs + n;
      if (a.outf) {
        float* o = a.outf + off;
        if (cnt == 16 && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
          for (int e = 0; e < 4; ++e)
            reinterpret_cast<float4*>(o)[e] = make_float4(f[4 * e], f[4 * e + 1], f[4 * e + 2], f[4 * e + 3]);
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e)
            if (e < cnt) o[e] = f[e];
        }
      } else {
        __nv_bfloat16* o = a.out + off;
        if (cnt == 16 && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
          reinterpret_cast<uint4*>(o)[0] = pack8_bf16(f);
          reinterpret_cast<uint4*>(o)[1] = pack8_bf16(f + 8);
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e)
            if (e < cnt) o[e] = __float2bfloat16_rn(f[e]);
        }
      }
      if (a.contact) {
        // trees (depth 4) rather than 16-long chains: four epilogue warps per SM leave latency
        // exposed
        float t[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) t[e] = e < cnt ? f[e] : -INFINITY;
#pragma unroll
        for (int w = 8; w > 0; w >>= 1)
#pragma unroll
          for (int e = 0; e < w; ++e) t[e] = fmaxf(t[e], t[e + w]);
        const float nm = fmaxf(mx, t[0]);
        const float scale = ex2_approx((mx - nm) * LOG2E_R);  // 0 on the first chunk (mx = -inf)
        float ex[16], es[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          ex[e] = e < cnt ? ex2_approx((f[e] - nm) * LOG2E_R) : 0.f;
          es[e] = n + e < a.contact_bins ? ex[e] : 0.f;
        }
#pragma unroll
        for (int w = 8; w > 0; w >>= 1)
#pragma unroll
          for (int e = 0; e < w; ++e) {
            ex[e] += ex[e + w];
            es[e] += es[e + w];
          }
        tot = fmaf(tot, scale, ex[0]);
        sel = fmaf(sel, scale, es[0]);
        mx = nm;
      }
    }
    if (a.contact && valid) a.contact[r * a.contact_rs + c * a.contact_cs] = sel / tot;
  } else {  // E_HBIAS
    uint32_t v[16];
    tmem_ld16(taddr, v);
    tmem_ld_wait();
    if (!valid) return;
#pragma unroll
    for (int h = 0; h < 16; ++h) {
      if (h >= a.heads) break;
      const float y = __uint_as_float(v[h]) * a.bias_scale;
      const int64_t idx = h * a.hs + r * a.bias_rs + c;
      if (a.bias_f16)
        reinterpret_cast<__half*>(a.bias)[idx] = __float2half_rn(y);
      else
        reinterpret_cast<float*>(a.bias)[idx] = y;
    }
  }
}

// Persistent: one CTA per SM walks the (position tile, output tile) list, output tile fastest
// (the CTAs running at one time share an A tile in L2). Warp 0: TMA producer; warp 1: TMEM
// allocation and the MMA thread; warps 2-5: epilogue (thread = TMEM lane = position).
template <int E, int AM>
__global__ void __launch_bounds__(192, 1) k_rowgemm(const __grid_constant__ CUtensorMap ta,
                                                    const __grid_constant__ CUtensorMap tb, const RowArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gsm = smem_raw + (base - raw);
  const uint32_t bars = base + R_STAGES * R_STAGE;
  // full[s] @8s, empty[s] @32+8s, acc_full[b] @64+8b, acc_empty[b] @80+8b, drain @96; TMEM slot @128
  auto full = [&](uint32_t s) { return bars + 8 * s; };
  auto empty = [&](uint32_t s) { return bars + 32 + 8 * s; };
  auto acc_full = [&](uint32_t b) { return bars + 64 + 8 * b; };
  auto acc_empty = [&](uint32_t b) { return bars + 80 + 8 * b; };
  const uint32_t bar_drain = bars + 96;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gsm + R_STAGES * R_STAGE + 128);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t G = gridDim.x;

  if (tid == 0) {
    for (int s = 0; s < R_STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full(b), 1);
      mbar_init(acc_empty(b), 4);
    }
    mbar_init(bar_drain, 1);
    fence_barrier_init();
    tma_prefetch_desc(&ta);
    tma_prefetch_desc(&tb);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t stage_tx = R_A_BYTES + (uint32_t)a.bn * (RB_K * 2);

  if (warp == 0) {
    if (lane == 0) {
      uint32_t cnt = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < a.n_work && ok; t += G) {
        const int64_t mt = t / a.n_tiles;
        const int n0 = (int)(t % a.n_tiles) * a.bn;
        for (int kb = 0; kb < a.kb; ++kb, ++cnt) {
          const uint32_t s = cnt % R_STAGES, u = cnt / R_STAGES;
          if (u > 0) ok = mbar_wait(empty(s), (u - 1) & 1, a.status) && ok;
          const uint32_t sa = base + s * R_STAGE, sb = sa + R_A_BYTES;
          mbar_arrive_expect_tx(full(s), stage_tx);
          if constexpr (AM == A_OUTER) {
            // rows (i, j0 .. j0 + 127), K block = outer-product channels c = 2 kb, 2 kb + 1
            tma_load_4d(sa, &ta, full(s), 0, (int)(mt % a.a_tpr) * RB_M, 2 * kb, (int)(mt / a.a_tpr));
          } else {
            tma_load_2d(sa, &ta, full(s), kb * RB_K, (int)(mt * RB_M));
          }
          tma_load_2d(sb, &tb, full(s), kb * RB_K, n0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(RB_M, a.bn, true);
      uint32_t cnt = 0, j = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < a.n_work && ok; t += G, ++j) {
        const uint32_t b = j & 1;
        if (j >= 2) ok = mbar_wait(acc_empty(b), ((j >> 1) - 1) & 1, a.status) && ok;
        tc_fence_after();
        const uint32_t acc = tmem + 256 * b;
        for (int kb = 0; kb < a.kb; ++kb, ++cnt) {
          const uint32_t s = cnt % R_STAGES, u = cnt / R_STAGES;
          ok = mbar_wait(full(s), u & 1, a.status) && ok;
          tc_fence_after();
          const uint32_t sa = base + s * R_STAGE, sb = sa + R_A_BYTES;
#pragma unroll
          for (int kk = 0; kk < RB_K / 16; ++kk) {
            // A_OUTER: two 64-byte-row SW64 atoms (one per outer-product channel c) of 8 KB
            const uint64_t ad = AM == A_OUTER ? sdesc(sa + (kk >> 1) * 8192 + (kk & 1) * 32, 512, SWZ_64B)
                                              : sdesc(sa + kk * 32, 1024, SWZ_128B);
            const uint64_t bd = sdesc(sb + kk * 32, 1024, SWZ_128B);
            umma_f16(acc, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(empty(s));  // frees the stage when these MMAs finish
        }
        umma_commit(acc_full(b));
      }
      umma_commit(bar_drain);  // every MMA complete before TMEM is released
      mbar_wait_drain(bar_drain, 0);
    }
  } else {
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;
    uint32_t j = 0;
    for (int64_t t = blockIdx.x; t < a.n_work; t += G, ++j) {
      const int64_t mt = t / a.n_tiles;
      const int n0 = (int)(t % a.n_tiles) * a.bn;
      const uint32_t b = j & 1;
      bool valid;
      int64_t p, r, c;
      if constexpr (AM == A_OUTER) {
        r = mt / a.a_tpr;
        c = (mt % a.a_tpr) * RB_M + row;
        valid = c < a.e_cols;
        p = r * a.e_cols + c;
      } else {
        p = mt * RB_M + row;
        valid = p < a.n_pos;
        r = valid ? p / a.e_cols : 0;
        c = valid ? p - r * a.e_cols : 0;
      }
      row_prefetch<E>(a, valid, p, r, c, n0);  // overlaps the wait for this tile's MMAs
      mbar_wait(acc_full(b), (j >> 1) & 1, a.status);
      tc_fence_after();
      row_epilogue<E>(a, tmem + 256 * b + ((uint32_t)(q * 32) << 16), valid, p, r, c, n0);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty(b));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ host helpers
template <class K>
int set_smem(K kernel, uint32_t bytes) {
  PF_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
  return PF_OK;
}

constexpr int CM_MAX_C = 768;  // k_ln_cmajor: c * 2 * CM_J B of shared memory

int ensure_attrs() {
  static std::atomic<unsigned long long> done{0};
  return once_per_device(done, []() -> int {
    PF_TRY(set_smem(k_rowgemm<E_STORE, A_ROWS>, R_SMEM + 1024));
    PF_TRY(set_smem(k_rowgemm<E_AB, A_ROWS>, R_SMEM + 1024));
    PF_TRY(set_smem(k_rowgemm<E_RESID, A_ROWS>, R_SMEM + 1024));
    PF_TRY(set_smem(k_rowgemm<E_SWIGLU, A_ROWS>, R_SMEM + 1024));
    PF_TRY(set_smem(k_rowgemm<E_QKVG, A_ROWS>, R_SMEM + 1024));
    PF_TRY(set_smem(k_rowgemm<E_HBIAS, A_ROWS>, R_SMEM + 1024));
    PF_TRY(set_smem(k_rowgemm<E_STOREF, A_ROWS>, R_SMEM + 1024));
    PF_TRY(set_smem(k_rowgemm<E_OPMAB, A_ROWS>, R_SMEM + 1024));
    PF_TRY(set_smem(k_rowgemm<E_RESID, A_OUTER>, R_SMEM + 1024));
    PF_TRY(set_smem(k_rowgemm<E_HEAD, A_ROWS>, R_SMEM + 1024));
    PF_TRY(set_smem(k_ln_cmajor, CM_MAX_C * CM_J * 2));
    return PF_OK;
  });
}

bool aligned16(const void* p) { return ((uintptr_t)p) % 16 == 0; }

int check_view(const pf_pair_view& v, const char* what) {
  if (!aligned16(v.ptr) || v.row_stride % 8 || v.col_stride % 8)
    return fail(PF_EINVAL_SHAPE, "%s: bf16 pair view needs a 16-byte aligned base and strides that are "
                "multiples of 8 elements", what);
  return PF_OK;
}

// LayerNorm of the positions (r < n_rows, s < n_cols) of a bf16 view into rows of c channels.
// With y (and its strides): of x + y; norm = 0: the plain x (+ y), no LayerNorm.
int ln_pos2(const __nv_bfloat16* x, int64_t rs, int64_t cs, const __nv_bfloat16* y, int64_t yrs, int64_t ycs,
            int norm, int64_t n_rows, int64_t n_cols, int c, const float* g, const float* b, __nv_bfloat16* out,
            cudaStream_t st) {
  const int64_t P = n_rows * n_cols;
  if (P == 0) return PF_OK;
  const int nvec = c / 8;
  int L = 1;
  while (L * 2 <= nvec && L < 16) L *= 2;
  const int maxv = (nvec + L - 1) / L;
  const unsigned grid = (unsigned)((P + 256 / L - 1) / (256 / L));
  PF_LAUNCH_SCOPE_WORK(st, "k_ln_pos", (y ? 6.0 : 4.0) * (double)P * c, 'b');
#define PF_LNPOS(LL, MV) \
  k_ln_pos<LL, MV><<<grid, 256, 0, st>>>(x, rs, cs, y, yrs, ycs, norm, n_rows, n_cols, c, g, b, out)
  if (L == 16) {
    if (maxv <= 1) PF_LNPOS(16, 1);
    else if (maxv <= 2) PF_LNPOS(16, 2);
    else if (maxv <= 3) PF_LNPOS(16, 3);
    else if (maxv <= 4) PF_LNPOS(16, 4);
    else if (maxv <= 8) PF_LNPOS(16, 8);
    else return fail(PF_EUNSUPPORTED, "LayerNorm width %d > 1024", c);
  } else if (L == 8) {
    PF_LNPOS(8, 2);
  } else if (L == 4) {
    PF_LNPOS(4, 2);
  } else if (L == 2) {
    PF_LNPOS(2, 2);
  } else {
    PF_LNPOS(1, 1);
  }
#undef PF_LNPOS
  PF_CHECK_LAUNCH();
  return PF_OK;
}

int ln_pos(const __nv_bfloat16* x, int64_t rs, int64_t cs, int64_t n_rows, int64_t n_cols, int c, const float* g,
           const float* b, __nv_bfloat16* out, cudaStream_t st) {
  return ln_pos2(x, rs, cs, nullptr, 0, 0, 1, n_rows, n_cols, c, g, b, out, st);
}

int ln_cmajor(const __nv_bfloat16* x, int64_t ld, int64_t n_i, int64_t n_j, int c, const float* g, const float* b,
              __nv_bfloat16* out, cudaStream_t st) {
  if (n_i * n_j == 0) return PF_OK;
  if (c > CM_MAX_C || c % 8) return fail(PF_EUNSUPPORTED, "LayerNorm over %d channel-major channels", c);
  PF_TRY(ensure_attrs());
  const int64_t blocks = n_i * ((n_j + CM_J - 1) / CM_J);
  if (blocks > 0x7fffffffll) return fail(PF_EUNSUPPORTED, "LayerNorm grid too large");
  PF_LAUNCH_SCOPE_WORK(st, "k_ln_cmajor", 4.0 * (double)n_i * n_j * c, 'b');
  k_ln_cmajor<<<(unsigned)blocks, 256, (size_t)c * CM_J * 2, st>>>(x, ld, n_i, n_j, c, g, b, out);
  PF_CHECK_LAUNCH();
  return PF_OK;
}

int pack_w(const void* const* srcs, int mode, int groups, int rows_per_src, int k, int64_t n_rows,
           __nv_bfloat16* dst, cudaStream_t st) {
  PackSrc s{};
  for (int i = 0; i < 4; ++i) {
    s.m[i] = (const __nv_bfloat16*)srcs[i];
    if (s.m[i] && !aligned16(s.m[i])) return fail(PF_EINVAL_ARG, "weights must be 16-byte aligned");
  }
  PF_LAUNCH_SCOPE(st, "k_pack_w");
  k_pack_w<<<(unsigned)n_rows, 64, 0, st>>>(s, mode, groups, rows_per_src, k, n_rows, dst);
  PF_CHECK_LAUNCH();
  return PF_OK;
}

int gate_mul(__nv_bfloat16* o, const __nv_bfloat16* g, int64_t n, cudaStream_t st) {
  if (n == 0) return PF_OK;
  const int64_t n8 = n / 8;
  PF_LAUNCH_SCOPE_WORK(st, "k_gate_mul", 6.0 * (double)n, 'b');
  k_gate_mul<<<(unsigned)((n8 + 255) / 256), 256, 0, st>>>(o, g, n8);
  PF_CHECK_LAUNCH();
  return PF_OK;
}

// Output tile width for n_out columns: the fewest tiles of at most 256 columns, each a
// multiple of `mult` (16 for plain epilogues, 128 for the paired ones).
int pick_bn(int n_out, int mult) {
  const int tiles = (n_out + 255) / 256;
  int bn = (n_out + tiles - 1) / tiles;
  bn = (bn + mult - 1) / mult * mult;
  return bn > 256 ? 256 : bn;
}

// D = A W^T with epilogue E: A is n_pos rows of k bf16 channels at row pitch lda (elements);
// W is w_rows x k bf16, row-major. `name` and `work` feed the launch profiler.
template <int E>
int rowgemm(const __nv_bfloat16* A, int64_t lda, int64_t n_pos, int k, const void* W, int w_rows, RowArgs ra,
            const char* name, unsigned int* status, cudaStream_t st) {
  if (n_pos == 0) return PF_OK;
  if (!aligned16(A) || !aligned16(W) || lda % 8 || k % 8)
    return fail(PF_EINVAL_SHAPE, "%s: operands need 16-byte alignment and widths that are multiples of 8", name);
  if (E == E_STORE || E == E_STOREF || E == E_RESID) {
    // few positions (the single representation: N rows): narrower output tiles, so that the
    // persistent grid still covers the SMs. Chosen before the B tensor map, whose box is bn rows.
    const int64_t m_tiles = (n_pos + RB_M - 1) / RB_M;
    while (ra.bn > 32 && m_tiles * ((ra.n_out + ra.bn - 1) / ra.bn) < sm_count()) {
      const int half = (ra.bn / 2 + 15) / 16 * 16;
      if (half < 32) break;
      ra.bn = half;
    }
  }
  if (ra.bn < 16 || ra.bn > RB_NMAX || ra.bn % 16) return fail(PF_EUNSUPPORTED, "%s: tile width %d", name, ra.bn);
  CUtensorMap ta, tb;
  {
    const uint64_t d[2] = {(uint64_t)k, (uint64_t)n_pos};
    const uint64_t s[1] = {(uint64_t)lda * 2};
    const uint32_t bx[2] = {RB_K, RB_M};
    PF_TRY(make_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, A, d, s, bx, CU_TENSOR_MAP_SWIZZLE_128B));
    const uint64_t dw[2] = {(uint64_t)k, (uint64_t)w_rows};
    const uint64_t sw[1] = {(uint64_t)k * 2};
    const uint32_t bw[2] = {RB_K, (uint32_t)ra.bn};
    PF_TRY(make_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, W, dw, sw, bw, CU_TENSOR_MAP_SWIZZLE_128B));
  }
  ra.n_pos = n_pos;
  ra.m_tiles = (n_pos + RB_M - 1) / RB_M;
  ra.n_tiles = (ra.n_out + ra.bn - 1) / ra.bn;
  ra.kb = (k + RB_K - 1) / RB_K;
  ra.n_work = ra.m_tiles * ra.n_tiles;
  ra.status = status;
  PF_TRY(ensure_attrs());
  const int64_t grid = ra.n_work < sm_count() ? ra.n_work : sm_count();
  {
    // the head GEMM (a few dozen bins per position) is bound by its bytes: the A rows read, the
    // logits and contact probabilities written
    const double work = E == E_HEAD ? (double)n_pos * (2.0 * k + (ra.outf ? 4.0 : 2.0) * ra.n_out +
                                                       (ra.contact ? 4.0 : 0.0))
                                    : 2.0 * (double)n_pos * ra.n_out * k;
    PF_LAUNCH_SCOPE_WORK(st, name, work, E == E_HEAD ? 'b' : 'f');
    k_rowgemm<E, A_ROWS><<<(unsigned)grid, 192, R_SMEM + 1024, st>>>(ta, tb, ra);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

int64_t pad8(int64_t n) { return (n + 7) / 8 * 8; }

// W_out applied to the outer products: rows (i, j) of an n_rows x n_cols grid, K = C*C read
// from x[(i*C + c)*ld_x + j*C + e] (bf16) through a 4-D tensor map {e, j, c, i}: one 64-channel K
// block is the two 32 x 128 boxes of channels c = 2 kb, 2 kb + 1, each a SW64 atom of 64-byte rows.
int rowgemm_outer(const __nv_bfloat16* x, int64_t ld_x, int64_t n_rows, int64_t n_cols, int C, const void* W,
                  int w_rows, RowArgs ra, const char* name, unsigned int* status, cudaStream_t st) {
  if (n_rows * n_cols == 0) return PF_OK;
  if (C != 32 || !aligned16(x) || !aligned16(W) || ld_x % 8)
    return fail(PF_EUNSUPPORTED, "%s: outer-product operand needs C = 32 and 16-byte alignment", name);
  CUtensorMap ta, tb;
  {
    const uint64_t d[4] = {(uint64_t)C, (uint64_t)n_cols, (uint64_t)C, (uint64_t)n_rows};
    const uint64_t str[3] = {(uint64_t)C * 2, (uint64_t)ld_x * 2, (uint64_t)C * ld_x * 2};
    const uint32_t bx[4] = {32, RB_M, 2, 1};
    PF_TRY(make_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, x, d, str, bx, CU_TENSOR_MAP_SWIZZLE_64B));
    const uint64_t dw[2] = {(uint64_t)C * C, (uint64_t)w_rows};
    const uint64_t sw[1] = {(uint64_t)C * C * 2};
    const uint32_t bw[2] = {RB_K, (uint32_t)ra.bn};
    PF_TRY(make_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, W, dw, sw, bw, CU_TENSOR_MAP_SWIZZLE_128B));
  }
  ra.n_pos = n_rows * n_cols;
  ra.e_cols = n_cols;
  ra.a_tpr = (n_cols + RB_M - 1) / RB_M;
  ra.m_tiles = n_rows * ra.a_tpr;
  ra.n_tiles = (ra.n_out + ra.bn - 1) / ra.bn;
  ra.kb = C * C / RB_K;
  ra.n_work = ra.m_tiles * ra.n_tiles;
  ra.status = status;
  PF_TRY(ensure_attrs());
  const int64_t grid = ra.n_work < sm_count() ? ra.n_work : sm_count();
  {
    PF_LAUNCH_SCOPE_WORK(st, name, 2.0 * (double)ra.n_pos * ra.n_out * C * C, 'f');
    k_rowgemm<E_RESID, A_OUTER><<<(unsigned)grid, 192, R_SMEM + 1024, st>>>(ta, tb, ra);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}



// ---------------------------------------------------------------- triangle update, by stage
struct ProjWs {
  __nv_bfloat16 *ln_a, *ln_b, *w;
};
void proj_plan(Arena& ar, int64_t n_rows_a, int64_t n_rows_b, int64_t n_cols, bool same, int c_z, int c_h,
               ProjWs& w) {
  w.ln_a = ar.take<__nv_bfloat16>((size_t)n_rows_a * n_cols * c_z);
  w.ln_b = same ? w.ln_a : ar.take<__nv_bfloat16>((size_t)n_rows_b * n_cols * c_z);
  w.w = ar.take<__nv_bfloat16>((size_t)4 * c_h * c_z);
}

// a(ch, r, s) of za (r < n_a), b(ch, r, s) of zb (r < n_b), s < n_k, channel-major at pitch ld.
int proj_run(const pf_trimul_params* p, pf_pair_view za, pf_pair_view zb, pf_mask_view ma, pf_mask_view mb,
             int64_t n_a, int64_t n_b, int64_t n_k, int c_z, int c_h, __nv_bfloat16* a, __nv_bfloat16* b,
             int64_t ld, const ProjWs& w, unsigned int* status, cudaStream_t st) {
  const bool same = w.ln_a == w.ln_b;
  PF_TRY(check_view(za, "trimul za"));
  PF_TRY(check_view(zb, "trimul zb"));
  PF_TRY(ln_pos((const __nv_bfloat16*)za.ptr, za.row_stride, za.col_stride, n_a, n_k, c_z, p->ln_in_w, p->ln_in_b,
                w.ln_a, st));
  if (!same)
    PF_TRY(ln_pos((const __nv_bfloat16*)zb.ptr, zb.row_stride, zb.col_stride, n_b, n_k, c_z, p->ln_in_w,
                  p->ln_in_b, w.ln_b, st));
  const void* srcs[4] = {p->w_ap, p->w_ag, p->w_bp, p->w_bg};
  const int groups = c_h / 64;
  PF_TRY(pack_w(srcs, 0, groups, 0, c_z, 4 * (int64_t)c_h, w.w, st));
  RowArgs ra{};
  ra.e_cols = n_k;
  ra.ld = ld;
  ra.ch_groups = groups;
  if (same) {
    ra.n_out = 4 * c_h;
    ra.bn = 256;
    ra.dst[0] = a;
    ra.dst[1] = b;
    ra.e_rows = n_a;
    ra.mask = ma;
    return rowgemm<E_AB>(w.ln_a, c_z, n_a * n_k, c_z, w.w, 4 * c_h, ra, "k_rowgemm_trimul_ab", status, st);
  }
  ra.n_out = 2 * c_h;
  ra.bn = 2 * c_h % 256 == 0 ? 256 : 128;
  ra.dst[0] = a;
  ra.dst[1] = a;
  ra.e_rows = n_a;
  ra.mask = ma;
  PF_TRY(rowgemm<E_AB>(w.ln_a, c_z, n_a * n_k, c_z, w.w, 2 * c_h, ra, "k_rowgemm_trimul_ab", status, st));
  ra.dst[0] = b;
  ra.dst[1] = b;
  ra.e_rows = n_b;
  ra.mask = mb;
  return rowgemm<E_AB>(w.ln_b, c_z, n_b * n_k, c_z, w.w + (size_t)2 * c_h * c_z, 2 * c_h, ra,
                       "k_rowgemm_trimul_ab", status, st);
}

struct CombWs {
  __nv_bfloat16 *x, *ln_x, *ln_g, *gate;
  int64_t ld_j;
};
void comb_plan(Arena& ar, int64_t n_i, int64_t n_j, int c_z, int c_h, CombWs& w) {
  w.ld_j = pad8(n_j);
  w.x = ar.take<__nv_bfloat16>((size_t)c_h * n_i * w.ld_j);
  w.ln_x = ar.take<__nv_bfloat16>((size_t)n_i * n_j * c_h);
  w.ln_g = ar.take<__nv_bfloat16>((size_t)n_i * n_j * c_z);
  w.gate = ar.take<__nv_bfloat16>((size_t)n_i * n_j * c_z);
}

int comb_run(const pf_trimul_params* p, const __nv_bfloat16* a, const __nv_bfloat16* b, int64_t ld, int64_t n_i,
             int64_t n_j, int64_t n_k, pf_pair_view zg, pf_pair_view zo, int c_z, int c_h, int acc, const CombWs& w,
             unsigned int* status, cudaStream_t st) {
  PF_TRY(check_view(zg, "trimul zg"));
  PF_TRY(check_view(zo, "trimul zo"));
  PF_TRY(trimul_contract(a, ld, b, ld, n_i, n_j, n_k, c_h, w.x, w.ld_j, status, st));
  PF_TRY(ln_cmajor(w.x, w.ld_j, n_i, n_j, c_h, p->ln_out_w, p->ln_out_b, w.ln_x, st));
  PF_TRY(ln_pos((const __nv_bfloat16*)zg.ptr, zg.row_stride, zg.col_stride, n_i, n_j, c_z, p->ln_in_w, p->ln_in_b,
                w.ln_g, st));
  const int64_t P = n_i * n_j;
  RowArgs rg{};
  rg.n_out = c_z;
  rg.bn = pick_bn(c_z, 16);
  rg.e_cols = n_j;
  rg.out = w.gate;
  rg.ldo = c_z;
  rg.act = 1;
  PF_TRY(rowgemm<E_STORE>(w.ln_g, c_z, P, c_z, p->w_g, c_z, rg, "k_rowgemm_gate", status, st));
  RowArgs ro{};
  ro.n_out = c_z;
  ro.bn = pick_bn(c_z, 16);
  ro.e_cols = n_j;
  ro.out = (__nv_bfloat16*)zo.ptr;
  ro.rs = zo.row_stride;
  ro.cs = zo.col_stride;
  ro.accumulate = acc;
  ro.gate = w.gate;
  ro.ldg = c_z;
  return rowgemm<E_RESID>(w.ln_x, c_h, P, c_h, p->w_z, c_z, ro, "k_rowgemm_resid", status, st);
}

bool same_view(const pf_pair_view& x, const pf_pair_view& y) {
  return x.ptr == y.ptr && x.row_stride == y.row_stride && x.col_stride == y.col_stride;
}

// ---------------------------------------------------------------- triangle attention
struct AttWs {
  __half *q, *k, *vt, *bias, *mb;
  __nv_bfloat16 *o, *g, *ln, *w;
  uint8_t *flags, *rowflags;
  int64_t ld_keys, ld_mb, n_tiles_k;
};
void att_plan(Arena& ar, int64_t n_rows, int64_t n_keys, int64_t n_q, int c, int H, bool own_bias, AttWs& w) {
  const int hd = H * RD;
  w.ld_keys = pad8(n_keys);
  w.n_tiles_k = (n_keys + 127) / 128;
  w.ld_mb = w.n_tiles_k * 128;
  w.q = ar.take<__half>((size_t)n_rows * hd * n_q);
  w.k = ar.take<__half>((size_t)n_rows * hd * w.ld_keys);
  w.vt = ar.take<__half>((size_t)n_rows * hd * w.ld_keys);
  w.bias = own_bias ? ar.take<__half>((size_t)H * n_q * w.ld_keys) : nullptr;
  w.o = ar.take<__nv_bfloat16>((size_t)n_rows * n_q * hd);
  w.g = ar.take<__nv_bfloat16>((size_t)n_rows * n_q * hd);
  w.ln = ar.take<__nv_bfloat16>((size_t)n_rows * n_keys * c);
  w.w = ar.take<__nv_bfloat16>((size_t)4 * hd * c);
  w.mb = ar.take<__half>((size_t)n_rows * w.ld_mb);
  w.flags = ar.take<uint8_t>((size_t)n_rows * w.n_tiles_k);
  w.rowflags = ar.take<uint8_t>((size_t)n_rows);
}

int head_bias(const __nv_bfloat16* ln, int64_t n_rows, int64_t n_cols, int c, const void* w_bias, int H,
              void* bias, int64_t hs, int64_t rs, bool f16, float scale, const char* name, unsigned int* status,
              cudaStream_t st) {
  RowArgs rb{};
  rb.n_out = 16;
  rb.bn = 16;
  rb.e_cols = n_cols;
  rb.heads = H;
  rb.bias = bias;
  rb.hs = hs;
  rb.bias_rs = rs;
  rb.bias_f16 = f16 ? 1 : 0;
  rb.bias_scale = scale;
  return rowgemm<E_HBIAS>(ln, c, n_rows * n_cols, c, w_bias, H, rb, name, status, st);
}

}  // namespace

// ================================================================== entry points (pf_tc.h)
bool rows_trimul_supported(int c_z, int c_h) {
  return c_z >= 8 && c_z % 8 == 0 && c_z <= 1024 && c_h >= 64 && c_h % 64 == 0 && c_h <= 512;
}
bool rows_triatt_supported(int c, int H, int d) {
  return c >= 8 && c % 8 == 0 && c <= 1024 && d == RD && H >= 1 && H <= 16 && (H * RD) % 128 == 0;
}
bool rows_bias_supported(int c, int H) { return c >= 8 && c % 8 == 0 && c <= 1024 && H >= 1 && H <= 16; }
bool rows_transition_supported(int c, int nm) {
  return c >= 8 && c % 8 == 0 && c <= 1024 && nm >= 1 && ((int64_t)nm * c) % 64 == 0 && (int64_t)nm * c <= 4096;
}

size_t rows_trimul_ws_bytes(int64_t n_i, int64_t n_j, int64_t n_k, int c_z, int c_h) {
  Arena ar(nullptr, 0);
  const int64_t ld_k = pad8(n_k);
  ar.take<__nv_bfloat16>((size_t)c_h * n_i * ld_k);
  ar.take<__nv_bfloat16>((size_t)c_h * n_j * ld_k);
  ProjWs pw;
  proj_plan(ar, n_i, n_j, n_k, false, c_z, c_h, pw);
  CombWs cw;
  comb_plan(ar, n_i, n_j, c_z, c_h, cw);
  return ar.used;
}

int rows_trimul(const pf_trimul_params* p, pf_pair_view za, pf_pair_view zb, pf_mask_view ma, pf_mask_view mb,
                pf_pair_view zg, pf_pair_view zo, int64_t n_i, int64_t n_j, int64_t n_k, int c_z, int c_h, int acc,
                void* ws, size_t ws_bytes, cudaStream_t st) {
  Arena ar(ws, ws_bytes);
  const int64_t ld_k = pad8(n_k);
  __nv_bfloat16* a = ar.take<__nv_bfloat16>((size_t)c_h * n_i * ld_k);
  __nv_bfloat16* b = ar.take<__nv_bfloat16>((size_t)c_h * n_j * ld_k);
  const bool same = same_view(za, zb) && n_i == n_j && (ma.ptr == mb.ptr) && ma.row_stride == mb.row_stride &&
                    ma.col_stride == mb.col_stride;
  ProjWs pw;
  proj_plan(ar, n_i, n_j, n_k, same, c_z, c_h, pw);
  CombWs cw;
  comb_plan(ar, n_i, n_j, c_z, c_h, cw);
  if (!ar.ok()) return fail(PF_EWORKSPACE, "trimul workspace too small");
  unsigned int* status;
  PF_TRY(device_status_ptr(&status));
  PF_TRY(proj_run(p, za, zb, ma, mb, n_i, n_j, n_k, c_z, c_h, a, b, ld_k, pw, status, st));
  return comb_run(p, a, b, ld_k, n_i, n_j, n_k, zg, zo, c_z, c_h, acc, cw, status, st);
}

size_t rows_trimul_project_ws_bytes(int64_t n_rows, int64_t n_cols, int c_z, int c_h) {
  Arena ar(nullptr, 0);
  ProjWs pw;
  proj_plan(ar, n_rows, n_rows, n_cols, true, c_z, c_h, pw);
  return ar.used;
}

int rows_trimul_project(const pf_trimul_params* p, pf_pair_view z, pf_mask_view m, int64_t n_rows, int64_t n_cols,
                        int c_z, int c_h, void* a, void* b, int64_t ld, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (!aligned16(a) || !aligned16(b) || ld % 8 || ld < n_cols)
    return fail(PF_EINVAL_SHAPE, "trimul project: channel-major outputs need 16-byte alignment and a pitch that is "
                "a multiple of 8 and >= n_cols");
  Arena ar(ws, ws_bytes);
  ProjWs pw;
  proj_plan(ar, n_rows, n_rows, n_cols, true, c_z, c_h, pw);
  if (!ar.ok()) return fail(PF_EWORKSPACE, "trimul project workspace too small");
  unsigned int* status;
  PF_TRY(device_status_ptr(&status));
  return proj_run(p, z, z, m, m, n_rows, n_rows, n_cols, c_z, c_h, (__nv_bfloat16*)a, (__nv_bfloat16*)b, ld, pw,
                  status, st);
}

size_t rows_trimul_combine_ws_bytes(int64_t n_i, int64_t n_j, int c_z, int c_h) {
  Arena ar(nullptr, 0);
  CombWs cw;
  comb_plan(ar, n_i, n_j, c_z, c_h, cw);
  return ar.used;
}

int rows_trimul_combine(const pf_trimul_params* p, const void* a, const void* b, int64_t ld, int64_t n_i,
                        int64_t n_j, int64_t n_k, pf_pair_view zg, pf_pair_view zo, int c_z, int c_h, int acc,
                        void* ws, size_t ws_bytes, cudaStream_t st) {
  if (!aligned16(a) || !aligned16(b) || ld % 8 || ld < n_k)
    return fail(PF_EINVAL_SHAPE, "trimul combine: channel-major operands need 16-byte alignment and a pitch that "
                "is a multiple of 8 and >= n_k");
  Arena ar(ws, ws_bytes);
  CombWs cw;
  comb_plan(ar, n_i, n_j, c_z, c_h, cw);
  if (!ar.ok()) return fail(PF_EWORKSPACE, "trimul combine workspace too small");
  unsigned int* status;
  PF_TRY(device_status_ptr(&status));
  return comb_run(p, (const __nv_bfloat16*)a, (const __nv_bfloat16*)b, ld, n_i, n_j, n_k, zg, zo, c_z, c_h, acc, cw,
                  status, st);
}

size_t rows_triatt_ws_bytes(int64_t n_rows, int64_t n_keys, int64_t n_q, int c, int H) {
  Arena ar(nullptr, 0);
  AttWs w;
  att_plan(ar, n_rows, n_keys, n_q, c, H, true, w);
  return ar.used;
}

int rows_triatt(const pf_triatt_params* p, pf_pair_view zs, pf_mask_view m, const void* bias, int64_t b_hs,
                int64_t b_rs, pf_pair_view zo, int64_t n_rows, int64_t n_keys, int64_t n_valid, int64_t q_col0,
                int64_t n_q, int c, int H, float inf, int acc, void* ws, size_t ws_bytes, cudaStream_t st) {
  Arena ar(ws, ws_bytes);
  AttWs w;
  att_plan(ar, n_rows, n_keys, n_q, c, H, bias == nullptr, w);
  if (!ar.ok()) return fail(PF_EWORKSPACE, "triatt workspace too small");
  PF_TRY(check_view(zs, "triatt zs"));
  PF_TRY(check_view(zo, "triatt zo"));
  const int hd = H * RD;
  unsigned int* status;
  PF_TRY(device_status_ptr(&status));
  CoreIO io{w.q, w.k, w.vt, bias, b_hs, b_rs, w.o, w.mb, w.flags, w.rowflags, w.ld_keys, w.ld_mb, w.n_tiles_k};
  PF_TRY(triatt_masks(m, n_rows, n_keys, n_valid, inf, io, st));
  PF_TRY(ln_pos((const __nv_bfloat16*)zs.ptr, zs.row_stride, zs.col_stride, n_rows, n_keys, c, p->ln_w, p->ln_b,
                w.ln, st));
  const void* srcs[4] = {p->w_q, p->w_k, p->w_v, p->w_g};
  PF_TRY(pack_w(srcs, 1, 0, hd, c, 4 * (int64_t)hd, w.w, st));
  RowArgs rq{};
  rq.n_out = 4 * hd;
  rq.bn = 128;
  rq.e_cols = n_keys;
  rq.q = w.q;
  rq.k = w.k;
  rq.vt = w.vt;
  rq.g = w.g;
  rq.heads = H;
  rq.n_q = n_q;
  rq.q_col0 = q_col0;
  rq.ld_keys = w.ld_keys;
  rq.q_scale = LOG2E_R / sqrtf((float)RD);
  PF_TRY(rowgemm<E_QKVG>(w.ln, c, n_rows * n_keys, c, w.w, 4 * hd, rq, "k_rowgemm_qkvg", status, st));
  if (bias == nullptr) {
    // the square single-device case: bias(h, j, key) from the same LayerNorm'd rows
    io.bias = w.bias;
    io.b_hs = n_q * w.ld_keys;
    io.b_rs = w.ld_keys;
    PF_TRY(head_bias(w.ln, n_rows, n_keys, c, p->w_bias, H, w.bias, io.b_hs, io.b_rs, true, LOG2E_R,
                     "k_rowgemm_bias", status, st));
  }
  PF_TRY(triatt_core(io, n_rows, n_keys, n_valid, n_q, H, status, st));
  PF_TRY(gate_mul(w.o, w.g, n_rows * n_q * hd, st));
  RowArgs ro{};
  ro.n_out = c;
  ro.bn = pick_bn(c, 16);
  ro.e_cols = n_q;
  ro.out = (__nv_bfloat16*)zo.ptr;
  ro.rs = zo.row_stride;
  ro.cs = zo.col_stride;
  ro.accumulate = acc;
  return rowgemm<E_RESID>(w.o, hd, n_rows * n_q, hd, p->w_o, c, ro, "k_rowgemm_resid", status, st);
}

size_t rows_bias_ws_bytes(int64_t n_rows, int64_t n_cols, int c) {
  return align_up((size_t)n_rows * n_cols * c * 2, 256);
}

// bias(h, r, s) of the triangle attention (f16, log2 units) or of AttentionPairBias (fp32)
int rows_head_bias(const float* ln_w, const float* ln_b, const void* w_bias, pf_pair_view z, int64_t n_rows,
                   int64_t n_cols, int c, int H, void* bias, int64_t hs, int64_t rs, bool f16_log2, void* ws,
                   size_t ws_bytes, cudaStream_t st) {
  if (ws_bytes < rows_bias_ws_bytes(n_rows, n_cols, c)) return fail(PF_EWORKSPACE, "bias workspace too small");
  PF_TRY(check_view(z, "bias z"));
  unsigned int* status;
  PF_TRY(device_status_ptr(&status));
  __nv_bfloat16* ln = (__nv_bfloat16*)ws;
  PF_TRY(ln_pos((const __nv_bfloat16*)z.ptr, z.row_stride, z.col_stride, n_rows, n_cols, c, ln_w, ln_b, ln, st));
  return head_bias(ln, n_rows, n_cols, c, w_bias, H, bias, hs, rs, f16_log2, f16_log2 ? LOG2E_R : 1.f,
                   f16_log2 ? "k_rowgemm_bias" : "k_rowgemm_apb_bias", status, st);
}

size_t rows_transition_ws_bytes(int64_t rows, int c, int nm) {
  Arena ar(nullptr, 0);
  ar.take<__nv_bfloat16>((size_t)rows * c);
  ar.take<__nv_bfloat16>((size_t)rows * nm * c);
  ar.take<__nv_bfloat16>((size_t)2 * nm * c * c);
  return ar.used;
}

int rows_transition(const pf_transition_params* p, const void* x, int64_t xs, void* out, int64_t os, int64_t rows,
                    int c, int nm, int acc, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (!aligned16(x) || !aligned16(out) || xs % 8 || os % 8)
    return fail(PF_EINVAL_SHAPE, "bf16 transition rows must be 16-byte aligned (row strides multiple of 8)");
  Arena ar(ws, ws_bytes);
  const int hid = nm * c;
  __nv_bfloat16* ln = ar.take<__nv_bfloat16>((size_t)rows * c);
  __nv_bfloat16* h = ar.take<__nv_bfloat16>((size_t)rows * hid);
  __nv_bfloat16* w = ar.take<__nv_bfloat16>((size_t)2 * hid * c);
  if (!ar.ok()) return fail(PF_EWORKSPACE, "transition workspace too small");
  unsigned int* status;
  PF_TRY(device_status_ptr(&status));
  PF_TRY(ln_pos((const __nv_bfloat16*)x, 0, xs, 1, rows, c, p->ln_w, p->ln_b, ln, st));
  // [a | b] interleaved per 64 hidden units: 2 * hid rows
  const void* srcs[4] = {p->w_a, p->w_b, nullptr, nullptr};
  const int64_t w_rows = 2 * (int64_t)hid;
  PF_TRY(pack_w(srcs, 0, hid / 64, 0, c, w_rows, w, st));
  RowArgs rs{};
  rs.n_out = (int)w_rows;
  rs.bn = w_rows % 256 == 0 ? 256 : 128;
  rs.e_cols = rows;
  rs.out = h;
  rs.ldo = hid;
  PF_TRY(rowgemm<E_SWIGLU>(ln, c, rows, c, w, (int)w_rows, rs, "k_rowgemm_swiglu", status, st));
  RowArgs ro{};
  ro.n_out = c;
  ro.bn = pick_bn(c, 16);
  ro.e_cols = rows;
  ro.out = (__nv_bfloat16*)out;
  ro.rs = 0;
  ro.cs = os;
  ro.accumulate = acc;
  return rowgemm<E_RESID>(h, hid, rows, hid, p->w_o, c, ro, "k_rowgemm_resid", status, st);
}

// ---------------------------------------------------------------- pair LN + linear (recycling)
bool rows_pair_ln_linear_supported(int c_in, int c_out) {
  return c_in >= 8 && c_in % 8 == 0 && c_in <= 1024 && c_out >= 8 && c_out % 8 == 0 && c_out <= 1024;
}

size_t rows_pair_ln_linear_ws_bytes(int64_t n_rows, int64_t n_cols, int c_in) {
  return align_up((size_t)n_rows * n_cols * c_in * 2, 256);
}

int rows_pair_ln_linear(const pf_pair_linear_params* p, pf_pair_view zi, pf_pair_view zo, int64_t n_rows,
                        int64_t n_cols, int c_in, int c_out, int acc, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (ws_bytes < rows_pair_ln_linear_ws_bytes(n_rows, n_cols, c_in))
    return fail(PF_EWORKSPACE, "pair LN-linear workspace too small");
  PF_TRY(check_view(zi, "pair LN-linear z_in"));
  PF_TRY(check_view(zo, "pair LN-linear z_out"));
  unsigned int* status;
  PF_TRY(device_status_ptr(&status));
  __nv_bfloat16* ln = (__nv_bfloat16*)ws;
  PF_TRY(ln_pos((const __nv_bfloat16*)zi.ptr, zi.row_stride, zi.col_stride, n_rows, n_cols, c_in, p->ln_w, p->ln_b,
                ln, st));
  RowArgs ro{};
  ro.n_out = c_out;
  ro.bn = pick_bn(c_out, 16);
  ro.e_cols = n_cols;
  ro.out = (__nv_bfloat16*)zo.ptr;
  ro.rs = zo.row_stride;
  ro.cs = zo.col_stride;
  ro.accumulate = acc;
  return rowgemm<E_RESID>(ln, c_in, n_rows * n_cols, c_in, p->w, c_out, ro, "k_rowgemm_resid", status, st);
}

// ---------------------------------------------------------------- pair heads
bool rows_pair_head_supported(int c_z, int n_bins) {
  return c_z >= 8 && c_z % 8 == 0 && c_z <= 1024 && n_bins >= 1 && n_bins <= RB_NMAX;
}

size_t rows_pair_head_ws_bytes(int64_t n_rows, int64_t n_cols, int c_z) {
  return align_up((size_t)n_rows * n_cols * c_z * 2, 256);
}

// A = LN(z) / LN(z + zt) / (z + zt) per position (k_ln_pos), then logits = A W^T + s b with the
// softmax contact sum in the epilogue (k_rowgemm<E_HEAD>, one output tile of <= 256 bins).
int rows_pair_head(const pf_pair_head_params* p, int mode, pf_pair_view z, pf_pair_view zt, int64_t n_rows,
                   int64_t n_cols, int c_z, int n_bins, pf_pair_view lo, int lo_f32, float* contact,
                   int64_t contact_rs, int64_t contact_cs, int contact_bins, void* ws, size_t ws_bytes,
                   cudaStream_t st) {
  if (ws_bytes < rows_pair_head_ws_bytes(n_rows, n_cols, c_z)) return fail(PF_EWORKSPACE, "pair head workspace too small");
  PF_TRY(check_view(z, "pair head z"));
  if (mode != PF_HEAD_PLAIN) PF_TRY(check_view(zt, "pair head zt"));
  unsigned int* status;
  PF_TRY(device_status_ptr(&status));
  __nv_bfloat16* a = (__nv_bfloat16*)ws;
  const bool sym = mode != PF_HEAD_PLAIN;
  PF_TRY(ln_pos2((const __nv_bfloat16*)z.ptr, z.row_stride, z.col_stride, sym ? (const __nv_bfloat16*)zt.ptr : nullptr,
                 zt.row_stride, zt.col_stride, mode != PF_HEAD_SYM_OUT, n_rows, n_cols, c_z, p->ln_w, p->ln_b, a, st));
  RowArgs ro{};
  ro.n_out = n_bins;
  ro.bn = pick_bn(n_bins, 16);
  ro.e_cols = n_cols;
  ro.rs = lo.row_stride;
  ro.cs = lo.col_stride;
  if (lo_f32)
    ro.outf = (float*)lo.ptr;
  else
    ro.out = (__nv_bfloat16*)lo.ptr;
  ro.colbias = p->b;
  ro.n_colbias = p->b ? n_bins : 0;
  ro.bias_scale = mode == PF_HEAD_SYM_OUT ? 2.f : 1.f;
  ro.contact = contact;
  ro.contact_rs = contact_rs;
  ro.contact_cs = contact_cs;
  ro.contact_bins = contact_bins;
  return rowgemm<E_HEAD>(a, c_z, n_rows * n_cols, c_z, p->w, n_bins, ro, "k_rowgemm_head", status, st);
}

// ---------------------------------------------------------------- OuterProductMean
bool rows_opm_supported(int c_m, int c_hidden, int c_z) {
  return c_m >= 8 && c_m % 8 == 0 && c_m <= 1024 && c_hidden == 32 && c_z >= 8 && c_z % 8 == 0 && c_z <= 1024;
}

namespace {
struct OpmWs {
  __nv_bfloat16 *ln, *at, *bt, *x;
  float* norm;
  int64_t ld_s, ld_x;
};
void opm_plan(Arena& ar, int64_t S, int64_t N, int64_t nr, int64_t nc, int c_m, int C, bool masked, OpmWs& w) {
  w.ld_s = pad8(S);
  w.ld_x = pad8(nc * C);
  w.ln = ar.take<__nv_bfloat16>((size_t)N * S * c_m);
  w.at = ar.take<__nv_bfloat16>((size_t)nr * C * w.ld_s);
  w.bt = ar.take<__nv_bfloat16>((size_t)nc * C * w.ld_s);
  w.x = ar.take<__nv_bfloat16>((size_t)nr * C * w.ld_x);
  w.norm = masked ? ar.take<float>((size_t)nr * nc) : nullptr;
}
}  // namespace

size_t rows_opm_ws_bytes(int64_t n_seq, int64_t n_res, int64_t n_rows, int64_t n_cols, int c_m, int C) {
  Arena ar(nullptr, 0);
  OpmWs w;
  opm_plan(ar, n_seq, n_res, n_rows, n_cols, c_m, C, true, w);
  return ar.used;
}

int rows_opm(const pf_opm_params* p, pf_pair_view m, pf_mask_view mask, pf_pair_view z_out, int64_t S, int64_t N,
             int64_t row0, int64_t nr, int64_t col0, int64_t nc, int c_m, int C, int c_z, float eps, int acc,
             void* ws, size_t ws_bytes, cudaStream_t st) {
  PF_TRY(check_view(m, "opm m"));
  PF_TRY(check_view(z_out, "opm z_out"));
  Arena ar(ws, ws_bytes);
  OpmWs w;
  opm_plan(ar, S, N, nr, nc, c_m, C, mask.ptr != nullptr, w);
  if (!ar.ok()) return fail(PF_EWORKSPACE, "OuterProductMean workspace too small");
  unsigned int* status;
  PF_TRY(device_status_ptr(&status));
  // LN of every position in (i, s) order: a residue's sequences are contiguous rows
  PF_TRY(ln_pos((const __nv_bfloat16*)m.ptr, m.col_stride, m.row_stride, N, S, c_m, p->ln_w, p->ln_b, w.ln, st));
  // aT[(i*C + c)*ld_s + s] = mask(s, row0 + i) * linear_1(ln(s, row0 + i))[c]; bT likewise
  RowArgs ra{};
  ra.n_out = C;
  ra.bn = C;
  ra.e_cols = S;
  ra.ld = w.ld_s;
  ra.dst[0] = w.at;
  ra.mask = pf_mask_view{mask.ptr ? mask.ptr + row0 * mask.col_stride : nullptr, mask.col_stride, mask.row_stride};
  PF_TRY(rowgemm<E_OPMAB>(w.ln + row0 * S * c_m, c_m, nr * S, c_m, p->w_1, C, ra, "k_rowgemm_opm_ab", status, st));
  ra.dst[0] = w.bt;
  ra.mask = pf_mask_view{mask.ptr ? mask.ptr + col0 * mask.col_stride : nullptr, mask.col_stride, mask.row_stride};
  PF_TRY(rowgemm<E_OPMAB>(w.ln + col0 * S * c_m, c_m, nc * S, c_m, p->w_2, C, ra, "k_rowgemm_opm_ab", status, st));
  // x[(i, c)][(j, e)] = sum_s aT[(i, c)][s] bT[(j, e)][s]: one channel of the per-channel contraction
  PF_TRY(trimul_contract(w.at, w.ld_s, w.bt, w.ld_s, nr * C, nc * C, S, 1, w.x, w.ld_x, status, st));
  if (mask.ptr) PF_TRY(simt::opm_norm(mask, S, row0, nr, col0, nc, eps, w.norm, st));
  RowArgs ro{};
  ro.n_out = c_z;
  ro.bn = pick_bn(c_z, 16);
  ro.out = (__nv_bfloat16*)z_out.ptr;
  ro.rs = z_out.row_stride;
  ro.cs = z_out.col_stride;
  ro.accumulate = acc;
  ro.colbias = p->b_out;
  ro.divide = 1;
  ro.rownorm = w.norm;
  ro.norm_const = (float)S + eps;
  return rowgemm_outer(w.x, w.ld_x, nr, nc, C, p->w_out, c_z, ro, "k_rowgemm_opm_out", status, st);
}

// ---------------------------------------------------------------- AttentionPairBias, single path
bool rows_apb_supported(int c_s, int H) {
  if (c_s < 8 || c_s % 8 || c_s > 1024 || H < 1 || c_s % H) return false;
  const int d = c_s / H;
  return d == 8 || d == 16 || d == 24 || d == 32 || d == 48 || d == 64;
}

size_t rows_apb_ws_bytes(int64_t n, int64_t nq, int c_s, int H) {
  Arena ar(nullptr, 0);
  ar.take<__nv_bfloat16>((size_t)n * c_s);           // LN_a(s)
  ar.take<__nv_bfloat16>((size_t)2 * c_s * c_s);     // [W_k; W_v]
  ar.take<__nv_bfloat16>((size_t)2 * c_s * c_s);     // [W_q; W_g]
  ar.take<float>((size_t)n * 2 * c_s);               // [k | v]
  ar.take<float>((size_t)nq * 2 * c_s);              // [q | g]
  ar.take<float>((size_t)nq * c_s);                  // o
  ar.take<__nv_bfloat16>((size_t)nq * c_s);          // o * sigmoid(g)
  ar.take<float>(simt::attn_split_part_floats(n, nq, c_s, H));
  return ar.used;
}

int rows_apb(const pf_apb_params* p, const void* s_in, void* s_out, const float* bias, int64_t b_hs, int64_t b_rs,
             int64_t n, int64_t q0, int64_t nq, int c_s, int H, int acc, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (!aligned16(s_in) || !aligned16(s_out)) return fail(PF_EINVAL_SHAPE, "apb: s must be 16-byte aligned");
  Arena ar(ws, ws_bytes);
  __nv_bfloat16* a = ar.take<__nv_bfloat16>((size_t)n * c_s);
  __nv_bfloat16* wkv = ar.take<__nv_bfloat16>((size_t)2 * c_s * c_s);
  __nv_bfloat16* wqg = ar.take<__nv_bfloat16>((size_t)2 * c_s * c_s);
  float* kv = ar.take<float>((size_t)n * 2 * c_s);
  float* qg = ar.take<float>((size_t)nq * 2 * c_s);
  float* o = ar.take<float>((size_t)nq * c_s);
  __nv_bfloat16* ob = ar.take<__nv_bfloat16>((size_t)nq * c_s);
  float* part = ar.take<float>(simt::attn_split_part_floats(n, nq, c_s, H));
  if (!ar.ok()) return fail(PF_EWORKSPACE, "apb workspace too small");
  unsigned int* status;
  PF_TRY(device_status_ptr(&status));
  // keys / values from LN_a(s) of all n rows; queries, gate and output for rows [q0, q0 + nq)
  PF_TRY(ln_pos((const __nv_bfloat16*)s_in, 0, c_s, 1, n, c_s, p->ln_a_w, p->ln_a_b, a, st));
  const void* kvsrc[4] = {p->w_k, p->w_v, nullptr, nullptr};
  PF_TRY(pack_w(kvsrc, 1, 0, c_s, c_s, 2 * (int64_t)c_s, wkv, st));
  const void* qgsrc[4] = {p->w_q, p->w_g, nullptr, nullptr};
  PF_TRY(pack_w(qgsrc, 1, 0, c_s, c_s, 2 * (int64_t)c_s, wqg, st));
  RowArgs rk{};
  rk.n_out = 2 * c_s;
  rk.bn = pick_bn(2 * c_s, 16);
  rk.e_cols = n;
  rk.outf = kv;
  rk.ldo = 2 * c_s;
  PF_TRY(rowgemm<E_STOREF>(a, c_s, n, c_s, wkv, 2 * c_s, rk, "k_rowgemm_single", status, st));
  RowArgs rq = rk;
  rq.e_cols = nq;
  rq.outf = qg;
  rq.colbias = p->b_q;
  rq.n_colbias = p->b_q ? c_s : 0;
  PF_TRY(rowgemm<E_STOREF>(a + q0 * c_s, c_s, nq, c_s, wqg, 2 * c_s, rq, "k_rowgemm_single", status, st));
  PF_TRY(simt::attn_split(c_s / H, qg, 2 * c_s, kv, kv + c_s, 2 * c_s, bias, b_hs, b_rs, nq, n, H, part, o, c_s,
                          st));
  {
    PF_LAUNCH_SCOPE(st, "k_gate_f32_bf16");
    k_gate_f32_bf16<<<(unsigned)((nq * c_s + 255) / 256), 256, 0, st>>>(o, qg + c_s, 2 * c_s, nq, c_s, ob);
  }
  PF_CHECK_LAUNCH();
  RowArgs ro{};
  ro.n_out = c_s;
  ro.bn = pick_bn(c_s, 16);
  ro.e_cols = nq;
  ro.out = (__nv_bfloat16*)s_out;
  ro.rs = 0;
  ro.cs = c_s;
  ro.accumulate = acc;
  return rowgemm<E_RESID>(ob, c_s, nq, c_s, p->w_o, c_s, ro, "k_rowgemm_resid", status, st);
}

}  // namespace tc
}  // namespace pf
