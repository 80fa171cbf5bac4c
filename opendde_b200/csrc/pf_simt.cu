// pf_simt.cu -- generic SIMT (FFMA) path of the pair stack.
//
// Serves two purposes:
//  * the fp32 mode (PF_F32): fp32 storage and fp32 arithmetic, evaluated in the same
//    operation order as the reference PyTorch modules so that the 1e-4 max-abs parity
//    holds (no TF32 anywhere);
//  * any shape the tcgen05 path does not cover (channel counts other than the tuned
//    ones), in either dtype. Intermediates are fp32 in the caller's workspace.
//
// Every op is a short sequence of: a LayerNorm-of-a-view kernel, a strided batched
// C = A * B^T GEMM, and small elementwise kernels.

#include <cmath>

#include "pf_common.cuh"
#include "pf_prof.h"
#include "pf_simt.h"

namespace pf {
namespace simt {

// ============================================================================ kernels

// LayerNorm over channels of every position (r, s) of a pair view -> contiguous output
// out[(r*n_cols + s) * c + ch]. One warp per position; two-pass (mean, then centred
// variance) like torch's CPU layer_norm.
template <class T, class TO>
__global__ void k_ln_view(const T* __restrict__ x, int64_t rs, int64_t cs, int64_t n_rows,
                          int64_t n_cols, int c, const float* __restrict__ gamma,
                          const float* __restrict__ beta, float eps, TO* __restrict__ out,
                          int64_t out_pos_stride) {
  const int lane = threadIdx.x & 31;
  const int64_t pos = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t npos = n_rows * n_cols;
  if (pos >= npos) return;
  const int64_t r = pos / n_cols, s = pos - r * n_cols;
  const T* xp = x + r * rs + s * cs;
  constexpr int MAXV = 32;  // c <= 1024
  float v[MAXV];
  float sum = 0.f;
  const int per = (c + 31) / 32;
#pragma unroll
  for (int t = 0; t < MAXV; ++t) {
    if (t < per) {
      int ch = t * 32 + lane;
      v[t] = ch < c ? to_f(xp[ch]) : 0.f;
      sum += v[t];
    }
  }
  const float mean = warp_sum(sum) / (float)c;
  float sq = 0.f;
#pragma unroll
  for (int t = 0; t < MAXV; ++t) {
    if (t < per) {
      int ch = t * 32 + lane;
      float d = ch < c ? v[t] - mean : 0.f;
      sq += d * d;
    }
  }
  const float var = warp_sum(sq) / (float)c;
  const float rstd = 1.0f / sqrtf(var + eps);
  TO* op = out + pos * out_pos_stride;
#pragma unroll
  for (int t = 0; t < MAXV; ++t) {
    if (t < per) {
      int ch = t * 32 + lane;
      if (ch < c) {
        float y = (v[t] - mean) * rstd;
        if (gamma) y = y * gamma[ch];
        if (beta) y = y + beta[ch];
        op[ch] = from_f<TO>(y);
      }
    }
  }
}

// Standalone LayerNorm of contiguous rows with 128-bit accesses: each row is read and written
// as 16-byte vectors (8 bf16 or 4 fp32 channels), L = 2^k <= 32 lanes per row (the largest
// power of two not above the row's vector count), 32 / L rows per warp; the row stays in
// registers between the two statistics passes (mean, then centred variance) and the output
// pass, so x is read from HBM once. Requires c * sizeof(T) % 16 == 0 and 16-byte aligned
// pointers (checked by the host).
template <class T>
struct VecTraits;
template <>
struct VecTraits<float> {
  static constexpr int E = 4;
  __device__ static void unpack(const uint4& u, float (&f)[4]) {
    f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y); f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
  }
  __device__ static uint4 pack(const float (&f)[4]) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
  }
};
template <>
struct VecTraits<__nv_bfloat16> {
  static constexpr int E = 8;
  __device__ static void unpack(const uint4& u, float (&f)[8]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  }
  __device__ static uint4 pack(const float (&f)[8]) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 v = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&v);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
};

template <class T, int L>
__global__ void __launch_bounds__(256) k_layernorm_rows(const T* __restrict__ x, T* __restrict__ y, int64_t rows,
                                                        int c, const float* __restrict__ gamma,
                                                        const float* __restrict__ beta, float eps) {
  constexpr int E = VecTraits<T>::E;
  // vectors per lane: L < 32 is chosen only for rows of fewer than 2L vectors; L = 32 up to c = 1024
  constexpr int MAXV = L < 32 ? 2 : (1024 / E) / 32;
  const int lane = threadIdx.x & 31;
  const int sub = lane & (L - 1);
  const int64_t row = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * (32 / L) + lane / L;
  const bool live = row < rows;
  const int nv = c / E;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (live ? row : 0) * (int64_t)c);
  uint4 raw[MAXV];
#pragma unroll
  for (int t = 0; t < MAXV; ++t) {
    const int v = sub + t * L;
    raw[t] = (live && v < nv) ? __ldg(xr + v) : make_uint4(0, 0, 0, 0);
  }
  float sum = 0.f;
#pragma unroll
  for (int t = 0; t < MAXV; ++t) {
    float f[E];
    VecTraits<T>::unpack(raw[t], f);
#pragma unroll
    for (int e = 0; e < E; ++e) sum += f[e];
  }
#pragma unroll
  for (int o = L / 2; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float mean = sum / (float)c;
  float sq = 0.f;
#pragma unroll
  for (int t = 0; t < MAXV; ++t) {
    if (sub + t * L < nv) {
      float f[E];
      VecTraits<T>::unpack(raw[t], f);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const float d = f[e] - mean;
        sq += d * d;
      }
    }
  }
#pragma unroll
  for (int o = L / 2; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  const float rstd = rsqrtf(sq / (float)c + eps);
  if (!live) return;
  uint4* yr = reinterpret_cast<uint4*>(y + row * (int64_t)c);
#pragma unroll
  for (int t = 0; t < MAXV; ++t) {
    const int v = sub + t * L;
    if (v < nv) {
      float f[E];
      VecTraits<T>::unpack(raw[t], f);
      const int ch0 = v * E;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        float o = (f[e] - mean) * rstd;
        if (gamma) o *= __ldg(gamma + ch0 + e);
        if (beta) o += __ldg(beta + ch0 + e);
        f[e] = o;
      }
      yr[v] = VecTraits<T>::pack(f);
    }
  }
}

// C[b](m, n) = alpha * sum_k A[b](m, k) * B[b](n, k)  (+ C if accumulate)
// A(m,k) = A + b*sAb + m*sAm + k ; B(n,k) = B + b*sBb + n*sBn + k ;
// C(m,n) = C + b*sCb + m*sCm + n*sCn.
// 64x64 tile, K step 16, 256 threads, 4x4 outputs per thread, fp32 FFMA.
template <class TA, class TB>
__global__ void __launch_bounds__(256) k_gemm_nt(const TA* __restrict__ A, int64_t sAb, int64_t sAm,
                                                 const TB* __restrict__ B, int64_t sBb, int64_t sBn,
                                                 float* __restrict__ C, int64_t sCb, int64_t sCm,
                                                 int64_t sCn, int64_t M, int64_t N, int64_t K,
                                                 float alpha, int accumulate) {
  __shared__ float As[16][64 + 4];
  __shared__ float Bs[16][64 + 4];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t b = blockIdx.z;
  const int64_t m0 = (int64_t)blockIdx.y * 64, n0 = (int64_t)blockIdx.x * 64;
  const TA* Ab = A + b * sAb;
  const TB* Bb = B + b * sBb;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  for (int64_t k0 = 0; k0 < K; k0 += 16) {
    // each thread loads 4 elements of A tile and 4 of B tile (64 rows x 16 k)
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      int idx = tid + t * 256;   // 0..1023
      int row = idx >> 4, kk = idx & 15;
      int64_t gm = m0 + row, gk = k0 + kk, gn = n0 + row;
      As[kk][row] = (gm < M && gk < K) ? to_f(Ab[gm * sAm + gk]) : 0.f;
      Bs[kk][row] = (gn < N && gk < K) ? to_f(Bb[gn * sBn + gk]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float a[4], bb[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bb[j] = Bs[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], bb[j], acc[i][j]);
    }
    __syncthreads();
  }
  float* Cb = C + b * sCb;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int64_t gm = m0 + ty + 16 * i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int64_t gn = n0 + tx + 16 * j;
      if (gn >= N) continue;
      float* cp = Cb + gm * sCm + gn * sCn;
      float val = alpha * acc[i][j];
      *cp = accumulate ? (*cp + val) : val;
    }
  }
}

// a(ch, r, k) = m(r, k) * sigmoid(pg[p, ch]) * pa[p, ch],  p = r*n_k + k  (channel-major out,
// element (ch, r, k) at out[(ch * n_r + r) * ld + k])
template <class TO>
__global__ void k_gate_to_cmajor(const float* __restrict__ pa, const float* __restrict__ pg,
                                 pf_mask_view m, int64_t n_r, int64_t n_k, int c_h,
                                 TO* __restrict__ out, int64_t ld) {
  const int64_t P = n_r * n_k;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= P * c_h) return;
  const int64_t ch = idx / P, p = idx - ch * P;
  const int64_t r = p / n_k, k = p - r * n_k;
  const float mv = m.ptr ? m.ptr[r * m.row_stride + k * m.col_stride] : 1.0f;
  // reference order: a = mask; a = a * sigmoid(g); a = a * p   (triangular.py:539-541)
  float v = mv * sigmoid_acc(pg[p * c_h + ch]);
  out[(ch * n_r + r) * ld + k] = from_f<TO>(v * pa[p * c_h + ch]);
}

// x[p, ch] = LN_out over ch of p_cm[ch, p]   (channel-major input, one warp per position)
__global__ void k_ln_cmajor(const float* __restrict__ pin, int64_t P, int c,
                            const float* __restrict__ gamma, const float* __restrict__ beta,
                            float eps, float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t pos = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (pos >= P) return;
  constexpr int MAXV = 32;
  float v[MAXV];
  const int per = (c + 31) / 32;
  float sum = 0.f;
#pragma unroll
  for (int t = 0; t < MAXV; ++t)
    if (t < per) {
      int ch = t * 32 + lane;
      v[t] = ch < c ? pin[(int64_t)ch * P + pos] : 0.f;
      sum += v[t];
    }
  const float mean = warp_sum(sum) / (float)c;
  float sq = 0.f;
#pragma unroll
  for (int t = 0; t < MAXV; ++t)
    if (t < per) {
      int ch = t * 32 + lane;
      float d = ch < c ? v[t] - mean : 0.f;
      sq += d * d;
    }
  const float rstd = 1.0f / sqrtf(warp_sum(sq) / (float)c + eps);
#pragma unroll
  for (int t = 0; t < MAXV; ++t)
    if (t < per) {
      int ch = t * 32 + lane;
      if (ch < c) {
        float y = (v[t] - mean) * rstd;
        if (gamma) y *= gamma[ch];
        if (beta) y += beta[ch];
        out[pos * c + ch] = y;
      }
    }
}

// dst(r, s, ch) = acc ? dst + y*sig(g) : y*sig(g) for positions of a view;
// y, g are contiguous [P, c]; g == nullptr => no gate.
template <class T>
__global__ void k_combine_view(T* __restrict__ dst, int64_t rs, int64_t cs, int64_t n_rows,
                               int64_t n_cols, int c, const float* __restrict__ y,
                               const float* __restrict__ g, int accumulate) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t P = n_rows * n_cols;
  if (idx >= P * c) return;
  const int64_t p = idx / c;
  const int ch = (int)(idx - p * c);
  const int64_t r = p / n_cols, s = p - r * n_cols;
  float u = y[idx];
  if (g) u = u * sigmoid_acc(g[idx]);
  T* d = dst + r * rs + s * cs + ch;
  float base = accumulate ? to_f(*d) : 0.f;
  *d = from_f<T>(base + u);
}

// o *= sigmoid(g), contiguous
__global__ void k_gate_inplace(float* __restrict__ o, const float* __restrict__ g, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) o[i] = o[i] * sigmoid_acc(g[i]);
}

// h = silu(a) * b, contiguous (reference: a = silu(a); b *= a, primitives.py:205-210)
__global__ void k_swiglu(const float* __restrict__ a, float* __restrict__ b, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) b[i] = b[i] * silu_acc(a[i]);
}

// y += bias[col] for a row-major [rows, cols] matrix
__global__ void k_add_bias(float* __restrict__ y, const float* __restrict__ bias, int64_t rows, int cols) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < rows * cols) y[i] += bias[i % cols];
}

// Online-softmax attention, one thread per query. Arithmetic order follows the
// reference: s = (q / sqrt(d)) . k ; s += mask_bias ; s += bias ; softmax ; @ v.
//   q(i, j)  = q + i*q_rs + (q_col0 + j)*q_ps + h*D      (projection, unscaled)
//   k,v(i,k) = k + i*kv_rs + k*kv_ps + h*D
//   bias(h, j, k) = bias[h*b_hs + j*b_rs + k] * bias_scale    (nullptr => 0)
//   mask(i, k): mask_bias = inf * (mask - 1)                   (ptr == nullptr => 0)
template <int D, class TB>
__global__ void __launch_bounds__(64) k_attn_simt(
    const float* __restrict__ q, int64_t q_rs, int64_t q_ps, int64_t q_col0,
    const float* __restrict__ k, const float* __restrict__ v, int64_t kv_rs, int64_t kv_ps,
    const TB* __restrict__ bias, int64_t b_hs, int64_t b_rs, float bias_scale,
    pf_mask_view m, float inf, int64_t n_q, int64_t n_valid_keys, float inv_sqrt_d_div,
    float* __restrict__ o, int64_t o_rs, int64_t o_ps) {
  __shared__ float Ks[64][D + 1];
  __shared__ float Vs[64][D + 1];
  const int h = blockIdx.y;
  const int64_t i = blockIdx.z;
  const int64_t j = (int64_t)blockIdx.x * 64 + threadIdx.x;
  const bool active = j < n_q;
  float qv[D];
  const float* qp = q + i * q_rs + (q_col0 + (active ? j : 0)) * q_ps + h * D;
#pragma unroll
  for (int t = 0; t < D; ++t) qv[t] = qp[t] / inv_sqrt_d_div;  // reference divides q by sqrt(d)
  float mrun = -INFINITY, l = 0.f;
  float acc[D];
#pragma unroll
  for (int t = 0; t < D; ++t) acc[t] = 0.f;
  const float* kb = k + i * kv_rs + h * D;
  const float* vb = v + i * kv_rs + h * D;
  for (int64_t k0 = 0; k0 < n_valid_keys; k0 += 64) {
    __syncthreads();
    {
      int64_t kk = k0 + threadIdx.x;
      if (kk < n_valid_keys) {
#pragma unroll
        for (int t = 0; t < D; ++t) {
          Ks[threadIdx.x][t] = kb[kk * kv_ps + t];
          Vs[threadIdx.x][t] = vb[kk * kv_ps + t];
        }
      }
    }
    __syncthreads();
    if (!active) continue;
    const int64_t rem = n_valid_keys - k0;
    const int nk = rem < 64 ? (int)rem : 64;
    for (int t = 0; t < nk; ++t) {
      const int64_t kk = k0 + t;
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < D; ++e) s = fmaf(qv[e], Ks[t][e], s);
      if (m.ptr) s = s + inf * (m.ptr[i * m.row_stride + kk * m.col_stride] - 1.0f);
      if (bias) s = s + to_f(bias[(int64_t)h * b_hs + j * b_rs + kk]) * bias_scale;
      if (s > mrun) {
        float corr = expf(mrun - s);  // exp(-inf) = 0 on the first key
        l *= corr;
#pragma unroll
        for (int e = 0; e < D; ++e) acc[e] *= corr;
        mrun = s;
      }
      float pexp = expf(s - mrun);
      l += pexp;
#pragma unroll
      for (int e = 0; e < D; ++e) acc[e] = fmaf(pexp, Vs[t][e], acc[e]);
    }
  }
  if (!active) return;
  float* op = o + i * o_rs + j * o_ps + h * D;
  const float inv = l > 0.f ? 1.0f / l : 0.f;
#pragma unroll
  for (int e = 0; e < D; ++e) op[e] = acc[e] * inv;
}

// Single-representation attention of AttentionPairBias split over the keys: a CTA handles 64
// queries x one head x one key range and writes its unnormalised partial (acc[D], running max,
// running sum) to part[((split * H + h) * n_q + j) * (D + 2)]; k_attn_merge combines the
// splits. With N queries x 16 heads there are too few (query block, head) pairs to fill the
// GPU (and fewer still per Fold-CP rank), so the keys supply the parallelism.
template <int D>
__global__ void __launch_bounds__(64) k_attn_split(const float* __restrict__ q, int64_t q_ps,
                                                   const float* __restrict__ k, const float* __restrict__ v,
                                                   int64_t kv_ps, const float* __restrict__ bias, int64_t b_hs,
                                                   int64_t b_rs, int64_t n_q, int64_t n_keys, int64_t per_split,
                                                   float inv_sqrt_d_div, int H, float* __restrict__ part) {
  // 32-key tiles: K, V and the 64 queries' bias rows of the tile staged in shared memory (the
  // bias by 128-byte rows, consecutive keys on consecutive threads), then per query all 32 logits
  // at once, one running-max update per tile, the exponentials and the P.V accumulation. The
  // tiles are copied with cp.async (4-byte copies, zero-filled past the key range) into two
  // buffers where both fit in the 48 KB of static shared memory, so the next tile's loads are in
  // flight during the current tile's math; otherwise into one.
  constexpr int KT = 32;
  constexpr int TILE_BYTES = (2 * KT * (D + 1) + 64 * (KT + 1)) * 4;
  constexpr int NB = 2 * TILE_BYTES <= 48 * 1024 ? 2 : 1;
  __shared__ float Ks[NB][KT][D + 1];
  __shared__ float Vs[NB][KT][D + 1];
  __shared__ float Bs[NB][64][KT + 1];
  const int h = blockIdx.y;
  const int64_t sp = blockIdx.z;
  const int64_t j0 = (int64_t)blockIdx.x * 64;
  const int64_t j = j0 + threadIdx.x;
  const bool active = j < n_q;
  float qv[D];
  const float* qp = q + (active ? j : 0) * q_ps + h * D;
#pragma unroll
  for (int t = 0; t < D; ++t) qv[t] = qp[t] / inv_sqrt_d_div;  // reference divides q by sqrt(d)
  float mrun = -INFINITY, l = 0.f;
  float acc[D];
#pragma unroll
  for (int t = 0; t < D; ++t) acc[t] = 0.f;
  const int64_t kb0 = sp * per_split;
  const int64_t kb1 = kb0 + per_split < n_keys ? kb0 + per_split : n_keys;
  const float* kb = k + h * D;
  const float* vb = v + h * D;
  const float* bh = bias + (int64_t)h * b_hs;
  const int tk = threadIdx.x & (KT - 1), half = threadIdx.x >> 5;
  // one 4-byte asynchronous copy; src_bytes = 0 writes a zero (the source is then not read)
  auto cp4 = [](float* dst, const float* src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src), "r"(valid ? 4 : 0)
                 : "memory");
  };
  // copies of the tile starting at key kt0 into buffer b, as one commit group
  auto prefetch = [&](int64_t kt0, int b) {
    for (int idx = threadIdx.x; idx < KT * D; idx += 64) {
      const int kt = idx / D, t = idx - kt * D;
      const int64_t kr = kt0 + kt;
      const bool ok = kr < kb1;
      cp4(&Ks[b][kt][t], ok ? kb + kr * kv_ps + t : kb, ok);
      cp4(&Vs[b][kt][t], ok ? vb + kr * kv_ps + t : vb, ok);
    }
    const int64_t kk = kt0 + tk;
    for (int qq = half; qq < 64; qq += 2) {
      const bool ok = kk < kb1 && j0 + qq < n_q;
      cp4(&Bs[b][qq][tk], ok ? bh + (j0 + qq) * b_rs + kk : bh, ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  if (kb0 < kb1) prefetch(kb0, 0);
  int it = 0;
  for (int64_t k0 = kb0; k0 < kb1; k0 += KT, ++it) {
    const int b = NB == 2 ? (it & 1) : 0;
    if (NB == 1 && it > 0) prefetch(k0, 0);  // the trailing barrier freed the one buffer
    if (NB == 2 && k0 + KT < kb1) {
      prefetch(k0 + KT, b ^ 1);  // the other buffer: freed by the previous tile's trailing barrier
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();  // this tile's copies, from every thread, are in shared memory
    if (active) {
      const int64_t rem = kb1 - k0;
      const int nk = rem < KT ? (int)rem : KT;
      float sc[KT];
      float tmax = -INFINITY;
#pragma unroll
      for (int t = 0; t < KT; ++t) {
        float s = -INFINITY;
        if (t < nk) {
          float d0 = 0.f;
#pragma unroll
          for (int e = 0; e < D; ++e) d0 = fmaf(qv[e], Ks[b][t][e], d0);
          s = d0 + Bs[b][threadIdx.x][t];
        }
        sc[t] = s;
        tmax = fmaxf(tmax, s);
      }
      if (tmax > mrun) {
        const float corr = expf(mrun - tmax);  // exp(-inf) = 0 on the first tile
        l *= corr;
#pragma unroll
        for (int e = 0; e < D; ++e) acc[e] *= corr;
        mrun = tmax;
      }
#pragma unroll
      for (int t = 0; t < KT; ++t) {
        if (t < nk) {
          const float pexp = expf(sc[t] - mrun);
          l += pexp;
#pragma unroll
          for (int e = 0; e < D; ++e) acc[e] = fmaf(pexp, Vs[b][t][e], acc[e]);
        }
      }
    }
    __syncthreads();  // every thread is done with buffer b before it is refilled
  }
  if (!active) return;
  float* out = part + ((sp * H + h) * n_q + j) * (D + 2);
#pragma unroll
  for (int e = 0; e < D; ++e) out[e] = acc[e];
  out[D] = mrun;
  out[D + 1] = l;
}

// o(j, h*D + e) = sum_s acc_s[e] exp(m_s - M) / sum_s l_s exp(m_s - M),  M = max_s m_s.
template <int D>
__global__ void k_attn_merge(const float* __restrict__ part, int splits, int H, int64_t n_q,
                             float* __restrict__ o, int64_t o_ps) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n_q * H) return;
  const int64_t j = idx / H;
  const int h = (int)(idx - j * H);
  float M = -INFINITY;
  for (int sp = 0; sp < splits; ++sp) M = fmaxf(M, part[(((int64_t)sp * H + h) * n_q + j) * (D + 2) + D]);
  float acc[D];
#pragma unroll
  for (int e = 0; e < D; ++e) acc[e] = 0.f;
  float L = 0.f;
  if (M > -INFINITY) {
    for (int sp = 0; sp < splits; ++sp) {
      const float* pp = part + (((int64_t)sp * H + h) * n_q + j) * (D + 2);
      const float w = expf(pp[D] - M);  // an empty split has m = -inf: weight 0
      L = fmaf(pp[D + 1], w, L);
#pragma unroll
      for (int e = 0; e < D; ++e) acc[e] = fmaf(pp[e], w, acc[e]);
    }
  }
  const float inv = L > 0.f ? 1.0f / L : 0.f;
  float* op = o + j * o_ps + h * D;
#pragma unroll
  for (int e = 0; e < D; ++e) op[e] = acc[e] * inv;
}

// ============================================================================ host side

static inline unsigned nblk(int64_t n, int t) { return (unsigned)((n + t - 1) / t); }

template <class T, class TO>
static int ln_view(const T* x, int64_t rs, int64_t cs, int64_t n_rows, int64_t n_cols, int c,
                   const float* g, const float* b, float eps, TO* out, int64_t ops,
                   cudaStream_t st) {
  if (c > 1024) return fail(PF_EUNSUPPORTED, "LayerNorm channel count %d > 1024", c);
  int64_t P = n_rows * n_cols;
  if (P == 0) return PF_OK;
  {
    PF_LAUNCH_SCOPE(st, "k_ln_view");
    k_ln_view<T, TO><<<nblk(P, 8), 256, 0, st>>>(x, rs, cs, n_rows, n_cols, c, g, b, eps, out, ops);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

template <class TA, class TB>
static int gemm(const TA* A, int64_t sAb, int64_t sAm, const TB* B, int64_t sBb, int64_t sBn,
                float* C, int64_t sCb, int64_t sCm, int64_t sCn, int64_t batch, int64_t M,
                int64_t N, int64_t K, float alpha, int acc, cudaStream_t st) {
  if (M == 0 || N == 0 || batch == 0) return PF_OK;
  if (batch > 65535 || (M + 63) / 64 > 65535)
    return fail(PF_EUNSUPPORTED, "SIMT GEMM grid too large (batch %lld, M %lld)",
                (long long)batch, (long long)M);
  dim3 grid(nblk(N, 64), nblk(M, 64), (unsigned)batch);
  {
    PF_LAUNCH_SCOPE(st, "k_gemm_nt");
    k_gemm_nt<TA, TB><<<grid, 256, 0, st>>>(A, sAb, sAm, B, sBb, sBn, C, sCb, sCm, sCn, M, N, K,
                                            alpha, acc);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

template <class T, int L>
static int ln_rows_launch(const T* x, T* y, int64_t rows, int c, const float* g, const float* b, float eps,
                          cudaStream_t st) {
  const int64_t rows_per_block = 8 * (32 / L);
  const int64_t blocks = (rows + rows_per_block - 1) / rows_per_block;
  if (blocks > 0x7FFFFFFF) return fail(PF_EUNSUPPORTED, "LayerNorm: %lld rows is too many", (long long)rows);
  {
    PF_LAUNCH_SCOPE_WORK(st, "k_layernorm_rows", 2.0 * (double)rows * c * sizeof(T), 'b');
    k_layernorm_rows<T, L><<<(unsigned)blocks, 256, 0, st>>>(x, y, rows, c, g, b, eps);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

template <class T>
static int ln_rows(const T* x, T* y, int64_t rows, int c, const float* g, const float* b, float eps,
                   cudaStream_t st) {
  const int nv = c * (int)sizeof(T) / 16;
  if (nv >= 32) return ln_rows_launch<T, 32>(x, y, rows, c, g, b, eps, st);
  if (nv >= 16) return ln_rows_launch<T, 16>(x, y, rows, c, g, b, eps, st);
  if (nv >= 8) return ln_rows_launch<T, 8>(x, y, rows, c, g, b, eps, st);
  if (nv >= 4) return ln_rows_launch<T, 4>(x, y, rows, c, g, b, eps, st);
  if (nv >= 2) return ln_rows_launch<T, 2>(x, y, rows, c, g, b, eps, st);
  return ln_rows_launch<T, 1>(x, y, rows, c, g, b, eps, st);
}

int layernorm(const void* x, void* y, const float* g, const float* b, int64_t rows, int c,
              float eps, int dtype, cudaStream_t st) {
  const size_t esz = dtype == PF_F32 ? 4 : 2;
  const bool vec = (c * esz) % 16 == 0 && ((uintptr_t)x) % 16 == 0 && ((uintptr_t)y) % 16 == 0;
  if (vec) {
    if (dtype == PF_F32) return ln_rows<float>((const float*)x, (float*)y, rows, c, g, b, eps, st);
    return ln_rows<__nv_bfloat16>((const __nv_bfloat16*)x, (__nv_bfloat16*)y, rows, c, g, b, eps, st);
  }
  // channel counts whose rows are not whole 16-byte vectors: the warp-per-row scalar kernel
  if (dtype == PF_F32)
    return ln_view<float, float>((const float*)x, c, 0, rows, 1, c, g, b, eps, (float*)y, c, st);
  return ln_view<__nv_bfloat16, __nv_bfloat16>((const __nv_bfloat16*)x, c, 0, rows, 1, c, g, b,
                                                eps, (__nv_bfloat16*)y, c, st);
}

// ---------------------------------------------------------------- triangle multiplication
// Stages: project (LN_in, the gated projection of one side into channel-major a/b) and
// combine (the per-channel contraction, LN_out, W_z, the gate from zg, the residual). The
// fused entry point runs project twice and combine once on fp32 intermediates; the split
// entry points (Fold-CP exchanges the projections) keep a/b in the storage dtype.
struct ProjWs {
  float *x, *pa, *pg;
};
static void proj_plan(Arena& ar, int64_t P, int c_z, int c_h, ProjWs& w) {
  w.x = ar.take<float>(P * c_z);
  w.pa = ar.take<float>(P * c_h);
  w.pg = ar.take<float>(P * c_h);
}
struct CombineWs {
  float *p, *xn, *y, *xo, *gg;
};
static void combine_plan(Arena& ar, int64_t Po, int c_z, int c_h, CombineWs& w) {
  w.p = ar.take<float>(Po * c_h);
  w.xn = ar.take<float>(Po * c_h);
  w.y = ar.take<float>(Po * c_z);
  w.xo = ar.take<float>(Po * c_z);
  w.gg = ar.take<float>(Po * c_z);
}

template <class T, class TO>
static int project_side(const pf_trimul_params* p, pf_pair_view z, pf_mask_view m, int64_t n_r, int64_t n_k,
                        int c_z, int c_h, const T* W_p, const T* W_g, TO* out, int64_t ld, const ProjWs& w,
                        cudaStream_t st) {
  const float eps = 1e-5f;
  const int64_t P = n_r * n_k;
  PF_TRY((ln_view<T, float>((const T*)z.ptr, z.row_stride, z.col_stride, n_r, n_k, c_z, p->ln_in_w,
                            p->ln_in_b, eps, w.x, c_z, st)));
  PF_TRY((gemm<float, T>(w.x, 0, c_z, W_p, 0, c_z, w.pa, 0, c_h, 1, 1, P, c_h, c_z, 1.f, 0, st)));
  PF_TRY((gemm<float, T>(w.x, 0, c_z, W_g, 0, c_z, w.pg, 0, c_h, 1, 1, P, c_h, c_z, 1.f, 0, st)));
  {
    PF_LAUNCH_SCOPE(st, "k_gate_to_cmajor");
    k_gate_to_cmajor<TO><<<nblk(P * c_h, 256), 256, 0, st>>>(w.pa, w.pg, m, n_r, n_k, c_h, out, ld);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

template <class T, class TA>
static int combine(const pf_trimul_params* p, const TA* a, int64_t lda, const TA* b, int64_t ldb, int64_t n_i,
                   int64_t n_j, int64_t n_k, pf_pair_view zg, pf_pair_view zo, int c_z, int c_h, int acc,
                   const CombineWs& w, cudaStream_t st) {
  const float eps = 1e-5f;
  const int64_t Po = n_i * n_j;
  // x[ch] = a[ch] b[ch]^T  (batched over channels)
  PF_TRY((gemm<TA, TA>(a, n_i * lda, lda, b, n_j * ldb, ldb, w.p, Po, n_j, 1, c_h, n_i, n_j, n_k, 1.f, 0,
                       st)));
  // LN_out, linear_z
  {
    PF_LAUNCH_SCOPE(st, "k_ln_cmajor");
    k_ln_cmajor<<<nblk(Po, 8), 256, 0, st>>>(w.p, Po, c_h, p->ln_out_w, p->ln_out_b, eps, w.xn);
  }
  PF_CHECK_LAUNCH();
  PF_TRY((gemm<float, T>(w.xn, 0, c_h, (const T*)p->w_z, 0, c_h, w.y, 0, c_z, 1, 1, Po, c_z, c_h,
                         1.f, 0, st)));
  // gate from LN_in(zg)
  PF_TRY((ln_view<T, float>((const T*)zg.ptr, zg.row_stride, zg.col_stride, n_i, n_j, c_z,
                            p->ln_in_w, p->ln_in_b, eps, w.xo, c_z, st)));
  PF_TRY((gemm<float, T>(w.xo, 0, c_z, (const T*)p->w_g, 0, c_z, w.gg, 0, c_z, 1, 1, Po, c_z, c_z,
                         1.f, 0, st)));
  {
    PF_LAUNCH_SCOPE(st, "k_combine_view");
    k_combine_view<T><<<nblk(Po * c_z, 256), 256, 0, st>>>((T*)zo.ptr, zo.row_stride, zo.col_stride,
                                                           n_i, n_j, c_z, w.y, w.gg, acc);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

struct TrimulWs {
  ProjWs pr;
  float *a, *b;
  CombineWs cb;
};
static void trimul_plan(Arena& ar, int64_t n_i, int64_t n_j, int64_t n_k, int c_z, int c_h,
                        TrimulWs& w) {
  int64_t Pa = n_i * n_k, Pb = n_j * n_k, Po = n_i * n_j;
  proj_plan(ar, Pa > Pb ? Pa : Pb, c_z, c_h, w.pr);
  w.a = ar.take<float>(Pa * c_h);
  w.b = ar.take<float>(Pb * c_h);
  combine_plan(ar, Po, c_z, c_h, w.cb);
}

size_t trimul_ws_bytes(int64_t n_i, int64_t n_j, int64_t n_k, int c_z, int c_h) {
  Arena ar(nullptr, 0);
  TrimulWs w;
  trimul_plan(ar, n_i, n_j, n_k, c_z, c_h, w);
  return ar.used;
}

template <class T>
static int trimul_t(const pf_trimul_params* p, pf_pair_view za, pf_pair_view zb, pf_mask_view ma,
                    pf_mask_view mb, pf_pair_view zg, pf_pair_view zo, int64_t n_i, int64_t n_j, int64_t n_k,
                    int c_z, int c_h, int acc, Arena& ar, cudaStream_t st) {
  TrimulWs w;
  trimul_plan(ar, n_i, n_j, n_k, c_z, c_h, w);
  if (!ar.ok()) return fail(PF_EWORKSPACE, "trimul workspace too small (%zu < %zu)", ar.cap, ar.used);
  PF_TRY((project_side<T, float>(p, za, ma, n_i, n_k, c_z, c_h, (const T*)p->w_ap, (const T*)p->w_ag, w.a, n_k,
                                 w.pr, st)));
  PF_TRY((project_side<T, float>(p, zb, mb, n_j, n_k, c_z, c_h, (const T*)p->w_bp, (const T*)p->w_bg, w.b, n_k,
                                 w.pr, st)));
  return combine<T, float>(p, w.a, n_k, w.b, n_k, n_i, n_j, n_k, zg, zo, c_z, c_h, acc, w.cb, st);
}

int trimul(const pf_trimul_params* p, pf_pair_view za, pf_pair_view zb, pf_mask_view ma,
           pf_mask_view mb, pf_pair_view zg, pf_pair_view zo, int64_t n_i, int64_t n_j, int64_t n_k, int c_z,
           int c_h, int acc, int dtype, void* ws, size_t ws_bytes, cudaStream_t st) {
  Arena ar(ws, ws_bytes);
  if (dtype == PF_F32)
    return trimul_t<float>(p, za, zb, ma, mb, zg, zo, n_i, n_j, n_k, c_z, c_h, acc, ar, st);
  return trimul_t<__nv_bfloat16>(p, za, zb, ma, mb, zg, zo, n_i, n_j, n_k, c_z, c_h, acc, ar, st);
}

size_t trimul_project_ws_bytes(int64_t n_rows, int64_t n_cols, int c_z, int c_h) {
  Arena ar(nullptr, 0);
  ProjWs w;
  proj_plan(ar, n_rows * n_cols, c_z, c_h, w);
  return ar.used;
}

int trimul_project(const pf_trimul_params* p, pf_pair_view z, pf_mask_view m, int64_t n_rows, int64_t n_cols,
                   int c_z, int c_h, int dtype, void* a, void* b, int64_t ld, void* ws, size_t ws_bytes,
                   cudaStream_t st) {
  Arena ar(ws, ws_bytes);
  ProjWs w;
  proj_plan(ar, n_rows * n_cols, c_z, c_h, w);
  if (!ar.ok()) return fail(PF_EWORKSPACE, "trimul project workspace too small (%zu < %zu)", ar.cap, ar.used);
  if (dtype == PF_F32) {
    PF_TRY((project_side<float, float>(p, z, m, n_rows, n_cols, c_z, c_h, (const float*)p->w_ap,
                                       (const float*)p->w_ag, (float*)a, ld, w, st)));
    return project_side<float, float>(p, z, m, n_rows, n_cols, c_z, c_h, (const float*)p->w_bp,
                                      (const float*)p->w_bg, (float*)b, ld, w, st);
  }
  using B = __nv_bfloat16;
  PF_TRY((project_side<B, B>(p, z, m, n_rows, n_cols, c_z, c_h, (const B*)p->w_ap, (const B*)p->w_ag, (B*)a,
                             ld, w, st)));
  return project_side<B, B>(p, z, m, n_rows, n_cols, c_z, c_h, (const B*)p->w_bp, (const B*)p->w_bg, (B*)b,
                            ld, w, st);
}

size_t trimul_combine_ws_bytes(int64_t n_i, int64_t n_j, int c_z, int c_h) {
  Arena ar(nullptr, 0);
  CombineWs w;
  combine_plan(ar, n_i * n_j, c_z, c_h, w);
  return ar.used;
}

int trimul_combine(const pf_trimul_params* p, const void* a, const void* b, int64_t ld, int64_t n_i, int64_t n_j,
                   int64_t n_k, pf_pair_view zg, pf_pair_view zo, int c_z, int c_h, int acc, int dtype, void* ws,
                   size_t ws_bytes, cudaStream_t st) {
  Arena ar(ws, ws_bytes);
  CombineWs w;
  combine_plan(ar, n_i * n_j, c_z, c_h, w);
  if (!ar.ok()) return fail(PF_EWORKSPACE, "trimul combine workspace too small (%zu < %zu)", ar.cap, ar.used);
  if (dtype == PF_F32)
    return combine<float, float>(p, (const float*)a, ld, (const float*)b, ld, n_i, n_j, n_k, zg, zo, c_z, c_h,
                                 acc, w, st);
  using B = __nv_bfloat16;
  return combine<B, B>(p, (const B*)a, ld, (const B*)b, ld, n_i, n_j, n_k, zg, zo, c_z, c_h, acc, w, st);
}

// ---------------------------------------------------------------- triangle attention
struct TriattWs {
  float *x, *q, *k, *v, *bias, *o, *g, *y;
};
static void triatt_plan(Arena& ar, int64_t n_rows, int64_t n_keys, int64_t n_q, int c, int H,
                        int d, bool own_bias, TriattWs& w) {
  int64_t P = n_rows * n_keys, Pq = n_rows * n_q;
  int hd = H * d;
  w.x = ar.take<float>(P * c);
  w.q = ar.take<float>(P * hd);
  w.k = ar.take<float>(P * hd);
  w.v = ar.take<float>(P * hd);
  w.bias = own_bias ? ar.take<float>((int64_t)H * n_keys * n_keys) : nullptr;
  w.o = ar.take<float>(Pq * hd);
  w.g = ar.take<float>(Pq * hd);
  w.y = ar.take<float>(Pq * c);
}

size_t triatt_ws_bytes(int64_t n_rows, int64_t n_keys, int64_t n_q, int c, int H, int d) {
  Arena ar(nullptr, 0);
  TriattWs w;
  triatt_plan(ar, n_rows, n_keys, n_q, c, H, d, true, w);
  return ar.used;
}

template <class T, class TB>
static int launch_attn(int d, const float* q, int64_t q_rs, int64_t q_ps, int64_t q_col0,
                       const float* k, const float* v, int64_t kv_rs, int64_t kv_ps,
                       const TB* bias, int64_t b_hs, int64_t b_rs, float bias_scale,
                       pf_mask_view m, float inf, int64_t n_rows, int64_t n_q, int H,
                       int64_t n_valid, float* o, int64_t o_rs, int64_t o_ps, cudaStream_t st) {
  if (n_rows > 65535) return fail(PF_EUNSUPPORTED, "too many attention rows (%lld)", (long long)n_rows);
  dim3 grid(nblk(n_q, 64), H, (unsigned)n_rows);
  float sd = sqrtf((float)d);
#define PF_ATTN_CASE(DD)                                                                       \
  case DD:                                                                                     \
    k_attn_simt<DD, TB><<<grid, 64, 0, st>>>(q, q_rs, q_ps, q_col0, k, v, kv_rs, kv_ps, bias,  \
                                             b_hs, b_rs, bias_scale, m, inf, n_q, n_valid, sd, \
                                             o, o_rs, o_ps);                                   \
    break;
  PF_LAUNCH_SCOPE(st, "k_attn_simt");
  switch (d) {
    PF_ATTN_CASE(8)
    PF_ATTN_CASE(16)
    PF_ATTN_CASE(24)
    PF_ATTN_CASE(32)
    PF_ATTN_CASE(48)
    PF_ATTN_CASE(64)
    default:
      return fail(PF_EUNSUPPORTED, "head dim %d not in {8,16,24,32,48,64}", d);
  }
#undef PF_ATTN_CASE
  PF_CHECK_LAUNCH();
  return PF_OK;
}

// Key splits of the APB single attention: enough CTAs (query blocks x heads x splits) for about
// eight 64-thread CTAs per SM of a 148-SM part, each split at least one 64-key tile.
static int64_t apb_splits(int64_t n, int64_t nq, int H) {
  const int64_t pairs = (int64_t)nblk(nq, 64) * H;
  int64_t s = (1184 + pairs - 1) / (pairs > 0 ? pairs : 1);
  const int64_t tiles = (n + 63) / 64;
  if (s > tiles) s = tiles;
  return s < 1 ? 1 : s;
}

static int launch_attn_split(int d, const float* q, int64_t q_ps, const float* k, const float* v, int64_t kv_ps,
                             const float* bias, int64_t b_hs, int64_t b_rs, int64_t n_q, int64_t n, int H,
                             float* part, float* o, int64_t o_ps, cudaStream_t st) {
  if (n_q == 0) return PF_OK;
  const int64_t splits = apb_splits(n, n_q, H);
  int64_t per = ((n + splits - 1) / splits + 63) / 64 * 64;
  if (per < 64) per = 64;
  const int64_t used = n > 0 ? (n + per - 1) / per : 1;
  if (used > 65535) return fail(PF_EUNSUPPORTED, "too many key splits (%lld)", (long long)used);
  dim3 grid(nblk(n_q, 64), H, (unsigned)used);
  const float sd = sqrtf((float)d);
  const unsigned mgrid = nblk(n_q * H, 128);
#define PF_SPLIT_CASE(DD)                                                                          \
  case DD: {                                                                                       \
    {                                                                                              \
      PF_LAUNCH_SCOPE(st, "k_attn_split");                                                         \
      k_attn_split<DD><<<grid, 64, 0, st>>>(q, q_ps, k, v, kv_ps, bias, b_hs, b_rs, n_q, n, per,   \
                                            sd, H, part);                                          \
    }                                                                                              \
    PF_CHECK_LAUNCH();                                                                             \
    PF_LAUNCH_SCOPE(st, "k_attn_merge");                                                           \
    k_attn_merge<DD><<<mgrid, 128, 0, st>>>(part, (int)used, H, n_q, o, o_ps);                     \
    break;                                                                                         \
  }
  switch (d) {
    PF_SPLIT_CASE(8)
    PF_SPLIT_CASE(16)
    PF_SPLIT_CASE(24)
    PF_SPLIT_CASE(32)
    PF_SPLIT_CASE(48)
    PF_SPLIT_CASE(64)
    default:
      return fail(PF_EUNSUPPORTED, "head dim %d not in {8,16,24,32,48,64}", d);
  }
#undef PF_SPLIT_CASE
  PF_CHECK_LAUNCH();
  return PF_OK;
}

static size_t apb_part_floats(int64_t n, int64_t nq, int c_s, int H) {
  return (size_t)apb_splits(n, nq, H) * nq * (c_s + 2 * H);  // splits x nq x H x (d + 2)
}

size_t attn_split_part_floats(int64_t n, int64_t nq, int c_s, int H) { return apb_part_floats(n, nq, c_s, H); }

int attn_split(int d, const float* q, int64_t q_ps, const float* k, const float* v, int64_t kv_ps, const float* bias,
               int64_t b_hs, int64_t b_rs, int64_t n_q, int64_t n, int H, float* part, float* o, int64_t o_ps,
               cudaStream_t st) {
  return launch_attn_split(d, q, q_ps, k, v, kv_ps, bias, b_hs, b_rs, n_q, n, H, part, o, o_ps, st);
}

template <class T>
static int triatt_bias_t(const pf_triatt_params* p, pf_pair_view z, int64_t n_rows, int64_t n_cols,
                         void* bias, int64_t hs, int64_t rs, int c, int H, float scale,
                         float* xbuf, cudaStream_t st) {
  // xbuf: LN(z) [n_rows*n_cols, c] (fp32), then bias(h, r, s) = scale * x . W_b[h]
  PF_TRY((ln_view<T, float>((const T*)z.ptr, z.row_stride, z.col_stride, n_rows, n_cols, c,
                            p->ln_w, p->ln_b, 1e-5f, xbuf, c, st)));
  return PF_OK;
}

template <class T>
static int triatt_t(const pf_triatt_params* p, pf_pair_view zs, pf_mask_view m, const void* bias,
                    int64_t b_hs, int64_t b_rs, pf_pair_view zo, int64_t n_rows, int64_t n_keys,
                    int64_t n_valid, int64_t q_col0, int64_t n_q, int c, int H, int d, float inf,
                    int acc, Arena& ar, cudaStream_t st) {
  TriattWs w;
  triatt_plan(ar, n_rows, n_keys, n_q, c, H, d, bias == nullptr, w);
  if (!ar.ok()) return fail(PF_EWORKSPACE, "triatt workspace too small (%zu < %zu)", ar.cap, ar.used);
  const int hd = H * d;
  const int64_t P = n_rows * n_keys, Pq = n_rows * n_q;
  PF_TRY((ln_view<T, float>((const T*)zs.ptr, zs.row_stride, zs.col_stride, n_rows, n_keys, c,
                            p->ln_w, p->ln_b, 1e-5f, w.x, c, st)));
  PF_TRY((gemm<float, T>(w.x, 0, c, (const T*)p->w_q, 0, c, w.q, 0, hd, 1, 1, P, hd, c, 1.f, 0, st)));
  PF_TRY((gemm<float, T>(w.x, 0, c, (const T*)p->w_k, 0, c, w.k, 0, hd, 1, 1, P, hd, c, 1.f, 0, st)));
  PF_TRY((gemm<float, T>(w.x, 0, c, (const T*)p->w_v, 0, c, w.v, 0, hd, 1, 1, P, hd, c, 1.f, 0, st)));
  if (bias == nullptr) {
    // square single-device case: bias(h, j, k) = W_b . x(j, k), written [H][n][n]
    PF_TRY((gemm<float, T>(w.x, 0, c, (const T*)p->w_bias, 0, c, w.bias, 0, 1, n_keys * n_keys, 1,
                           P, H, c, 1.f, 0, st)));
    PF_TRY((launch_attn<T, float>(d, w.q, n_keys * hd, hd, q_col0, w.k, w.v, n_keys * hd, hd,
                                  w.bias, n_keys * n_keys, n_keys, 1.0f, m, inf, n_rows, n_q, H,
                                  n_valid, w.o, n_q * hd, hd, st)));
  } else if (sizeof(T) == 4) {
    PF_TRY((launch_attn<T, float>(d, w.q, n_keys * hd, hd, q_col0, w.k, w.v, n_keys * hd, hd,
                                  (const float*)bias, b_hs, b_rs, 1.0f, m, inf, n_rows, n_q, H,
                                  n_valid, w.o, n_q * hd, hd, st)));
  } else {
    // bf16-mode bias buffers hold f16 log2-scaled values (the tensor-core path's format)
    PF_TRY((launch_attn<T, __half>(d, w.q, n_keys * hd, hd, q_col0, w.k, w.v, n_keys * hd,
                                          hd, (const __half*)bias, b_hs, b_rs,
                                          0.69314718055994531f, m, inf, n_rows, n_q, H, n_valid,
                                          w.o, n_q * hd, hd, st)));
  }
  // gate from LN'd query input, then output projection
  PF_TRY((gemm<float, T>(w.x + q_col0 * c, n_keys * c, c, (const T*)p->w_g, 0, c, w.g, n_q * hd,
                         hd, 1, n_rows, n_q, hd, c, 1.f, 0, st)));
  {
    PF_LAUNCH_SCOPE(st, "k_gate_inplace");
    k_gate_inplace<<<nblk(Pq * hd, 256), 256, 0, st>>>(w.o, w.g, Pq * hd);
  }
  PF_CHECK_LAUNCH();
  PF_TRY((gemm<float, T>(w.o, 0, hd, (const T*)p->w_o, 0, hd, w.y, 0, c, 1, 1, Pq, c, hd, 1.f, 0, st)));
  {
    PF_LAUNCH_SCOPE(st, "k_combine_view");
    k_combine_view<T><<<nblk(Pq * c, 256), 256, 0, st>>>((T*)zo.ptr, zo.row_stride, zo.col_stride,
                                                         n_rows, n_q, c, w.y, nullptr, acc);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

int triatt(const pf_triatt_params* p, pf_pair_view zs, pf_mask_view m, const void* bias,
           int64_t b_hs, int64_t b_rs, pf_pair_view zo, int64_t n_rows, int64_t n_keys,
           int64_t n_valid, int64_t q_col0, int64_t n_q, int c, int H, int d, float inf, int acc,
           int dtype, void* ws, size_t ws_bytes, cudaStream_t st) {
  Arena ar(ws, ws_bytes);
  if (dtype == PF_F32)
    return triatt_t<float>(p, zs, m, bias, b_hs, b_rs, zo, n_rows, n_keys, n_valid, q_col0, n_q, c,
                           H, d, inf, acc, ar, st);
  return triatt_t<__nv_bfloat16>(p, zs, m, bias, b_hs, b_rs, zo, n_rows, n_keys, n_valid, q_col0,
                                 n_q, c, H, d, inf, acc, ar, st);
}

size_t triatt_bias_ws_bytes(int64_t n_rows, int64_t n_cols, int c, int H) {
  return align_up((size_t)(n_rows * n_cols) * (c + H) * sizeof(float), 256);
}

// fp32 -> fp32 (scale 1) or -> bf16 scaled by log2(e)
template <class TO>
__global__ void k_bias_store(const float* __restrict__ src, int64_t n_rows, int64_t n_cols, int H,
                             TO* __restrict__ dst, int64_t hs, int64_t rs, float scale) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t P = n_rows * n_cols;
  if (idx >= P * H) return;
  const int64_t h = idx / P, p = idx - h * P;
  const int64_t r = p / n_cols, s = p - r * n_cols;
  dst[h * hs + r * rs + s] = from_f<TO>(src[p * H + h] * scale);
}

int triatt_bias(const pf_triatt_params* p, pf_pair_view z, int64_t n_rows, int64_t n_cols,
                void* bias, int64_t hs, int64_t rs, int c, int H, int dtype, void* ws,
                size_t ws_bytes, cudaStream_t st) {
  Arena ar(ws, ws_bytes);
  int64_t P = n_rows * n_cols;
  float* x = ar.take<float>(P * c);
  float* bb = ar.take<float>(P * H);
  if (!ar.ok()) return fail(PF_EWORKSPACE, "triatt_bias workspace too small");
  if (dtype == PF_F32) {
    PF_TRY(triatt_bias_t<float>(p, z, n_rows, n_cols, bias, hs, rs, c, H, 1.f, x, st));
    PF_TRY((gemm<float, float>(x, 0, c, (const float*)p->w_bias, 0, c, bb, 0, H, 1, 1, P, H, c, 1.f, 0, st)));
    {
      PF_LAUNCH_SCOPE(st, "k_bias_store");
      k_bias_store<float><<<nblk(P * H, 256), 256, 0, st>>>(bb, n_rows, n_cols, H, (float*)bias, hs, rs, 1.f);
    }
  } else {
    PF_TRY(triatt_bias_t<__nv_bfloat16>(p, z, n_rows, n_cols, bias, hs, rs, c, H, 1.f, x, st));
    PF_TRY((gemm<float, __nv_bfloat16>(x, 0, c, (const __nv_bfloat16*)p->w_bias, 0, c, bb, 0, H, 1, 1,
                                       P, H, c, 1.f, 0, st)));
    {
      PF_LAUNCH_SCOPE(st, "k_bias_store");
      k_bias_store<__half><<<nblk(P * H, 256), 256, 0, st>>>(
          bb, n_rows, n_cols, H, (__half*)bias, hs, rs, 1.4426950408889634f);
    }
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

// ---------------------------------------------------------------- transition
size_t transition_ws_bytes(int64_t rows, int c, int nm) {
  Arena ar(nullptr, 0);
  ar.take<float>(rows * c);
  ar.take<float>(rows * c * nm);
  ar.take<float>(rows * c * nm);
  ar.take<float>(rows * c);
  return ar.used;
}

template <class T>
static int transition_t(const pf_transition_params* p, const T* x, int64_t xs, T* out, int64_t os,
                        int64_t rows, int c, int nm, int acc, Arena& ar, cudaStream_t st) {
  float* y = ar.take<float>(rows * c);
  float* a = ar.take<float>(rows * c * nm);
  float* b = ar.take<float>(rows * c * nm);
  float* o = ar.take<float>(rows * c);
  if (!ar.ok()) return fail(PF_EWORKSPACE, "transition workspace too small");
  const int hc = c * nm;
  PF_TRY((ln_view<T, float>(x, xs, 0, rows, 1, c, p->ln_w, p->ln_b, 1e-5f, y, c, st)));
  PF_TRY((gemm<float, T>(y, 0, c, (const T*)p->w_a, 0, c, a, 0, hc, 1, 1, rows, hc, c, 1.f, 0, st)));
  PF_TRY((gemm<float, T>(y, 0, c, (const T*)p->w_b, 0, c, b, 0, hc, 1, 1, rows, hc, c, 1.f, 0, st)));
  {
    PF_LAUNCH_SCOPE(st, "k_swiglu");
    k_swiglu<<<nblk(rows * hc, 256), 256, 0, st>>>(a, b, rows * hc);
  }
  PF_CHECK_LAUNCH();
  PF_TRY((gemm<float, T>(b, 0, hc, (const T*)p->w_o, 0, hc, o, 0, c, 1, 1, rows, c, hc, 1.f, 0, st)));
  {
    PF_LAUNCH_SCOPE(st, "k_combine_view");
    k_combine_view<T><<<nblk(rows * c, 256), 256, 0, st>>>(out, os, 0, rows, 1, c, o, nullptr, acc);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

int transition(const pf_transition_params* p, const void* x, int64_t xs, void* out, int64_t os,
               int64_t rows, int c, int nm, int acc, int dtype, void* ws, size_t ws_bytes,
               cudaStream_t st) {
  Arena ar(ws, ws_bytes);
  if (dtype == PF_F32)
    return transition_t<float>(p, (const float*)x, xs, (float*)out, os, rows, c, nm, acc, ar, st);
  return transition_t<__nv_bfloat16>(p, (const __nv_bfloat16*)x, xs, (__nv_bfloat16*)out, os, rows,
                                     c, nm, acc, ar, st);
}

// ---------------------------------------------------------------- AttentionPairBias
size_t apb_pair_bias_ws_bytes(int64_t P, int c_z, int H) {
  return align_up((size_t)P * c_z * 4, 256) + align_up((size_t)P * H * 4, 256);
}

int apb_pair_bias(const pf_apb_params* p, pf_pair_view z, int64_t n_rows, int64_t n_cols,
                  float* bias, int64_t hs, int64_t rs, int c_z, int H, int dtype, void* ws,
                  size_t ws_bytes, cudaStream_t st) {
  Arena ar(ws, ws_bytes);
  int64_t P = n_rows * n_cols;
  float* x = ar.take<float>(P * c_z);
  float* bb = ar.take<float>(P * H);
  if (!ar.ok()) return fail(PF_EWORKSPACE, "apb_pair_bias workspace too small");
  if (dtype == PF_F32) {
    PF_TRY((ln_view<float, float>((const float*)z.ptr, z.row_stride, z.col_stride, n_rows, n_cols,
                                  c_z, p->ln_z_w, p->ln_z_b, 1e-5f, x, c_z, st)));
    PF_TRY((gemm<float, float>(x, 0, c_z, (const float*)p->w_z, 0, c_z, bb, 0, H, 1, 1, P, H, c_z, 1.f, 0, st)));
  } else {
    PF_TRY((ln_view<__nv_bfloat16, float>((const __nv_bfloat16*)z.ptr, z.row_stride, z.col_stride,
                                          n_rows, n_cols, c_z, p->ln_z_w, p->ln_z_b, 1e-5f, x, c_z, st)));
    PF_TRY((gemm<float, __nv_bfloat16>(x, 0, c_z, (const __nv_bfloat16*)p->w_z, 0, c_z, bb, 0, H, 1,
                                       1, P, H, c_z, 1.f, 0, st)));
  }
  {
    PF_LAUNCH_SCOPE(st, "k_bias_store");
    k_bias_store<float><<<nblk(P * H, 256), 256, 0, st>>>(bb, n_rows, n_cols, H, bias, hs, rs, 1.f);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

template <class T>
static int apb_t(const pf_apb_params* p, const T* s_in, T* s_out, const float* bias, int64_t b_hs,
                 int64_t b_rs, int64_t n, int64_t q0, int64_t nq, int c_s, int H, int acc, Arena& ar,
                 cudaStream_t st) {
  // keys/values need LN(s) of all n rows; queries, gate and output only rows [q0, q0 + nq)
  float* a = ar.take<float>(n * c_s);
  float* kv = ar.take<float>(n * c_s * 2);
  float* qg = ar.take<float>(nq * c_s * 2);
  float* o = ar.take<float>(nq * c_s);
  float* y = ar.take<float>(nq * c_s);
  float* part = ar.take<float>(apb_part_floats(n, nq, c_s, H));
  if (!ar.ok()) return fail(PF_EWORKSPACE, "apb workspace too small");
  float *k = kv, *v = kv + n * c_s, *q = qg, *g = qg + nq * c_s;
  const float* aq = a + q0 * c_s;
  const int d = c_s / H;
  PF_TRY((ln_view<T, float>(s_in, c_s, 0, n, 1, c_s, p->ln_a_w, p->ln_a_b, 1e-5f, a, c_s, st)));
  PF_TRY((gemm<float, T>(aq, 0, c_s, (const T*)p->w_q, 0, c_s, q, 0, c_s, 1, 1, nq, c_s, c_s, 1.f, 0, st)));
  if (p->b_q) {
    {
      PF_LAUNCH_SCOPE(st, "k_add_bias");
      k_add_bias<<<nblk(nq * c_s, 256), 256, 0, st>>>(q, p->b_q, nq, c_s);
    }
    PF_CHECK_LAUNCH();
  }
  PF_TRY((gemm<float, T>(a, 0, c_s, (const T*)p->w_k, 0, c_s, k, 0, c_s, 1, 1, n, c_s, c_s, 1.f, 0, st)));
  PF_TRY((gemm<float, T>(a, 0, c_s, (const T*)p->w_v, 0, c_s, v, 0, c_s, 1, 1, n, c_s, c_s, 1.f, 0, st)));
  PF_TRY((gemm<float, T>(aq, 0, c_s, (const T*)p->w_g, 0, c_s, g, 0, c_s, 1, 1, nq, c_s, c_s, 1.f, 0, st)));
  // nq queries over n keys; bias(h, j, k) = bias[h*b_hs + j*b_rs + k]
  PF_TRY(launch_attn_split(d, q, c_s, k, v, c_s, bias, b_hs, b_rs, nq, n, H, part, o, c_s, st));
  {
    PF_LAUNCH_SCOPE(st, "k_gate_inplace");
    k_gate_inplace<<<nblk(nq * c_s, 256), 256, 0, st>>>(o, g, nq * c_s);
  }
  PF_CHECK_LAUNCH();
  PF_TRY((gemm<float, T>(o, 0, c_s, (const T*)p->w_o, 0, c_s, y, 0, c_s, 1, 1, nq, c_s, c_s, 1.f, 0, st)));
  {
    PF_LAUNCH_SCOPE(st, "k_combine_view");
    k_combine_view<T><<<nblk(nq * c_s, 256), 256, 0, st>>>(s_out, c_s, 0, nq, 1, c_s, y, nullptr, acc);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

size_t apb_rows_ws_bytes(int64_t n, int64_t nq, int c_s, int H) {
  Arena ar(nullptr, 0);
  ar.take<float>(n * c_s);
  ar.take<float>(n * c_s * 2);
  ar.take<float>(nq * c_s * 2);
  ar.take<float>(nq * c_s);
  ar.take<float>(nq * c_s);
  ar.take<float>(apb_part_floats(n, nq, c_s, H));
  return ar.used + 1024;
}

int apb_rows(const pf_apb_params* p, const void* s_in, void* s_out, const float* bias, int64_t b_hs,
             int64_t b_rs, int64_t n, int64_t q0, int64_t nq, int c_s, int H, int acc, int dtype, void* ws,
             size_t ws_bytes, cudaStream_t st) {
  Arena ar(ws, ws_bytes);
  if (dtype == PF_F32)
    return apb_t<float>(p, (const float*)s_in, (float*)s_out, bias, b_hs, b_rs, n, q0, nq, c_s, H, acc,
                        ar, st);
  return apb_t<__nv_bfloat16>(p, (const __nv_bfloat16*)s_in, (__nv_bfloat16*)s_out, bias, b_hs, b_rs, n,
                              q0, nq, c_s, H, acc, ar, st);
}

// ---------------------------------------------------------------- row projections, pair LN + linear
template <class T>
int gemm_rows(const T* a, int64_t lda, const T* w, float* c, int64_t m, int n, int k, cudaStream_t st) {
  return gemm<T, T>(a, 0, lda, w, 0, k, c, 0, n, 1, 1, m, n, k, 1.f, 0, st);
}
template int gemm_rows<float>(const float*, int64_t, const float*, float*, int64_t, int, int, cudaStream_t);
template int gemm_rows<__nv_bfloat16>(const __nv_bfloat16*, int64_t, const __nv_bfloat16*, float*, int64_t, int, int,
                                      cudaStream_t);

size_t pair_ln_linear_ws_bytes(int64_t n_rows, int64_t n_cols, int c_in, int c_out) {
  Arena ar(nullptr, 0);
  ar.take<float>((size_t)n_rows * n_cols * c_in);
  ar.take<float>((size_t)n_rows * n_cols * c_out);
  return ar.used;
}

template <class T>
static int pair_ln_linear_t(const pf_pair_linear_params* p, pf_pair_view zi, pf_pair_view zo, int64_t n_rows,
                            int64_t n_cols, int c_in, int c_out, int acc, Arena& ar, cudaStream_t st) {
  const int64_t P = n_rows * n_cols;
  float* y = ar.take<float>((size_t)P * c_in);
  float* o = ar.take<float>((size_t)P * c_out);
  if (!ar.ok()) return fail(PF_EWORKSPACE, "pair LN-linear workspace too small");
  PF_TRY((ln_view<T, float>((const T*)zi.ptr, zi.row_stride, zi.col_stride, n_rows, n_cols, c_in, p->ln_w, p->ln_b,
                            1e-5f, y, c_in, st)));
  PF_TRY((gemm<float, T>(y, 0, c_in, (const T*)p->w, 0, c_in, o, 0, c_out, 1, 1, P, c_out, c_in, 1.f, 0, st)));
  {
    PF_LAUNCH_SCOPE(st, "k_combine_view");
    k_combine_view<T><<<nblk(P * c_out, 256), 256, 0, st>>>((T*)zo.ptr, zo.row_stride, zo.col_stride, n_rows, n_cols,
                                                          c_out, o, nullptr, acc);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

int pair_ln_linear(const pf_pair_linear_params* p, pf_pair_view zi, pf_pair_view zo, int64_t n_rows, int64_t n_cols,
                   int c_in, int c_out, int acc, int dtype, void* ws, size_t ws_bytes, cudaStream_t st) {
  Arena ar(ws, ws_bytes);
  if (dtype == PF_F32) return pair_ln_linear_t<float>(p, zi, zo, n_rows, n_cols, c_in, c_out, acc, ar, st);
  return pair_ln_linear_t<__nv_bfloat16>(p, zi, zo, n_rows, n_cols, c_in, c_out, acc, ar, st);
}

// ---------------------------------------------------------------- pair heads
// out[p*c + ch] = (LN unless norm = 0)(x(r, s) + (y ? y(r, s) : 0)), fp32; one warp per position
template <class T>
__global__ void k_head_in(const T* __restrict__ x, int64_t rs, int64_t cs, const T* __restrict__ y, int64_t yrs,
                          int64_t ycs, int norm, int64_t n_rows, int64_t n_cols, int c,
                          const float* __restrict__ gamma, const float* __restrict__ beta, float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t pos = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (pos >= n_rows * n_cols) return;
  const int64_t r = pos / n_cols, s = pos - r * n_cols;
  const T* xp = x + r * rs + s * cs;
  const T* yp = y ? y + r * yrs + s * ycs : nullptr;
  constexpr int MAXV = 32;  // c <= 1024
  const int per = (c + 31) / 32;
  float v[MAXV];
  float sum = 0.f;
#pragma unroll
  for (int t = 0; t < MAXV; ++t) {
    if (t < per) {
      const int ch = t * 32 + lane;
      v[t] = ch < c ? to_f(xp[ch]) + (yp ? to_f(yp[ch]) : 0.f) : 0.f;
      sum += v[t];
    }
  }
  float mean = 0.f, rstd = 1.f;
  if (norm) {
    mean = warp_sum(sum) / (float)c;
    float sq = 0.f;
#pragma unroll
    for (int t = 0; t < MAXV; ++t) {
      if (t < per) {
        const int ch = t * 32 + lane;
        const float d = ch < c ? v[t] - mean : 0.f;
        sq += d * d;
      }
    }
    rstd = 1.0f / sqrtf(warp_sum(sq) / (float)c + 1e-5f);
  }
  float* op = out + pos * c;
#pragma unroll
  for (int t = 0; t < MAXV; ++t) {
    if (t < per) {
      const int ch = t * 32 + lane;
      if (ch < c) {
        float o = v[t];
        if (norm) {
          o = (o - mean) * rstd;
          if (gamma) o *= gamma[ch];
          if (beta) o += beta[ch];
        }
        op[ch] = o;
      }
    }
  }
}

// logits(r, s, n) = acc[p*nb + n] + bscale * bias[n]; contact(r, s) = the softmax mass of the
// first cbins bins. One warp per position.
template <class TO>
__global__ void k_head_out(const float* __restrict__ acc, int64_t n_rows, int64_t n_cols, int nb,
                           const float* __restrict__ bias, float bscale, TO* __restrict__ lo, int64_t lrs,
                           int64_t lcs, float* __restrict__ contact, int64_t crs, int64_t ccs, int cbins) {
  const int lane = threadIdx.x & 31;
  const int64_t pos = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (pos >= n_rows * n_cols) return;
  const int64_t r = pos / n_cols, s = pos - r * n_cols;
  const float* ap = acc + pos * nb;
  TO* op = lo + r * lrs + s * lcs;
  float mx = -INFINITY;
  for (int n = lane; n < nb; n += 32) {
    const float y = ap[n] + (bias ? bscale * bias[n] : 0.f);
    op[n] = from_f<TO>(y);
    mx = fmaxf(mx, y);
  }
  if (!contact) return;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float tot = 0.f, sel = 0.f;
  for (int n = lane; n < nb; n += 32) {
    const float e = expf(ap[n] + (bias ? bscale * bias[n] : 0.f) - mx);
    tot += e;
    if (n < cbins) sel += e;
  }
  tot = warp_sum(tot);
  sel = warp_sum(sel);
  if (lane == 0) contact[r * crs + s * ccs] = sel / tot;
}

size_t pair_head_ws_bytes(int64_t n_rows, int64_t n_cols, int c_z, int n_bins) {
  Arena ar(nullptr, 0);
  ar.take<float>((size_t)n_rows * n_cols * c_z);
  ar.take<float>((size_t)n_rows * n_cols * n_bins);
  return ar.used;
}

template <class T>
static int pair_head_t(const pf_pair_head_params* p, int mode, pf_pair_view z, pf_pair_view zt, int64_t n_rows,
                       int64_t n_cols, int c_z, int nb, pf_pair_view lo, int lo_f32, float* contact, int64_t crs,
                       int64_t ccs, int cbins, Arena& ar, cudaStream_t st) {
  const int64_t P = n_rows * n_cols;
  float* a = ar.take<float>((size_t)P * c_z);
  float* acc = ar.take<float>((size_t)P * nb);
  if (!ar.ok()) return fail(PF_EWORKSPACE, "pair head workspace too small");
  if (P == 0) return PF_OK;
  {
    PF_LAUNCH_SCOPE(st, "k_head_in");
    k_head_in<T><<<nblk(P, 8), 256, 0, st>>>((const T*)z.ptr, z.row_stride, z.col_stride,
                                             mode == PF_HEAD_PLAIN ? nullptr : (const T*)zt.ptr, zt.row_stride,
                                             zt.col_stride, mode != PF_HEAD_SYM_OUT, n_rows, n_cols, c_z, p->ln_w,
                                             p->ln_b, a);
  }
  PF_CHECK_LAUNCH();
  PF_TRY((gemm<float, T>(a, 0, c_z, (const T*)p->w, 0, c_z, acc, 0, nb, 1, 1, P, nb, c_z, 1.f, 0, st)));
  const float bscale = mode == PF_HEAD_SYM_OUT ? 2.f : 1.f;
  {
    PF_LAUNCH_SCOPE(st, "k_head_out");
    if (lo_f32)
      k_head_out<float><<<nblk(P, 8), 256, 0, st>>>(acc, n_rows, n_cols, nb, p->b, bscale, (float*)lo.ptr,
                                                    lo.row_stride, lo.col_stride, contact, crs, ccs, cbins);
    else
      k_head_out<T><<<nblk(P, 8), 256, 0, st>>>(acc, n_rows, n_cols, nb, p->b, bscale, (T*)lo.ptr, lo.row_stride,
                                                lo.col_stride, contact, crs, ccs, cbins);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

int pair_head(const pf_pair_head_params* p, int mode, pf_pair_view z, pf_pair_view zt, int64_t n_rows, int64_t n_cols,
              int c_z, int n_bins, pf_pair_view lo, int lo_f32, float* contact, int64_t crs, int64_t ccs, int cbins,
              int dtype, void* ws, size_t ws_bytes, cudaStream_t st) {
  Arena ar(ws, ws_bytes);
  if (dtype == PF_F32)
    return pair_head_t<float>(p, mode, z, zt, n_rows, n_cols, c_z, n_bins, lo, lo_f32, contact, crs, ccs, cbins, ar,
                              st);
  return pair_head_t<__nv_bfloat16>(p, mode, z, zt, n_rows, n_cols, c_z, n_bins, lo, lo_f32, contact, crs, ccs, cbins,
                                    ar, st);
}

// ---------------------------------------------------------------- OuterProductMean
// norm[i*n_cols + j] = sum_s mask(s, row0 + i) mask(s, col0 + j) + eps, 16 x 16 outputs per CTA,
// the mask rows staged 64 sequences at a time (the reference's einsum "...abc,...adc->...bdc").
__global__ void __launch_bounds__(256) k_opm_norm(pf_mask_view m, int64_t n_seq, int64_t row0, int64_t n_rows,
                                                  int64_t col0, int64_t n_cols, float eps, float* __restrict__ norm) {
  __shared__ float mi[64][17], mj[64][17];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t i0 = (int64_t)blockIdx.y * 16, j0 = (int64_t)blockIdx.x * 16;
  float acc = 0.f;
  for (int64_t s0 = 0; s0 < n_seq; s0 += 64) {
    __syncthreads();
    for (int t = threadIdx.x; t < 64 * 16; t += 256) {
      const int ss = t >> 4, e = t & 15;
      const int64_t s = s0 + ss;
      const int64_t i = i0 + e, j = j0 + e;
      mi[ss][e] = (s < n_seq && i < n_rows) ? m.ptr[s * m.row_stride + (row0 + i) * m.col_stride] : 0.f;
      mj[ss][e] = (s < n_seq && j < n_cols) ? m.ptr[s * m.row_stride + (col0 + j) * m.col_stride] : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int ss = 0; ss < 64; ++ss) acc = fmaf(mi[ss][ty], mj[ss][tx], acc);
  }
  const int64_t i = i0 + ty, j = j0 + tx;
  if (i < n_rows && j < n_cols) norm[i * n_cols + j] = acc + eps;
}

int opm_norm(pf_mask_view m, int64_t n_seq, int64_t row0, int64_t n_rows, int64_t col0, int64_t n_cols, float eps,
             float* norm, cudaStream_t st) {
  if ((n_rows + 15) / 16 > 65535) return fail(PF_EUNSUPPORTED, "OuterProductMean: too many rows");
  dim3 grid(nblk(n_cols, 16), nblk(n_rows, 16));
  PF_LAUNCH_SCOPE(st, "k_opm_norm");
  k_opm_norm<<<grid, 256, 0, st>>>(m, n_seq, row0, n_rows, col0, n_cols, eps, norm);
  PF_CHECK_LAUNCH();
  return PF_OK;
}

// aT[(i*C + c)*n_seq + s] *= mask(s, r0 + i)
__global__ void k_opm_mask(float* __restrict__ at, pf_mask_view m, int64_t r0, int64_t n, int C, int64_t n_seq) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n * C * n_seq || m.ptr == nullptr) return;
  const int64_t s = idx % n_seq, i = idx / (n_seq * C);
  at[idx] *= m.ptr[s * m.row_stride + (r0 + i) * m.col_stride];
}

// xr[((i*n_cols + j)*C + c)*C + e] = x[(i*C + c)*(n_cols*C) + j*C + e]
__global__ void k_opm_relayout(const float* __restrict__ x, int64_t n_rows, int64_t n_cols, int C,
                               float* __restrict__ xr) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t cc = (int64_t)C * C;
  if (idx >= n_rows * n_cols * cc) return;
  const int64_t p = idx / cc, k = idx - p * cc;
  const int64_t i = p / n_cols, j = p - i * n_cols;
  const int64_t c = k / C, e = k - c * C;
  xr[idx] = x[(i * C + c) * (n_cols * C) + j * C + e];
}

// z(i, j, n) = (acc ? z : 0) + (y[p*c_z + n] + b[n]) / (norm ? norm[p] : norm_const), p = i*n_cols + j
template <class T>
__global__ void k_opm_out(T* __restrict__ z, int64_t rs, int64_t cs, const float* __restrict__ y,
                          const float* __restrict__ b, const float* __restrict__ norm, float norm_const,
                          int64_t n_rows, int64_t n_cols, int c_z, int acc) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n_rows * n_cols * c_z) return;
  const int64_t p = idx / c_z;
  const int n = (int)(idx - p * c_z);
  const int64_t i = p / n_cols, j = p - i * n_cols;
  const float v = (y[idx] + (b ? b[n] : 0.f)) / (norm ? norm[p] : norm_const);
  T* d = z + i * rs + j * cs + n;
  *d = from_f<T>((acc ? to_f(*d) : 0.f) + v);
}

size_t opm_ws_bytes(int64_t n_seq, int64_t n_res, int64_t n_rows, int64_t n_cols, int c_m, int C, int c_z) {
  Arena ar(nullptr, 0);
  ar.take<float>((size_t)n_res * n_seq * c_m);
  ar.take<float>((size_t)n_rows * C * n_seq);
  ar.take<float>((size_t)n_cols * C * n_seq);
  ar.take<float>((size_t)n_rows * C * n_cols * C);
  ar.take<float>((size_t)n_rows * n_cols * C * C);
  ar.take<float>((size_t)n_rows * n_cols * c_z);
  ar.take<float>((size_t)n_rows * n_cols);
  return ar.used;
}

template <class T>
static int opm_t(const pf_opm_params* p, pf_pair_view m, pf_mask_view mask, pf_pair_view zo, int64_t S, int64_t N,
                 int64_t row0, int64_t nr, int64_t col0, int64_t nc, int c_m, int C, int c_z, float eps, int acc,
                 Arena& ar, cudaStream_t st) {
  float* ln = ar.take<float>((size_t)N * S * c_m);
  float* at = ar.take<float>((size_t)nr * C * S);
  float* bt = ar.take<float>((size_t)nc * C * S);
  float* x = ar.take<float>((size_t)nr * C * nc * C);
  float* xr = ar.take<float>((size_t)nr * nc * C * C);
  float* y = ar.take<float>((size_t)nr * nc * c_z);
  float* norm = ar.take<float>((size_t)nr * nc);
  if (!ar.ok()) return fail(PF_EWORKSPACE, "OuterProductMean workspace too small");
  // LN over the (i, s) order of the positions, so that a residue's sequences are contiguous
  PF_TRY((ln_view<T, float>((const T*)m.ptr, m.col_stride, m.row_stride, N, S, c_m, p->ln_w, p->ln_b, 1e-5f, ln,
                            c_m, st)));
  // aT[(i*C + c)*S + s] = linear_1(ln(s, row0 + i))[c]; the same for bT with linear_2
  PF_TRY((gemm<float, T>(ln + row0 * S * c_m, S * c_m, c_m, (const T*)p->w_1, 0, c_m, at, (int64_t)C * S, 1, S, nr,
                         S, C, c_m, 1.f, 0, st)));
  PF_TRY((gemm<float, T>(ln + col0 * S * c_m, S * c_m, c_m, (const T*)p->w_2, 0, c_m, bt, (int64_t)C * S, 1, S, nc,
                         S, C, c_m, 1.f, 0, st)));
  {
    PF_LAUNCH_SCOPE(st, "k_opm_mask");
    k_opm_mask<<<nblk(nr * C * S, 256), 256, 0, st>>>(at, mask, row0, nr, C, S);
  }
  PF_CHECK_LAUNCH();
  {
    PF_LAUNCH_SCOPE(st, "k_opm_mask");
    k_opm_mask<<<nblk(nc * C * S, 256), 256, 0, st>>>(bt, mask, col0, nc, C, S);
  }
  PF_CHECK_LAUNCH();
  // x[(i, c)][(j, e)] = sum_s aT[(i, c)][s] bT[(j, e)][s]
  PF_TRY((gemm<float, float>(at, 0, S, bt, 0, S, x, 0, nc * C, 1, 1, nr * C, nc * C, S, 1.f, 0, st)));
  {
    PF_LAUNCH_SCOPE(st, "k_opm_relayout");
    k_opm_relayout<<<nblk(nr * nc * C * C, 256), 256, 0, st>>>(x, nr, nc, C, xr);
  }
  PF_CHECK_LAUNCH();
  PF_TRY((gemm<float, T>(xr, 0, (int64_t)C * C, (const T*)p->w_out, 0, (int64_t)C * C, y, 0, c_z, 1, 1, nr * nc, c_z,
                         (int64_t)C * C, 1.f, 0, st)));
  if (mask.ptr) PF_TRY(opm_norm(mask, S, row0, nr, col0, nc, eps, norm, st));
  {
    PF_LAUNCH_SCOPE(st, "k_opm_out");
    k_opm_out<T><<<nblk(nr * nc * c_z, 256), 256, 0, st>>>((T*)zo.ptr, zo.row_stride, zo.col_stride, y, p->b_out,
                                                          mask.ptr ? norm : nullptr, (float)S + eps, nr, nc, c_z,
                                                          acc);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

int opm(const pf_opm_params* p, pf_pair_view m, pf_mask_view mask, pf_pair_view z_out, int64_t n_seq, int64_t n_res,
        int64_t row0, int64_t n_rows, int64_t col0, int64_t n_cols, int c_m, int C, int c_z, float eps, int acc,
        int dtype, void* ws, size_t ws_bytes, cudaStream_t st) {
  Arena ar(ws, ws_bytes);
  if (dtype == PF_F32)
    return opm_t<float>(p, m, mask, z_out, n_seq, n_res, row0, n_rows, col0, n_cols, c_m, C, c_z, eps, acc, ar, st);
  return opm_t<__nv_bfloat16>(p, m, mask, z_out, n_seq, n_res, row0, n_rows, col0, n_cols, c_m, C, c_z, eps, acc, ar,
                              st);
}

}  // namespace simt
}  // namespace pf
