// pf_tc_triatt.cu -- triangle attention (starting node; the ending node is the same code on
// transposed views) on tcgen05 tensor cores. c = 128, H = 4, d = 32.
//
// Kernels (intermediates in the caller's workspace):
//   k_triatt_maskprep : per row i, the log2-domain key bias inf*(m-1)*log2(e) (or -inf for keys
//                       that do not exist), and a per-128-key-tile flag: no bias add needed /
//                       add per element / skip the tile (every key masked while the row has a
//                       fully valid key, so exp() underflows to exactly 0 in the reference too).
//   k_triatt_proj     : TMA tile of 128 positions -> LayerNorm in place -> one UMMA chain into
//                       512 TMEM columns: [q | k] (N=256) and [v | bias] (N=144). q is stored
//                       pre-scaled by log2(e)/sqrt(d); v transposed (keys contiguous, f16) so the
//                       P.V MMA reads it K-major; the triangle bias in log2 units.
//   k_triatt_core     : one CTA per (row i, head h, 128 queries). Per 128-key tile: S = Q K^T
//                       (UMMA, TMEM), softmax in registers (one thread per query, exp2), P in f16
//                       to shared memory, then [o | l] = P [V^T ; 1]^T in one UMMA (the ones row
//                       gives the row sum of exactly the f16 P used for o).
//   k_triatt_out      : persistent; LN(z) -> gate logits (UMMA), o * sigmoid(gate) -> W_o (UMMA)
//                       -> residual, TMA-stored.
// Reference: opendde/model/triangular/triangular.py:648-706, layers.py:302-424.

#include "pf_common.cuh"
#include "pf_prof.h"
#include "pf_sm100.cuh"
#include "pf_tc.h"
#include "pf_tc_internal.h"
#include "pf_tile_common.cuh"
#include "pf_tmap.h"

namespace pf {
namespace tc {
using namespace sm100;

namespace {

constexpr int CH = 128, H = 4, D = 32, HD = 128, TILE = 128;
constexpr float LOG2E = 1.4426950408889634f;

enum TileFlag : uint8_t { TF_NOADD = 0, TF_ADD = 1, TF_SKIP = 2 };

// ------------------------------------------------------------------ mask prep
// Key bias per row in f16 log2 units: 0 for a key with mask >= 1, -inf for a masked key (the
// reference's inf*(m-1) with inf = 1e9 sends it to exactly zero weight next to any valid key)
// and for keys that do not exist. A row with no key of mask 1 is a "uniform" row: the
// reference's logits are all ~ -1e9 there and its softmax is the uniform average over the
// keys, so its bias is 0 on existing keys and the core ignores the logits (rowflags bit 0).
__global__ void k_triatt_maskprep(pf_mask_view m, int64_t n_keys, int64_t n_valid, float inf,
                                  __half* __restrict__ mb, int64_t ld_mb, uint8_t* __restrict__ flags,
                                  uint8_t* __restrict__ rowflags, int n_tiles) {
  const int64_t i = blockIdx.x;
  const int tid = threadIdx.x;  // 128 threads
  __shared__ int s_any_full;
  if (tid == 0) s_any_full = 0;
  __syncthreads();
  int any_full = 0;
  for (int64_t k = tid; k < n_valid; k += 128) {
    const float mv = m.ptr ? m.ptr[i * m.row_stride + k * m.col_stride] : 1.0f;
    any_full |= (mv >= 1.0f);
  }
  if (any_full) atomicOr(&s_any_full, 1);
  __syncthreads();
  const bool row_full = s_any_full != 0;
  if (tid == 0) rowflags[i] = row_full ? 0 : 1;
  for (int kt = 0; kt < n_tiles; ++kt) {
    const int64_t k = (int64_t)kt * 128 + tid;
    float mv = 0.f;
    const bool exists = k < n_valid;
    if (exists) mv = m.ptr ? m.ptr[i * m.row_stride + k * m.col_stride] : 1.0f;
    const bool live = exists && (mv >= 1.0f || !row_full);
    mb[i * ld_mb + k] = live ? __float2half_rn(0.f) : __float2half_rn(-INFINITY);
    const int all_live = __syncthreads_and(live);
    const int all_dead = __syncthreads_and(!live);
    if (tid == 0) flags[i * n_tiles + kt] = all_dead ? TF_SKIP : (all_live ? TF_NOADD : TF_ADD);
  }
}

// ------------------------------------------------------------------ projection
// Persistent, one CTA per SM; tile k of a CTA goes to compute warpgroup k & 1 (its own z
// stage and 256 TMEM columns). Per tile: LN(z) in place, then two UMMA chains into the same
// columns: [q | k] (N = 256), and after the warpgroup has read them, [v | bias] (N = 144).
// q, k (f16, 64 B per head and position) and the bias are stored directly; v^T is transposed
// into the stage as [(h, d)][key] and TMA-stored.
struct ProjArgs {
  int64_t n_rows, n_keys, tiles_per_row, n_tiles;
  int64_t q_col0, n_q;
  int want_qkv, want_bias;
  __half* q;          // [(i*H+h)*n_q + j][D]     f16, x log2(e)/sqrt(d)
  __half* k;          // [(i*H+h)*ld_keys + key][D] f16
  __half* bias;       // bias + h*b_hs + r*b_rs + s (f16, log2 units)
  int64_t ld_keys, b_hs, b_rs;
  const float *ln_w, *ln_b;
  float q_scale;
  unsigned int* status;
};

constexpr uint32_t PB_ATOM = 400 * 128;               // 400 weight rows x 128 B per K atom
constexpr uint32_t PJ_STAGE = 2 * PB_ATOM, PJ_STAGE_BYTES = 32768;
constexpr uint32_t PJ_LN = PJ_STAGE + 2 * PJ_STAGE_BYTES, PJ_BAR = PJ_LN + 1024;
constexpr uint32_t PROJ_SMEM = PJ_BAR + 256;

__global__ void __launch_bounds__(320, 1) k_triatt_proj(const __grid_constant__ CUtensorMap tz,
                                                        const __grid_constant__ CUtensorMap twq,
                                                        const __grid_constant__ CUtensorMap twk,
                                                        const __grid_constant__ CUtensorMap twv,
                                                        const __grid_constant__ CUtensorMap twb,
                                                        const __grid_constant__ CUtensorMap tvt,
                                                        const ProjArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* g = smem_raw + (base - raw);
  const uint32_t bars = base + PJ_BAR, wbar = bars;
  auto full = [&](int w) { return bars + 8 + 8 * w; };
  auto empty = [&](int w) { return bars + 24 + 8 * w; };
  auto ready = [&](int w) { return bars + 40 + 8 * w; };
  auto done_a = [&](int w) { return bars + 56 + 8 * w; };
  auto tfree = [&](int w) { return bars + 72 + 8 * w; };
  auto done_b = [&](int w) { return bars + 88 + 8 * w; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(g + PJ_BAR + 128);
  float* lnp = reinterpret_cast<float*>(g + PJ_LN);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    mbar_init(wbar, 1);
    for (int w = 0; w < 2; ++w) {
      mbar_init(full(w), 1);
      mbar_init(empty(w), 1);
      mbar_init(ready(w), 1);
      mbar_init(done_a(w), 1);
      mbar_init(tfree(w), 1);
      mbar_init(done_b(w), 1);
    }
    mbar_init(bars + 104, 1);
    fence_barrier_init();
  }
  for (int c = tid; c < CH; c += blockDim.x) {
    lnp[c] = a.ln_w[c];
    lnp[CH + c] = a.ln_b[c];
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int64_t G = gridDim.x;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tz);
      mbar_arrive_expect_tx(wbar, 2 * PB_ATOM);
#pragma unroll
      for (int at = 0; at < 2; ++at) {
        const uint32_t b0 = base + at * PB_ATOM;
        tma_load_2d(b0, &twq, wbar, at * 64, 0);
        tma_load_2d(b0 + 128 * 128, &twk, wbar, at * 64, 0);
        tma_load_2d(b0 + 256 * 128, &twv, wbar, at * 64, 0);
        tma_load_2d(b0 + 384 * 128, &twb, wbar, at * 64, 0);  // 16 rows, rows >= H read 0
      }
      for (int64_t k = 0;; ++k) {
        const int64_t t = blockIdx.x + k * G;
        if (t >= a.n_tiles) break;
        const int w = (int)(k & 1);
        const int64_t n = k >> 1;
        if (n > 0) mbar_wait(empty(w), (uint32_t)((n - 1) & 1), a.status);
        const int r = (int)(t / a.tiles_per_row);
        const int c0 = (int)((t % a.tiles_per_row) * TILE);
        const uint32_t st = base + PJ_STAGE + w * PJ_STAGE_BYTES;
        mbar_arrive_expect_tx(full(w), 32768);
        tma_load_3d(st, &tz, full(w), 0, c0, r);
        tma_load_3d(st + 16384, &tz, full(w), 64, c0, r);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      mbar_wait(wbar, 0, a.status);
      for (int64_t k = 0;; ++k) {
        const int64_t t = blockIdx.x + k * G;
        if (t >= a.n_tiles) break;
        const int w = (int)(k & 1);
        const uint32_t par = (uint32_t)((k >> 1) & 1);
        const uint32_t sA = base + PJ_STAGE + w * PJ_STAGE_BYTES;
        mbar_wait(ready(w), par, a.status);
        tc_fence_after();
        tile::umma_k128(tmem + w * 256, sA, base, PB_ATOM, idesc_f16(128, 256, true));              // q | k
        umma_commit(done_a(w));
        mbar_wait(tfree(w), par, a.status);
        tc_fence_after();
        tile::umma_k128(tmem + w * 256, sA, base + 256 * 128, PB_ATOM, idesc_f16(128, 144, true));  // v | bias
        umma_commit(done_b(w));
      }
      umma_commit(bars + 104);  // drain: every MMA complete before TMEM is released
      mbar_wait_drain(bars + 104, 0);
    }
  } else {
    const int wg = (warp - 2) >> 2;
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const bool leader = (warp == 2 + 4 * wg) && lane == 0;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    uint8_t* zt = g + PJ_STAGE + wg * PJ_STAGE_BYTES;
    const uint32_t st = base + PJ_STAGE + wg * PJ_STAGE_BYTES;
    const uint32_t tm = tmem + lane_base + wg * 256;
    for (int64_t k = wg;; k += 2) {
      const int64_t t = blockIdx.x + k * G;
      if (t >= a.n_tiles) break;
      const uint32_t par = (uint32_t)((k >> 1) & 1);
      const int r = (int)(t / a.tiles_per_row);
      const int c0 = (int)((t % a.tiles_per_row) * TILE);
      mbar_wait(full(wg), par, a.status);
      {
        uint32_t zr[64];
        float m, rs;
        tile::load_row(zt, row, zr);
        tile::row_stats(zr, 1e-5f, m, rs);
        tile::store_norm_row(zt, row, zr, m, rs, lnp, lnp + CH);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      named_bar_sync(1 + wg, 128);
      if (leader) mbar_arrive(ready(wg));
      const int64_t col = (int64_t)c0 + row;
      const bool valid = col < a.n_keys && a.want_qkv;
      const int64_t jq = col - a.q_col0;
      const bool qvalid = valid && jq >= 0 && jq < a.n_q;
      mbar_wait(done_a(wg), par, a.status);
      tc_fence_after();
#pragma unroll 1
      for (int h = 0; h < H; ++h) {
        uint32_t qv[32], kv[32];
        tmem_ld32(tm + h * D, qv);
        tmem_ld32(tm + 128 + h * D, kv);
        tmem_ld_wait();
        if (qvalid) {
          uint4* dq = reinterpret_cast<uint4*>(a.q + (((int64_t)r * H + h) * a.n_q + jq) * D);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            uint4 w4;
            w4.x = pack_f16(__uint_as_float(qv[e * 8 + 0]) * a.q_scale, __uint_as_float(qv[e * 8 + 1]) * a.q_scale);
            w4.y = pack_f16(__uint_as_float(qv[e * 8 + 2]) * a.q_scale, __uint_as_float(qv[e * 8 + 3]) * a.q_scale);
            w4.z = pack_f16(__uint_as_float(qv[e * 8 + 4]) * a.q_scale, __uint_as_float(qv[e * 8 + 5]) * a.q_scale);
            w4.w = pack_f16(__uint_as_float(qv[e * 8 + 6]) * a.q_scale, __uint_as_float(qv[e * 8 + 7]) * a.q_scale);
            dq[e] = w4;
          }
        }
        if (valid) {
          uint4* dk = reinterpret_cast<uint4*>(a.k + (((int64_t)r * H + h) * a.ld_keys + col) * D);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            uint4 w4;
            w4.x = pack_f16(__uint_as_float(kv[e * 8 + 0]), __uint_as_float(kv[e * 8 + 1]));
            w4.y = pack_f16(__uint_as_float(kv[e * 8 + 2]), __uint_as_float(kv[e * 8 + 3]));
            w4.z = pack_f16(__uint_as_float(kv[e * 8 + 4]), __uint_as_float(kv[e * 8 + 5]));
            w4.w = pack_f16(__uint_as_float(kv[e * 8 + 6]), __uint_as_float(kv[e * 8 + 7]));
            dk[e] = w4;
          }
        }
      }
      tc_fence_before();
      named_bar_sync(1 + wg, 128);
      if (leader) mbar_arrive(tfree(wg));
      mbar_wait(done_b(wg), par, a.status);
      tc_fence_after();
      // v^T staged as [(h, d)][key] over the consumed z tile
      unsigned short* vs = reinterpret_cast<unsigned short*>(zt);
#pragma unroll
      for (int cc = 0; cc < HD; cc += 16) {
        uint32_t vv[16];
        tmem_ld16(tm + cc, vv);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 16; ++e) vs[(cc + e) * TILE + row] = __half_as_ushort(__float2half_rn(__uint_as_float(vv[e])));
      }
      {
        uint32_t bv[16];
        tmem_ld16(tm + HD, bv);
        tmem_ld_wait();
        if (a.want_bias && col < a.n_keys) {
#pragma unroll
          for (int h = 0; h < H; ++h)
            a.bias[h * a.b_hs + (int64_t)r * a.b_rs + col] = __float2half_rn(__uint_as_float(bv[h]) * LOG2E);
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      named_bar_sync(1 + wg, 128);
      if (leader) {
        if (a.want_qkv) {
          tma_store_2d(&tvt, st, c0, r * HD);
          bulk_commit_group();
          bulk_wait_group_read0();
        }
        mbar_arrive(empty(wg));
      }
    }
    if (leader) bulk_wait_group0();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ core
#include "pf_triatt_core.cuh"

// ------------------------------------------------------------------ output
// Persistent, one CTA per SM; tile k of a CTA goes to compute warpgroup k & 1, which owns
// shared-memory stage k & 1 (z tile + o tile) and TMEM columns [256 w, 256 w + 256).
//   warp 0     TMA producer (W_g, W_o once; z and o tiles per tile)
//   warp 1     MMA issuer: gate = W_g LN(z) (cols +128), then y = W_o (o * sigmoid(gate)) (cols +0)
//   warps 2-9  LN(z) in place; o * sigmoid(gate) in place; y (+ residual read from zo, fetched
//              while the W_o GEMM runs) written into the z buffer and TMA-stored to zo.
struct OutArgs {
  int64_t n_rows, n_q, tiles_per_row, n_tiles, q_col0;
  const __nv_bfloat16* zo;
  int64_t zo_rs, zo_cs;
  const float *ln_w, *ln_b;
  int accumulate;
  unsigned int* status;
};
constexpr uint32_t O_WG = 0, O_WO = 32768, O_STAGE = 65536, O_STAGE_BYTES = 65536;
constexpr uint32_t O_LN = O_STAGE + 2 * O_STAGE_BYTES, O_BAR = O_LN + 1024;
constexpr uint32_t OUT_SMEM = O_BAR + 256;

__global__ void __launch_bounds__(320, 1) k_triatt_out(const __grid_constant__ CUtensorMap tz,
                                                       const __grid_constant__ CUtensorMap to,
                                                       const __grid_constant__ CUtensorMap tzo,
                                                       const __grid_constant__ CUtensorMap twg,
                                                       const __grid_constant__ CUtensorMap two,
                                                       const OutArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* g = smem_raw + (base - raw);
  const uint32_t bars = base + O_BAR, wbar = bars;
  auto full = [&](int w) { return bars + 8 + 8 * w; };
  auto empty = [&](int w) { return bars + 24 + 8 * w; };
  auto rg = [&](int w) { return bars + 40 + 8 * w; };
  auto ro = [&](int w) { return bars + 56 + 8 * w; };
  auto mg = [&](int w) { return bars + 72 + 8 * w; };
  auto mo = [&](int w) { return bars + 88 + 8 * w; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(g + O_BAR + 128);
  float* lnp = reinterpret_cast<float*>(g + O_LN);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    mbar_init(wbar, 1);
    for (int w = 0; w < 2; ++w) {
      mbar_init(full(w), 1);
      mbar_init(empty(w), 1);
      mbar_init(rg(w), 1);
      mbar_init(ro(w), 1);
      mbar_init(mg(w), 1);
      mbar_init(mo(w), 1);
    }
    mbar_init(bars + 104, 1);
    fence_barrier_init();
  }
  for (int c = tid; c < CH; c += blockDim.x) {
    lnp[c] = a.ln_w[c];
    lnp[CH + c] = a.ln_b[c];
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int64_t G = gridDim.x;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tz);
      tma_prefetch_desc(&to);
      mbar_arrive_expect_tx(wbar, 65536);
      tma_load_2d(base + O_WG, &twg, wbar, 0, 0);
      tma_load_2d(base + O_WG + 16384, &twg, wbar, 64, 0);
      tma_load_2d(base + O_WO, &two, wbar, 0, 0);
      tma_load_2d(base + O_WO + 16384, &two, wbar, 64, 0);
      for (int64_t k = 0;; ++k) {
        const int64_t t = blockIdx.x + k * G;
        if (t >= a.n_tiles) break;
        const int w = (int)(k & 1);
        const int64_t n = k >> 1;
        if (n > 0) mbar_wait(empty(w), (uint32_t)((n - 1) & 1), a.status);
        const int i = (int)(t / a.tiles_per_row);
        const int j0 = (int)((t % a.tiles_per_row) * TILE);
        const uint32_t st = base + O_STAGE + w * O_STAGE_BYTES;
        mbar_arrive_expect_tx(full(w), 65536);
        tma_load_3d(st, &tz, full(w), 0, (int)(a.q_col0 + j0), i);
        tma_load_3d(st + 16384, &tz, full(w), 64, (int)(a.q_col0 + j0), i);
        tma_load_3d(st + 32768, &to, full(w), 0, j0, i);
        tma_load_3d(st + 49152, &to, full(w), 64, j0, i);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      mbar_wait(wbar, 0, a.status);
      for (int64_t k = 0;; ++k) {
        const int64_t t = blockIdx.x + k * G;
        if (t >= a.n_tiles) break;
        const int w = (int)(k & 1);
        const uint32_t par = (uint32_t)((k >> 1) & 1);
        const uint32_t sZ = base + O_STAGE + w * O_STAGE_BYTES, sO = sZ + 32768;
        mbar_wait(rg(w), par, a.status);
        tc_fence_after();
        tile::umma_k128(tmem + w * 256 + 128, sZ, base + O_WG, 16384, idesc_f16(128, 128, true));
        umma_commit(mg(w));
        mbar_wait(ro(w), par, a.status);
        tc_fence_after();
        tile::umma_k128(tmem + w * 256, sO, base + O_WO, 16384, idesc_f16(128, 128, true));
        umma_commit(mo(w));
      }
      umma_commit(bars + 104);  // drain: every MMA complete before TMEM is released
      mbar_wait_drain(bars + 104, 0);
    }
  } else {
    const int wg = (warp - 2) >> 2;
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const bool leader = (warp == 2 + 4 * wg) && lane == 0;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    uint8_t* zt = g + O_STAGE + wg * O_STAGE_BYTES;
    uint8_t* ot = zt + 32768;
    const uint32_t st = base + O_STAGE + wg * O_STAGE_BYTES;
    for (int64_t k = wg;; k += 2) {
      const int64_t t = blockIdx.x + k * G;
      if (t >= a.n_tiles) break;
      const uint32_t par = (uint32_t)((k >> 1) & 1);
      const int i = (int)(t / a.tiles_per_row);
      const int j0 = (int)((t % a.tiles_per_row) * TILE);
      mbar_wait(full(wg), par, a.status);
      {
        uint32_t zr[64];
        float m, r;
        tile::load_row(zt, row, zr);
        tile::row_stats(zr, 1e-5f, m, r);
        tile::store_norm_row(zt, row, zr, m, r, lnp, lnp + CH);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      named_bar_sync(1 + wg, 128);
      if (leader) mbar_arrive(rg(wg));
      mbar_wait(mg(wg), par, a.status);
      tc_fence_after();
      // o * sigmoid(gate), in place in the o tile
#pragma unroll
      for (int cc = 0; cc < HD; cc += 16) {
        uint32_t gv[16];
        tmem_ld16(tmem + lane_base + wg * 256 + 128 + cc, gv);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          uint4* p = reinterpret_cast<uint4*>(ot + tile::chunk_off(row, (cc >> 3) + e));
          uint4 v = *p;
          const float* gg = reinterpret_cast<const float*>(gv) + e * 8;
          v.x = pack_bf16(bf16lo(v.x) * fast_sigmoid(gg[0]), bf16hi(v.x) * fast_sigmoid(gg[1]));
          v.y = pack_bf16(bf16lo(v.y) * fast_sigmoid(gg[2]), bf16hi(v.y) * fast_sigmoid(gg[3]));
          v.z = pack_bf16(bf16lo(v.z) * fast_sigmoid(gg[4]), bf16hi(v.z) * fast_sigmoid(gg[5]));
          v.w = pack_bf16(bf16lo(v.w) * fast_sigmoid(gg[6]), bf16hi(v.w) * fast_sigmoid(gg[7]));
          *p = v;
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      named_bar_sync(1 + wg, 128);
      if (leader) mbar_arrive(ro(wg));
      const int64_t j = (int64_t)j0 + row;
      const bool rd = a.accumulate && j < a.n_q;
      const uint4* zp = reinterpret_cast<const uint4*>(a.zo + (int64_t)i * a.zo_rs + (rd ? j : 0) * a.zo_cs);
      uint4 old[16];
#pragma unroll
      for (int c = 0; c < 8; ++c) old[c] = rd ? __ldg(zp + c) : make_uint4(0, 0, 0, 0);
      mbar_wait(mo(wg), par, a.status);
      tc_fence_after();
#pragma unroll
      for (int c = 8; c < 16; ++c) old[c] = rd ? __ldg(zp + c) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int cc = 0; cc < CH; cc += 16) {
        uint32_t ov[16];
        tmem_ld16(tmem + lane_base + wg * 256 + cc, ov);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int chunk = (cc >> 3) + e;
          const uint4 o = old[chunk];
          float u[8];
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) u[kk] = __uint_as_float(ov[e * 8 + kk]);
          u[0] += bf16lo(o.x); u[1] += bf16hi(o.x); u[2] += bf16lo(o.y); u[3] += bf16hi(o.y);
          u[4] += bf16lo(o.z); u[5] += bf16hi(o.z); u[6] += bf16lo(o.w); u[7] += bf16hi(o.w);
          uint4 wv;
          wv.x = pack_bf16(u[0], u[1]); wv.y = pack_bf16(u[2], u[3]);
          wv.z = pack_bf16(u[4], u[5]); wv.w = pack_bf16(u[6], u[7]);
          *reinterpret_cast<uint4*>(zt + tile::chunk_off(row, chunk)) = wv;
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      named_bar_sync(1 + wg, 128);
      if (leader) {
        tma_store_3d(&tzo, st, 0, j0, i);
        tma_store_3d(&tzo, st + 16384, 64, j0, i);
        bulk_commit_group();
        bulk_wait_group_read0();
        mbar_arrive(empty(wg));
      }
    }
    if (leader) bulk_wait_group0();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ host
int pair_tmap(CUtensorMap* m, const void* ptr, int64_t rs, int64_t cs, int64_t n_rows, int64_t n_cols) {
  if (rs % 8 || cs % 8)
    return fail(PF_EINVAL_SHAPE, "bf16 pair views need row/col strides that are multiples of 8 elements");
  const uint64_t dims[3] = {(uint64_t)CH, (uint64_t)n_cols, (uint64_t)n_rows};
  const uint64_t str[2] = {(uint64_t)cs * 2, (uint64_t)rs * 2};
  const uint32_t box[3] = {64, (uint32_t)TILE, 1};
  return make_tmap(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, ptr, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

int weight_tmap(CUtensorMap* m, const void* w, int rows, int cols, int box_rows) {
  const uint64_t dims[2] = {(uint64_t)cols, (uint64_t)rows};
  const uint64_t str[1] = {(uint64_t)cols * 2};
  const uint32_t box[2] = {64, (uint32_t)box_rows};
  return make_tmap(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

int64_t num_sms() { return sm_count(); }

template <class K>
int set_smem(K kernel, uint32_t bytes) {
  PF_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
  return PF_OK;
}

// Dynamic shared-memory limits, set once on every device that runs these kernels.
int ensure_attrs() {
  static std::atomic<unsigned long long> done{0};
  return once_per_device(done, []() -> int {
    PF_TRY(set_smem(k_triatt_proj, PROJ_SMEM + 1024));
    PF_TRY(set_smem(k_triatt_core<H>, CORE3_SMEM + 1024));
    PF_TRY(set_smem(k_triatt_core<0>, CORE3_SMEM + 1024));
    PF_TRY(set_smem(k_triatt_out, OUT_SMEM + 1024));
    return PF_OK;
  });
}

struct TriattWs {
  __half *q, *k;
  __nv_bfloat16* o;
  __half *vt, *bias, *mb;
  uint8_t *flags, *rowflags;
  int64_t ld_keys, ld_mb, n_tiles_k;
};

void triatt_plan(Arena& ar, int64_t n_rows, int64_t n_keys, int64_t n_q, bool own_bias, TriattWs& w) {
  w.ld_keys = (n_keys + 7) / 8 * 8;
  w.n_tiles_k = (n_keys + TILE - 1) / TILE;
  w.ld_mb = w.n_tiles_k * TILE;
  w.q = ar.take<__half>((size_t)n_rows * H * n_q * D);
  w.k = ar.take<__half>((size_t)n_rows * H * w.ld_keys * D);
  w.vt = ar.take<__half>((size_t)n_rows * H * D * w.ld_keys);
  w.bias = own_bias ? ar.take<__half>((size_t)H * n_q * w.ld_keys) : nullptr;
  w.o = ar.take<__nv_bfloat16>((size_t)n_rows * n_q * HD);
  w.mb = ar.take<__half>((size_t)n_rows * w.ld_mb);
  w.flags = ar.take<uint8_t>((size_t)n_rows * w.n_tiles_k);
  w.rowflags = ar.take<uint8_t>((size_t)n_rows);
}

int launch_proj(const pf_triatt_params* p, const void* zptr, int64_t rs, int64_t cs, int64_t n_rows,
                int64_t n_cols, ProjArgs pa, __half* vt, cudaStream_t st) {
  CUtensorMap tz, twq, twk, twv, twb, tvt;
  PF_TRY(pair_tmap(&tz, zptr, rs, cs, n_rows, n_cols));
  PF_TRY(weight_tmap(&twq, p->w_q, HD, CH, 128));
  PF_TRY(weight_tmap(&twk, p->w_k, HD, CH, 128));
  PF_TRY(weight_tmap(&twv, p->w_v, HD, CH, 128));
  PF_TRY(weight_tmap(&twb, p->w_bias, H, CH, 16));
  if (vt) {
    const uint64_t dv[2] = {(uint64_t)n_cols, (uint64_t)n_rows * HD};
    const uint64_t sv[1] = {(uint64_t)pa.ld_keys * 2};
    const uint32_t bv[2] = {(uint32_t)TILE, (uint32_t)HD};
    PF_TRY(make_tmap(&tvt, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, vt, dv, sv, bv, CU_TENSOR_MAP_SWIZZLE_NONE));
  } else {
    tvt = tz;  // unused (no q/k/v wanted)
  }
  pa.tiles_per_row = (n_cols + TILE - 1) / TILE;
  pa.n_tiles = n_rows * pa.tiles_per_row;
  {
    const int64_t grid_p = pa.n_tiles < num_sms() ? pa.n_tiles : num_sms();
    // read z; write q (queries), k and v^T (all keys) and / or the bias (f16)
    const double pos = (double)n_rows * n_cols;
    double bytes = 2.0 * pos * CH;
    if (pa.want_qkv) bytes += 2.0 * ((double)n_rows * pa.n_q * HD + 2.0 * pos * HD);
    if (pa.want_bias) bytes += 2.0 * H * (pa.want_qkv ? (double)pa.n_q * n_cols : pos);
    PF_LAUNCH_SCOPE_WORK(st, "k_triatt_proj", bytes, 'b');
    k_triatt_proj<<<(unsigned)grid_p, 320, PROJ_SMEM + 1024, st>>>(tz, twq, twk, twv, twb, tvt, pa);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

}  // namespace

bool triatt_bias_supported(int c, int heads) { return c == CH && heads == H; }
bool triatt_supported(int c, int heads, int d) { return c == CH && heads == H && d == D; }

size_t triatt_ws_bytes(int64_t n_rows, int64_t n_keys, int64_t n_q, int, int, int) {
  Arena ar(nullptr, 0);
  TriattWs w;
  triatt_plan(ar, n_rows, n_keys, n_q, true, w);
  return ar.used;
}

int triatt_bias(const pf_triatt_params* p, pf_pair_view z, int64_t n_rows, int64_t n_cols, void* bias,
                int64_t hs, int64_t rs, int, int, cudaStream_t st) {
  PF_TRY(ensure_attrs());
  unsigned int* status;
  PF_TRY(device_status_ptr(&status));
  ProjArgs pa{};
  pa.n_rows = n_rows;
  pa.n_keys = n_cols;
  pa.q_col0 = 0;
  pa.n_q = 0;
  pa.want_qkv = 0;
  pa.want_bias = 1;
  pa.bias = (__half*)bias;
  pa.b_hs = hs;
  pa.b_rs = rs;
  pa.ln_w = p->ln_w;
  pa.ln_b = p->ln_b;
  pa.status = status;
  return launch_proj(p, z.ptr, z.row_stride, z.col_stride, n_rows, n_cols, pa, nullptr, st);
}

int triatt(const pf_triatt_params* p, pf_pair_view zs, pf_mask_view m, const void* bias, int64_t b_hs,
           int64_t b_rs, pf_pair_view zo, int64_t n_rows, int64_t n_keys, int64_t n_valid, int64_t q_col0,
           int64_t n_q, int, int, int, float inf, int acc, void* ws, size_t ws_bytes, cudaStream_t st) {
  Arena ar(ws, ws_bytes);
  TriattWs w;
  triatt_plan(ar, n_rows, n_keys, n_q, bias == nullptr, w);
  if (!ar.ok()) return fail(PF_EWORKSPACE, "triatt workspace too small");
  if (zo.row_stride % 8 || zo.col_stride % 8 || ((uintptr_t)zo.ptr) % 16)
    return fail(PF_EINVAL_SHAPE, "bf16 output view must be 16-byte aligned with strides multiple of 8");
  if (bias != nullptr && (b_hs % 8 || b_rs % 8 || ((uintptr_t)bias) % 16))
    return fail(PF_EINVAL_SHAPE, "bias buffer must be 16-byte aligned with strides multiple of 8");
  if (n_rows * H > 0x7fffffffll || w.n_tiles_k > 0x7fffffffll)
    return fail(PF_EUNSUPPORTED, "triatt problem too large");
  PF_TRY(ensure_attrs());
  unsigned int* status;
  PF_TRY(device_status_ptr(&status));
  // 0. mask bias + tile flags
  const CoreIO io{w.q, w.k, w.vt, nullptr, 0, 0, w.o, w.mb, w.flags, w.rowflags, w.ld_keys, w.ld_mb, w.n_tiles_k};
  PF_TRY(triatt_masks(m, n_rows, n_keys, n_valid, inf, io, st));
  // 1. projections (+ own bias in the square single-device case)
  ProjArgs pa{};
  pa.n_rows = n_rows;
  pa.n_keys = n_keys;
  pa.q_col0 = q_col0;
  pa.n_q = n_q;
  pa.want_qkv = 1;
  pa.want_bias = bias == nullptr;
  pa.q = w.q;
  pa.k = w.k;
  pa.bias = w.bias;
  pa.ld_keys = w.ld_keys;
  pa.b_hs = (int64_t)n_q * w.ld_keys;
  pa.b_rs = w.ld_keys;
  pa.ln_w = p->ln_w;
  pa.ln_b = p->ln_b;
  pa.q_scale = LOG2E / sqrtf((float)D);
  pa.status = status;
  PF_TRY(launch_proj(p, zs.ptr, zs.row_stride, zs.col_stride, n_rows, n_keys, pa, w.vt, st));
  // 2. attention core
  CoreIO cio = io;
  cio.bias = bias ? bias : (const void*)w.bias;
  cio.b_hs = bias ? b_hs : pa.b_hs;
  cio.b_rs = bias ? b_rs : pa.b_rs;
  PF_TRY(triatt_core(cio, n_rows, n_keys, n_valid, n_q, H, status, st));
  // 3. gate, output projection, residual
  CUtensorMap tz, to, twg, two;
  PF_TRY(pair_tmap(&tz, zs.ptr, zs.row_stride, zs.col_stride, n_rows, n_keys));
  {
    const uint64_t d3[3] = {(uint64_t)HD, (uint64_t)n_q, (uint64_t)n_rows};
    const uint64_t s3[2] = {(uint64_t)HD * 2, (uint64_t)n_q * HD * 2};
    const uint32_t b3[3] = {64, TILE, 1};
    PF_TRY(make_tmap(&to, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, w.o, d3, s3, b3, CU_TENSOR_MAP_SWIZZLE_128B));
  }
  PF_TRY(weight_tmap(&twg, p->w_g, HD, CH, 128));
  PF_TRY(weight_tmap(&two, p->w_o, CH, HD, 128));
  CUtensorMap tzo;
  PF_TRY(pair_tmap(&tzo, zo.ptr, zo.row_stride, zo.col_stride, n_rows, n_q));
  OutArgs oa{};
  oa.n_rows = n_rows;
  oa.n_q = n_q;
  oa.tiles_per_row = (n_q + TILE - 1) / TILE;
  oa.n_tiles = n_rows * oa.tiles_per_row;
  oa.q_col0 = q_col0;
  oa.zo = (const __nv_bfloat16*)zo.ptr;
  oa.zo_rs = zo.row_stride;
  oa.zo_cs = zo.col_stride;
  oa.ln_w = p->ln_w;
  oa.ln_b = p->ln_b;
  oa.accumulate = acc;
  oa.status = status;
  {
    const int64_t grid_o = oa.n_tiles < num_sms() ? oa.n_tiles : num_sms();
    // read o and the gate source z, (read the residual if it is another view), write the output
    const bool resid_apart = acc && (zo.ptr != zs.ptr || zo.row_stride != zs.row_stride || q_col0 != 0);
    const double bytes = 2.0 * (double)n_rows * n_q * (HD + CH + (resid_apart ? CH : 0) + CH);
    PF_LAUNCH_SCOPE_WORK(st, "k_triatt_out", bytes, 'b');
    k_triatt_out<<<(unsigned)grid_o, 320, OUT_SMEM + 1024, st>>>(tz, to, tzo, twg, two, oa);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}


// ------------------------------------------------------------------ shared with the general path
int triatt_masks(pf_mask_view m, int64_t n_rows, int64_t n_keys, int64_t n_valid, float inf, const CoreIO& io,
                 cudaStream_t st) {
  {
    PF_LAUNCH_SCOPE(st, "k_triatt_maskprep");
    k_triatt_maskprep<<<(unsigned)n_rows, 128, 0, st>>>(m, n_keys, n_valid, inf, io.mb, io.ld_mb, io.flags,
                                                        io.rowflags, (int)io.n_tiles_k);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

int triatt_core(const CoreIO& io, int64_t n_rows, int64_t n_keys, int64_t n_valid, int64_t n_q, int heads,
                unsigned int* status, cudaStream_t st) {
  if (n_rows * heads > 0x7fffffffll || io.n_tiles_k > 0x7fffffffll)
    return fail(PF_EUNSUPPORTED, "triatt problem too large");
  if (io.bias == nullptr || io.b_hs % 8 || io.b_rs % 8 || ((uintptr_t)io.bias) % 16)
    return fail(PF_EINVAL_SHAPE, "bias buffer must be 16-byte aligned with strides multiple of 8");
  PF_TRY(ensure_attrs());
  const int64_t hd = (int64_t)heads * D;
  if (n_valid == 0) {
    // no key exists: every attention output is zero
    PF_CUDA_TRY(cudaMemsetAsync(io.o, 0, (size_t)n_rows * n_q * hd * sizeof(__nv_bfloat16), st));
    return PF_OK;
  }
  CUtensorMap tk, tvt, tb, tmb;
  {
    const uint32_t bq[3] = {D, TILE, 1};
    const uint64_t dk[3] = {(uint64_t)D, (uint64_t)n_keys, (uint64_t)(n_rows * heads)};
    const uint64_t sk[2] = {(uint64_t)D * 2, (uint64_t)io.ld_keys * D * 2};
    PF_TRY(make_tmap(&tk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, io.k, dk, sk, bq, CU_TENSOR_MAP_SWIZZLE_64B));
    const uint64_t dv[3] = {(uint64_t)n_keys, (uint64_t)D, (uint64_t)(n_rows * heads)};
    const uint64_t sv[2] = {(uint64_t)io.ld_keys * 2, (uint64_t)D * io.ld_keys * 2};
    const uint32_t bv[3] = {64, D, 1};
    PF_TRY(make_tmap(&tvt, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, io.vt, dv, sv, bv, CU_TENSOR_MAP_SWIZZLE_128B));
    const uint64_t db[3] = {(uint64_t)n_keys, (uint64_t)n_q, (uint64_t)heads};
    const uint64_t sb[2] = {(uint64_t)io.b_rs * 2, (uint64_t)io.b_hs * 2};
    const uint32_t bb[3] = {64, TILE, 1};
    PF_TRY(make_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, io.bias, db, sb, bb, CU_TENSOR_MAP_SWIZZLE_128B));
    const uint64_t dm[2] = {(uint64_t)io.ld_mb, (uint64_t)n_rows};
    const uint64_t sm[1] = {(uint64_t)io.ld_mb * 2};
    const uint32_t bm[2] = {TILE, 1};
    PF_TRY(make_tmap(&tmb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, io.mb, dm, sm, bm, CU_TENSOR_MAP_SWIZZLE_NONE));
  }
  CoreArgs ca{};
  ca.n_rows = n_rows;
  ca.n_q = n_q;
  ca.n_tiles_k = io.n_tiles_k;
  ca.n_qt = (n_q + TILE - 1) / TILE;
  ca.n_items = ((n_rows + 1) / 2) * heads * ca.n_qt;
  ca.heads = heads;
  ca.flags = io.flags;
  ca.rowflags = io.rowflags;
  ca.q = io.q;
  ca.o = io.o;
  ca.status = status;
  const int64_t grid = ca.n_items < num_sms() ? ca.n_items : num_sms();
  {
    // QK^T and PV over every existing key: 4 H d flops per (row, query, key)
    PF_LAUNCH_SCOPE_WORK(st, "k_triatt_core", 4.0 * heads * D * (double)n_rows * n_q * n_valid, 'f');
    if (heads == H)
      k_triatt_core<H><<<(unsigned)grid, CORE_THREADS, CORE3_SMEM + 1024, st>>>(tk, tvt, tb, tmb, ca);
    else
      k_triatt_core<0><<<(unsigned)grid, CORE_THREADS, CORE3_SMEM + 1024, st>>>(tk, tvt, tb, tmb, ca);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

}  // namespace tc
}  // namespace pf
