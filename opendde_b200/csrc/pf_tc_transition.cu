// pf_tc_transition.cu -- pair Transition (LN -> SiLU(W_a y) * (W_b y) -> W_out, + residual) on
// tcgen05 tensor cores, c = 128, hidden = 4c = 512, bf16 in / fp32 accumulate.
//
// Persistent: one CTA per SM walks pairs of 128-row tiles (A and B). The 512-wide hidden layer
// never leaves the SM: it is produced and consumed in 8 chunks of 64, and every weight chunk
// brought in by TMA serves both tiles (half the L2 weight traffic of one tile per CTA):
//   [a | b](chunk)  = LN(x) [W_a(chunk); W_b(chunk)]^T     UMMA 128x128x128 -> TMEM
//   h(chunk)        = silu(a) * b  -> bf16 -> shared memory (SW128 K-major)
//   out            += h(chunk) W_o(:, chunk)^T             UMMA 128x128x64  -> TMEM
// Warps 0-3 / 4-7: tile A / tile B (thread = row): LayerNorm prologue, silu per chunk, final
// residual epilogue (output rows stored from registers). Warp 8: TMA producer (x tiles; the
// [W_a;W_b] chunks in a ring of 3 slots, the W_o chunks in a ring of 2, both running on across
// pairs). Warps 9 / 10: MMA issuers of tile A / B. While one warpgroup turns a chunk into h, the
// tensor core works on the other tile, so the SiLU and the MMAs overlap. A tile's x buffer is
// free once the last chunk's [W_a;W_b] MMA has read it, so the next pair's x tiles load during
// the current pair's last chunk; the warpgroup normalises them before the current pair's
// epilogue, so the next pair's first MMAs run while that epilogue stores its rows.
// Reference: opendde/model/modules/primitives.py:182-217.

#include "pf_common.cuh"
#include "pf_prof.h"
#include "pf_sm100.cuh"
#include "pf_tc.h"
#include "pf_tile_common.cuh"
#include "pf_tmap.h"

namespace pf {
namespace tc {
using namespace sm100;

namespace {

constexpr int C = 128, HID = 512, CHUNK = 64, NCHUNK = HID / CHUNK, TILE = 128;

// shared memory (offsets from the 1 KB aligned base)
// Two weight rings: [W_a;W_b] of a chunk (2 atoms x 128 rows, 32 KB) three deep, W_o of a chunk
// (128 rows x 128 B, 16 KB) two deep, so that a chunk's [W_a;W_b] is in flight while the two
// chunks before it are still in use (one 48 KB slot pair per chunk, two deep, put the next chunk's
// L2 load on the path of every chunk).
constexpr int NWAB = 3, NWO = 2;
constexpr uint32_t S_X = 0;                          // 2 tiles x 32 KB: x, LN(x) in place
constexpr uint32_t S_WAB = 65536, WAB_SLOT = 32768;
constexpr uint32_t S_WO = S_WAB + NWAB * WAB_SLOT, WO_SLOT = 16384;
constexpr uint32_t S_H = S_WO + NWO * WO_SLOT;       // 2 tiles x 16 KB: h 128 rows x 64 (128 B)
constexpr uint32_t S_LN = S_H + 2 * 16384;           // LayerNorm weight and bias (fp32)
constexpr uint32_t S_BAR = S_LN + 1024;
constexpr uint32_t TR_SMEM = S_BAR + 256;
static_assert(TR_SMEM + 1024 <= 232448, "transition shared memory");

struct TrArgs {
  int64_t rows, n_pairs;
  __nv_bfloat16* out;        // output rows; with accumulate also the residual source (old values)
  int64_t out_stride;
  const float *ln_w, *ln_b;
  int accumulate;
  unsigned int* status;
};

__device__ __forceinline__ float silu_fast(float a) {
  // a * sigmoid(a), sigmoid(a) = 0.5 + 0.5 tanh(a / 2)  (one MUFU op)
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(0.5f * a));
  return a * fmaf(0.5f, t, 0.5f);
}

__global__ void __launch_bounds__(352, 1) k_transition(const __grid_constant__ CUtensorMap tx,
                                                       const __grid_constant__ CUtensorMap twa,
                                                       const __grid_constant__ CUtensorMap twb,
                                                       const __grid_constant__ CUtensorMap two,
                                                       const TrArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* g = smem_raw + (base - raw);
  const uint32_t bars = base + S_BAR;
  // barriers (per tile t = 0, 1 at +8t): x_full @0, ln_ready @16, ab_full @32, ab_empty @48,
  // h_full @64, h_empty @80, out_full @96, x_free @200, out_free @216; [W_a;W_b] slots s:
  // full @112+8s, empty @136+8s; W_o slots: full @160+8s, empty @176+8s; drain @192; TMEM slot
  // @240. Per-chunk barriers count chunks over the CTA's whole pair sequence (gc = 8 k + hc for
  // its k-th pair), per-pair barriers count pairs.
  auto b_x = [&](int t) { return bars + 8 * t; };
  auto b_ln = [&](int t) { return bars + 16 + 8 * t; };
  auto b_abf = [&](int t) { return bars + 32 + 8 * t; };
  auto b_abe = [&](int t) { return bars + 48 + 8 * t; };
  auto b_hf = [&](int t) { return bars + 64 + 8 * t; };
  auto b_he = [&](int t) { return bars + 80 + 8 * t; };
  auto b_out = [&](int t) { return bars + 96 + 8 * t; };
  auto b_abw_f = [&](int s) { return bars + 112 + 8 * s; };  // [W_a;W_b] slot full / empty
  auto b_abw_e = [&](int s) { return bars + 136 + 8 * s; };
  auto b_ow_f = [&](int s) { return bars + 160 + 8 * s; };   // W_o slot full / empty
  auto b_ow_e = [&](int s) { return bars + 176 + 8 * s; };
  auto b_xf = [&](int t) { return bars + 200 + 8 * t; };    // x buffer read by the last ab MMA
  auto b_of = [&](int t) { return bars + 216 + 8 * t; };    // D_out read by the epilogue
  const uint32_t b_drain = bars + 192;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(g + S_BAR + 240);
  float* lnp = reinterpret_cast<float*>(g + S_LN);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // tiles of pair p: 2, or 1 for a last pair whose tile B holds no row
  auto ntile_of = [&](int64_t p) { return p * (2 * TILE) + TILE < a.rows ? 2 : 1; };

  if (tid == 0) {
    for (int t = 0; t < 2; ++t) {
      mbar_init(b_x(t), 1);
      mbar_init(b_ln(t), 4);
      mbar_init(b_abf(t), 1);
      mbar_init(b_abe(t), 4);
      mbar_init(b_hf(t), 4);
      mbar_init(b_he(t), 1);
      mbar_init(b_out(t), 1);
      mbar_init(b_xf(t), 1);
      mbar_init(b_of(t), 4);
    }
    for (int k = 0; k < NWAB; ++k) {
      mbar_init(b_abw_f(k), 1);
      mbar_init(b_abw_e(k), 2);  // one arrive per MMA issuer
    }
    for (int k = 0; k < NWO; ++k) {
      mbar_init(b_ow_f(k), 1);
      mbar_init(b_ow_e(k), 2);
    }
    mbar_init(b_drain, 2);
    fence_barrier_init();
  }
  for (int c = tid; c < C; c += blockDim.x) {
    lnp[c] = a.ln_w[c];
    lnp[C + c] = a.ln_b[c];
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // tile t: D_ab at 256 t, D_out at 256 t + 128

  if (warp == 8) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      bool ok = true;
      uint32_t k = 0;
      for (int64_t p = blockIdx.x; p < a.n_pairs && ok; p += gridDim.x, ++k) {
        const int64_t r0 = p * (2 * TILE);
        const int nt = ntile_of(p);
        for (int t = 0; t < nt && ok; ++t) {
          if (k > 0) ok = mbar_wait(b_xf(t), (k - 1) & 1, a.status);  // previous pair done with x
          if (!ok) break;
          mbar_arrive_expect_tx(b_x(t), 32768);
          tma_load_2d(base + S_X + t * 32768, &tx, b_x(t), 0, (int)(r0 + t * TILE));
          tma_load_2d(base + S_X + t * 32768 + 16384, &tx, b_x(t), 64, (int)(r0 + t * TILE));
        }
        for (int hc = 0; hc < NCHUNK && ok; ++hc) {
          const uint32_t gc = k * NCHUNK + hc;
          const uint32_t sa = gc % NWAB, na = gc / NWAB;  // slot, and its use number
          if (na > 0 && !mbar_wait(b_abw_e(sa), (na - 1) & 1, a.status)) { ok = false; break; }
          const uint32_t w = base + S_WAB + sa * WAB_SLOT;
          mbar_arrive_expect_tx(b_abw_f(sa), WAB_SLOT);
          // atom k (K 64k..64k+63): rows 0..63 = W_a chunk, rows 64..127 = W_b chunk
          tma_load_2d(w, &twa, b_abw_f(sa), 0, hc * CHUNK);
          tma_load_2d(w + 8192, &twb, b_abw_f(sa), 0, hc * CHUNK);
          tma_load_2d(w + 16384, &twa, b_abw_f(sa), 64, hc * CHUNK);
          tma_load_2d(w + 16384 + 8192, &twb, b_abw_f(sa), 64, hc * CHUNK);
          const uint32_t so = gc % NWO, no = gc / NWO;
          if (no > 0 && !mbar_wait(b_ow_e(so), (no - 1) & 1, a.status)) { ok = false; break; }
          mbar_arrive_expect_tx(b_ow_f(so), WO_SLOT);
          tma_load_2d(base + S_WO + so * WO_SLOT, &two, b_ow_f(so), hc * CHUNK, 0);  // W_o[:, chunk] 128 x 64
        }
      }
    }
  } else if (warp == 9 || warp == 10) {
    // ---------------------------------------------------------------- MMA issuers
    // Warp 9 issues tile A's MMAs, warp 10 tile B's, so a tile's chain (ab(hc) read out ->
    // ab(hc + 1), h(hc) written -> out(hc)) never waits behind the other tile's warpgroup. Per
    // chunk: ab(t, hc + 1) as soon as t's warpgroup has read ab(t, hc) out of TMEM, then out(t, hc)
    // once it has written h(t, hc). A weight slot is free once both issuers have arrived on its
    // empty barrier (count 2); an issuer whose tile holds no row in the CTA's last pair still
    // waits for each slot to fill and then arrives, so the counts stay paired.
    if (lane == 0) {
      const int t = warp - 9;
      constexpr uint32_t id_ab = idesc_f16(128, 128, true);
      constexpr uint32_t id_o = idesc_f16(128, 128, true);
      const uint32_t tab = tmem + 256 * t, xs = base + S_X + t * 32768, hb = base + S_H + t * 16384;
      bool ok = true;
      uint32_t k = 0;
      for (int64_t p = blockIdx.x; p < a.n_pairs && ok; p += gridDim.x, ++k) {
        const bool active = t < ntile_of(p);
        const uint32_t gc0 = k * NCHUNK;
        if (active) ok = mbar_wait(b_ln(t), k & 1, a.status) && ok;  // LN(x) in smem
        ok = mbar_wait(b_abw_f(gc0 % NWAB), (gc0 / NWAB) & 1, a.status) && ok;
        if (active) {
          // the previous pair's last ab(t) must have been read out of TMEM
          if (k > 0) ok = mbar_wait(b_abe(t), (gc0 - 1) & 1, a.status) && ok;
          tc_fence_after();
          tile::umma_k128(tab, xs, base + S_WAB + (gc0 % NWAB) * WAB_SLOT, 16384, id_ab);
          umma_commit(b_abf(t));
          umma_commit(b_abw_e(gc0 % NWAB));  // this tile is done with chunk 0's [W_a;W_b]
        } else {
          mbar_arrive(b_abw_e(gc0 % NWAB));
        }
        for (int hc = 0; hc < NCHUNK; ++hc) {
          const uint32_t gc = gc0 + hc;
          const uint32_t s1 = (gc + 1) % NWAB, so = gc % NWO;
          const uint32_t w1 = base + S_WAB + s1 * WAB_SLOT, wo = base + S_WO + so * WO_SLOT;
          const bool next = hc + 1 < NCHUNK;
          if (next) ok = mbar_wait(b_abw_f(s1), ((gc + 1) / NWAB) & 1, a.status) && ok;
          ok = mbar_wait(b_ow_f(so), (gc / NWO) & 1, a.status) && ok;
          if (!active) {
            if (next) mbar_arrive(b_abw_e(s1));
            mbar_arrive(b_ow_e(so));
            continue;
          }
          if (next) {
            ok = mbar_wait(b_abe(t), gc & 1, a.status) && ok;  // ab(t, hc) read out
            tc_fence_after();
            tile::umma_k128(tab, xs, w1, 16384, id_ab);
            umma_commit(b_abf(t));
            if (hc + 2 == NCHUNK) umma_commit(b_xf(t));  // the last ab(t) of the pair: x(t) no longer read
            umma_commit(b_abw_e(s1));                      // this tile is done with chunk hc + 1's [W_a;W_b]
          }
          ok = mbar_wait(b_hf(t), gc & 1, a.status) && ok;
          // D_out(t) of the previous pair must have been read by its epilogue
          if (hc == 0 && k > 0) ok = mbar_wait(b_of(t), (k - 1) & 1, a.status) && ok;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(tab + 128, sdesc(hb + kk * 32, 1024, SWZ_128B), sdesc(wo + kk * 32, 1024, SWZ_128B), id_o,
                     (hc > 0 || kk > 0) ? 1u : 0u);
          umma_commit(b_he(t));    // h buffer of tile t free when this MMA finishes
          umma_commit(b_ow_e(so)); // this tile is done with chunk hc's W_o
        }
        if (active) umma_commit(b_out(t));
      }
      umma_commit(b_drain);  // drain (count 2): every MMA of both issuers complete before TMEM is released
      mbar_wait_drain(b_drain, 0);
    }
  } else {
    // ---------------------------------------------------------------- compute warpgroups
    const int t = warp >> 2;
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    uint8_t* xt = g + S_X + t * 32768;
    // LayerNorm of the CTA's kk-th pair's x tile, in place, then ln_ready
    auto layer_norm = [&](uint32_t kk) {
      mbar_wait(b_x(t), kk & 1, a.status);
      {
        uint32_t xr[64];
        float m, rs;
        tile::load_row(xt, row, xr);
        tile::row_stats(xr, 1e-5f, m, rs);
        tile::store_norm_row(xt, row, xr, m, rs, lnp, lnp + C);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(b_ln(t));
    };
    uint32_t k = 0;
    for (int64_t p = blockIdx.x; p < a.n_pairs; p += gridDim.x, ++k) {
      if (t >= ntile_of(p)) break;  // the last pair's tile B holds no row
      const int64_t grow = p * (2 * TILE) + t * TILE + row;
      if (k == 0) layer_norm(0);  // later pairs were normalised before the previous epilogue
      const uint32_t tab = tmem + 256 * t + lane_base;
      uint8_t* hb = g + S_H + t * 16384;
      for (int hc = 0; hc < NCHUNK; ++hc) {
        const uint32_t gc = k * NCHUNK + hc;
        mbar_wait(b_abf(t), gc & 1, a.status);
        tc_fence_after();
        uint32_t hv[32];  // 64 bf16 of h for this row
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t av[32], bv[32];
          tmem_ld32(tab + half * 32, av);
          tmem_ld32(tab + 64 + half * 32, bv);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 16; ++e)
            hv[half * 16 + e] = pack_bf16(silu_fast(__uint_as_float(av[2 * e])) * __uint_as_float(bv[2 * e]),
                                          silu_fast(__uint_as_float(av[2 * e + 1])) * __uint_as_float(bv[2 * e + 1]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(b_abe(t));  // D_ab may be overwritten
        if (gc > 0) mbar_wait(b_he(t), (gc - 1) & 1, a.status);  // out MMA of the previous chunk read h
#pragma unroll
        for (int ch = 0; ch < 8; ++ch)
          *reinterpret_cast<uint4*>(hb + sw128_off(row, ch)) =
              make_uint4(hv[ch * 4 + 0], hv[ch * 4 + 1], hv[ch * 4 + 2], hv[ch * 4 + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(b_hf(t));
      }
      // The next pair's x tile (loaded once this pair's last ab MMA read x) is normalised first,
      // so that pair's first ab MMA runs during this epilogue.
      const int64_t p2 = p + gridDim.x;
      if (p2 < a.n_pairs && t < ntile_of(p2)) layer_norm(k + 1);
      // residual epilogue: out (+ old rows, an L2 hit) stored from registers, 256 B per row
      const bool valid = grow < a.rows;
      const bool rd = a.accumulate && valid;
      const uint4* op = reinterpret_cast<const uint4*>(a.out + (valid ? grow : 0) * a.out_stride);
      uint4 old[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) old[c] = rd ? __ldg(op + c) : make_uint4(0, 0, 0, 0);
      mbar_wait(b_out(t), k & 1, a.status);
      tc_fence_after();
      uint4* dst = reinterpret_cast<uint4*>(a.out + (valid ? grow : 0) * a.out_stride);
#pragma unroll
      for (int cc = 0; cc < C; cc += 16) {
        uint32_t ov[16];
        tmem_ld16(tmem + 256 * t + 128 + lane_base + cc, ov);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int chunk = (cc >> 3) + e;
          const uint4 o = old[chunk];
          float u[8];
#pragma unroll
          for (int v = 0; v < 8; ++v) u[v] = __uint_as_float(ov[e * 8 + v]);
          u[0] += bf16lo(o.x); u[1] += bf16hi(o.x); u[2] += bf16lo(o.y); u[3] += bf16hi(o.y);
          u[4] += bf16lo(o.z); u[5] += bf16hi(o.z); u[6] += bf16lo(o.w); u[7] += bf16hi(o.w);
          uint4 wv;
          wv.x = pack_bf16(u[0], u[1]); wv.y = pack_bf16(u[2], u[3]);
          wv.z = pack_bf16(u[4], u[5]); wv.w = pack_bf16(u[6], u[7]);
          if (valid) dst[chunk] = wv;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(b_of(t));  // D_out(t) may be overwritten by the next pair
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

int wmap(CUtensorMap* m, const void* w, int rows, int cols, int box_cols, int box_rows) {
  const uint64_t dims[2] = {(uint64_t)cols, (uint64_t)rows};
  const uint64_t str[1] = {(uint64_t)cols * 2};
  const uint32_t box[2] = {(uint32_t)box_cols, (uint32_t)box_rows};
  return make_tmap(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace

bool transition_supported(int c, int nm) { return c == C && nm * c == HID; }

int transition(const pf_transition_params* p, const void* x, int64_t xs, void* out, int64_t os, int64_t rows,
               int, int, int acc, cudaStream_t st) {
  if (xs % 8 || os % 8 || ((uintptr_t)x) % 16 || ((uintptr_t)out) % 16)
    return fail(PF_EINVAL_SHAPE, "bf16 transition rows must be 16-byte aligned (row strides multiple of 8)");
  static std::atomic<unsigned long long> attr_done{0};
  PF_TRY(once_per_device(attr_done, []() -> int {
    PF_CUDA_TRY(cudaFuncSetAttribute(k_transition, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(TR_SMEM + 1024)));
    return PF_OK;
  }));
  unsigned int* status;
  PF_TRY(device_status_ptr(&status));
  CUtensorMap tx, twa, twb, two;
  {
    const uint64_t dims[2] = {(uint64_t)C, (uint64_t)rows};
    const uint64_t str[1] = {(uint64_t)xs * 2};
    const uint32_t box[2] = {64, TILE};
    PF_TRY(make_tmap(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B));
  }
  PF_TRY(wmap(&twa, p->w_a, HID, C, 64, CHUNK));
  PF_TRY(wmap(&twb, p->w_b, HID, C, 64, CHUNK));
  PF_TRY(wmap(&two, p->w_o, C, HID, 64, C));
  const int64_t n_pairs = (rows + 2 * TILE - 1) / (2 * TILE);
  if (n_pairs * 2 * TILE > 0x7fffffffll) return fail(PF_EUNSUPPORTED, "transition row count too large");
  if (n_pairs == 0) return PF_OK;
  TrArgs a{rows, n_pairs, (__nv_bfloat16*)out, os, p->ln_w, p->ln_b, acc, status};
  const int64_t grid = n_pairs < (int64_t)sm_count() ? n_pairs : (int64_t)sm_count();
  {
    // [W_a; W_b] (2 x C x HID) and W_out (HID x C) per row: 6 C HID flops
    PF_LAUNCH_SCOPE_WORK(st, "k_transition", 6.0 * C * HID * (double)rows, 'f');
    k_transition<<<(unsigned)grid, 352, TR_SMEM + 1024, st>>>(tx, twa, twb, two, a);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

}  // namespace tc
}  // namespace pf
