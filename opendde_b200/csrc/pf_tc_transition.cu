// pf_tc_transition.cu -- pair Transition (LN -> SiLU(W_a y) * (W_b y) -> W_out, + residual) on
// tcgen05 tensor cores, c = 128, hidden = 4c = 512, bf16 in / fp32 accumulate.
//
// One CTA = two 128-row tiles (A and B). The 512-wide hidden layer never leaves the SM: it is
// produced and consumed in 8 chunks of 64, and every weight chunk brought in by TMA serves
// both tiles (half the L2 weight traffic of one tile per CTA):
//   [a | b](chunk)  = LN(x) [W_a(chunk); W_b(chunk)]^T     UMMA 128x128x128 -> TMEM
//   h(chunk)        = silu(a) * b  -> bf16 -> shared memory (SW128 K-major)
//   out            += h(chunk) W_o(:, chunk)^T             UMMA 128x128x64  -> TMEM
// Warps 0-3 / 4-7: tile A / tile B (thread = row): LayerNorm prologue, silu per chunk, final
// residual epilogue (TMA store). Warp 8: TMA producer (x tiles; the [W_a;W_b] chunks in a ring
// of 3 slots, the W_o chunks in a ring of 2).
// Warp 9: MMA issuer. While one warpgroup turns a chunk into h, the tensor core works on the
// other tile, so the SiLU and the MMAs overlap.
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
constexpr uint32_t S_X = 0;                          // 2 tiles x 32 KB: x, LN(x) in place, then the output tile
constexpr uint32_t S_WAB = 65536, WAB_SLOT = 32768;
constexpr uint32_t S_WO = S_WAB + NWAB * WAB_SLOT, WO_SLOT = 16384;
constexpr uint32_t S_H = S_WO + NWO * WO_SLOT;       // 2 tiles x 16 KB: h 128 rows x 64 (128 B)
constexpr uint32_t S_LN = S_H + 2 * 16384;           // LayerNorm weight and bias (fp32)
constexpr uint32_t S_BAR = S_LN + 1024;
constexpr uint32_t TR_SMEM = S_BAR + 256;
static_assert(TR_SMEM + 1024 <= 232448, "transition shared memory");

struct TrArgs {
  int64_t rows;
  const __nv_bfloat16* out;  // residual source (the output rows' old values)
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

__global__ void __launch_bounds__(320, 1) k_transition(const __grid_constant__ CUtensorMap tx,
                                                       const __grid_constant__ CUtensorMap tout,
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
  // h_full @64, h_empty @80, out_full @96; weight slots s: w_full @112+8s, w_empty @128+8s;
  // drain @144; TMEM slot @192
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
  const uint32_t b_drain = bars + 192;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(g + S_BAR + 224);
  float* lnp = reinterpret_cast<float*>(g + S_LN);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t r0 = (int64_t)blockIdx.x * (2 * TILE);
  const bool has_b = r0 + TILE < a.rows;  // tile B holds at least one row
  const int ntile = has_b ? 2 : 1;

  if (tid == 0) {
    for (int t = 0; t < 2; ++t) {
      mbar_init(b_x(t), 1);
      mbar_init(b_ln(t), 4);
      mbar_init(b_abf(t), 1);
      mbar_init(b_abe(t), 4);
      mbar_init(b_hf(t), 4);
      mbar_init(b_he(t), 1);
      mbar_init(b_out(t), 1);
    }
    for (int k = 0; k < NWAB; ++k) {
      mbar_init(b_abw_f(k), 1);
      mbar_init(b_abw_e(k), 1);
    }
    for (int k = 0; k < NWO; ++k) {
      mbar_init(b_ow_f(k), 1);
      mbar_init(b_ow_e(k), 1);
    }
    mbar_init(b_drain, 1);
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
      for (int t = 0; t < ntile; ++t) {
        mbar_arrive_expect_tx(b_x(t), 32768);
        tma_load_2d(base + S_X + t * 32768, &tx, b_x(t), 0, (int)(r0 + t * TILE));
        tma_load_2d(base + S_X + t * 32768 + 16384, &tx, b_x(t), 64, (int)(r0 + t * TILE));
      }
      for (int hc = 0; hc < NCHUNK; ++hc) {
        const int sa = hc % NWAB, na = hc / NWAB;  // slot, and its use number
        if (na > 0 && !mbar_wait(b_abw_e(sa), (na - 1) & 1, a.status)) break;
        const uint32_t w = base + S_WAB + sa * WAB_SLOT;
        mbar_arrive_expect_tx(b_abw_f(sa), WAB_SLOT);
        // atom k (K 64k..64k+63): rows 0..63 = W_a chunk, rows 64..127 = W_b chunk
        tma_load_2d(w, &twa, b_abw_f(sa), 0, hc * CHUNK);
        tma_load_2d(w + 8192, &twb, b_abw_f(sa), 0, hc * CHUNK);
        tma_load_2d(w + 16384, &twa, b_abw_f(sa), 64, hc * CHUNK);
        tma_load_2d(w + 16384 + 8192, &twb, b_abw_f(sa), 64, hc * CHUNK);
        const int so = hc % NWO, no = hc / NWO;
        if (no > 0 && !mbar_wait(b_ow_e(so), (no - 1) & 1, a.status)) break;
        mbar_arrive_expect_tx(b_ow_f(so), WO_SLOT);
        tma_load_2d(base + S_WO + so * WO_SLOT, &two, b_ow_f(so), hc * CHUNK, 0);  // W_o[:, chunk] 128 x 64
      }
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------------- MMA issuer
    // Per chunk hc and tile t: ab(t, hc + 1) as soon as t's warpgroup has read ab(t, hc) out of
    // TMEM, then out(t, hc) once it has written h(t, hc): the next chunk's ab MMAs run while the
    // warpgroup is still turning the current chunk into h, and the other tile's work fills the
    // rest.
    if (lane == 0) {
      constexpr uint32_t id_ab = idesc_f16(128, 128, true);
      constexpr uint32_t id_o = idesc_f16(128, 128, true);
      bool ok = true;
      for (int t = 0; t < ntile; ++t) ok = mbar_wait(b_ln(t), 0, a.status) && ok;  // LN(x) in smem
      ok = mbar_wait(b_abw_f(0), 0, a.status) && ok;
      for (int t = 0; t < ntile; ++t) {
        tc_fence_after();
        tile::umma_k128(tmem + 256 * t, base + S_X + t * 32768, base + S_WAB, 16384, id_ab);
        umma_commit(b_abf(t));
      }
      umma_commit(b_abw_e(0));  // [W_a;W_b] of chunk 0 free once both tiles' ab MMAs are done
      for (int hc = 0; hc < NCHUNK; ++hc) {
        const int s1 = (hc + 1) % NWAB, so = hc % NWO;
        const uint32_t w1 = base + S_WAB + s1 * WAB_SLOT, wo = base + S_WO + so * WO_SLOT;
        const bool next = hc + 1 < NCHUNK;
        if (next) ok = mbar_wait(b_abw_f(s1), ((hc + 1) / NWAB) & 1, a.status) && ok;
        ok = mbar_wait(b_ow_f(so), (hc / NWO) & 1, a.status) && ok;
        for (int t = 0; t < ntile; ++t) {
          if (next) {
            ok = mbar_wait(b_abe(t), hc & 1, a.status) && ok;  // ab(t, hc) read out
            tc_fence_after();
            tile::umma_k128(tmem + 256 * t, base + S_X + t * 32768, w1, 16384, id_ab);
            umma_commit(b_abf(t));
          }
          ok = mbar_wait(b_hf(t), hc & 1, a.status) && ok;
          tc_fence_after();
          const uint32_t hb = base + S_H + t * 16384;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(tmem + 256 * t + 128, sdesc(hb + kk * 32, 1024, SWZ_128B), sdesc(wo + kk * 32, 1024, SWZ_128B),
                     id_o, (hc > 0 || kk > 0) ? 1u : 0u);
          umma_commit(b_he(t));  // h buffer of tile t free when this MMA finishes
        }
        if (next) umma_commit(b_abw_e(s1));  // [W_a;W_b] of chunk hc + 1 free after its ab MMAs
        umma_commit(b_ow_e(so));             // W_o of chunk hc free after its out MMAs
      }
      for (int t = 0; t < ntile; ++t) umma_commit(b_out(t));
      umma_commit(b_drain);  // drain: every MMA complete before TMEM is released
      mbar_wait_drain(b_drain, 0);
    }
  } else {
    // ---------------------------------------------------------------- compute warpgroups
    const int t = warp >> 2;
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    uint8_t* xt = g + S_X + t * 32768;
    const int64_t grow = r0 + t * TILE + row;
    if (t < ntile) {
      mbar_wait(b_x(t), 0, a.status);
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
      const uint32_t tab = tmem + 256 * t + lane_base;
      uint8_t* hb = g + S_H + t * 16384;
      for (int hc = 0; hc < NCHUNK; ++hc) {
        mbar_wait(b_abf(t), hc & 1, a.status);
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
        if (hc > 0) mbar_wait(b_he(t), (hc - 1) & 1, a.status);
#pragma unroll
        for (int ch = 0; ch < 8; ++ch)
          *reinterpret_cast<uint4*>(hb + sw128_off(row, ch)) =
              make_uint4(hv[ch * 4 + 0], hv[ch * 4 + 1], hv[ch * 4 + 2], hv[ch * 4 + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(b_hf(t));
      }
      // residual epilogue: out (+ old rows, an L2 hit) written over the x tile and TMA-stored
      const bool valid = grow < a.rows;
      const bool rd = a.accumulate && valid;
      const uint4* op = reinterpret_cast<const uint4*>(a.out + (valid ? grow : 0) * a.out_stride);
      uint4 old[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) old[c] = rd ? __ldg(op + c) : make_uint4(0, 0, 0, 0);
      mbar_wait(b_out(t), 0, a.status);
      tc_fence_after();
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
          for (int k = 0; k < 8; ++k) u[k] = __uint_as_float(ov[e * 8 + k]);
          u[0] += bf16lo(o.x); u[1] += bf16hi(o.x); u[2] += bf16lo(o.y); u[3] += bf16hi(o.y);
          u[4] += bf16lo(o.z); u[5] += bf16hi(o.z); u[6] += bf16lo(o.w); u[7] += bf16hi(o.w);
          uint4 wv;
          wv.x = pack_bf16(u[0], u[1]); wv.y = pack_bf16(u[2], u[3]);
          wv.z = pack_bf16(u[4], u[5]); wv.w = pack_bf16(u[6], u[7]);
          *reinterpret_cast<uint4*>(xt + tile::chunk_off(row, chunk)) = wv;
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      named_bar_sync(1 + t, 128);
      if (warp == 4 * t && lane == 0) {
        tma_store_2d(&tout, base + S_X + t * 32768, 0, (int)(r0 + t * TILE));
        tma_store_2d(&tout, base + S_X + t * 32768 + 16384, 64, (int)(r0 + t * TILE));
        bulk_commit_group();
        bulk_wait_group0();
      }
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
  CUtensorMap tout;
  {
    const uint64_t dims[2] = {(uint64_t)C, (uint64_t)rows};
    const uint64_t str[1] = {(uint64_t)os * 2};
    const uint32_t box[2] = {64, TILE};
    PF_TRY(make_tmap(&tout, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, out, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B));
  }
  TrArgs a{rows, (const __nv_bfloat16*)out, os, p->ln_w, p->ln_b, acc, status};
  const int64_t nt = (rows + 2 * TILE - 1) / (2 * TILE);
  if (nt > 0x7fffffffll) return fail(PF_EUNSUPPORTED, "transition grid too large");
  {
    // [W_a; W_b] (2 x C x HID) and W_out (HID x C) per row: 6 C HID flops
    PF_LAUNCH_SCOPE_WORK(st, "k_transition", 6.0 * C * HID * (double)rows, 'f');
    k_transition<<<(unsigned)nt, 320, TR_SMEM + 1024, st>>>(tx, tout, twa, twb, two, a);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

}  // namespace tc
}  // namespace pf
