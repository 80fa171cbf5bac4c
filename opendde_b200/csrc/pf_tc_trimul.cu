// pf_tc_trimul.cu -- triangle multiplicative update on tcgen05 tensor cores (bf16 in,
// fp32 accumulate), c_z = c_h = 128.
//
// Three kernels, intermediates in the caller's workspace (bf16):
//   1. k_trimul_proj : persistent; per (128-position tile, side) the z tile is TMA-loaded
//      (128B swizzle), LayerNorm'd in place, multiplied by [W_p; W_g] (one 128x256x128 UMMA
//      chain into TMEM) and a(ch, r, k) = mask * sigmoid(g) * p is transposed in shared memory
//      and TMA-stored channel-major. Channel-major rows are exactly the K-major operands of
//      the contraction, so neither the incoming direction nor the ending node needs a
//      physical transpose.
//   2. k_trimul_bgemm: x[ch] = a[ch] * b[ch]^T for every channel: 128x256 output tiles, a
//      4-stage TMA -> UMMA pipeline (one producer thread, one MMA thread, 4 epilogue warps
//      reading the TMEM accumulator), bf16 output x[ch][i][j].
//   3. k_trimul_out  : persistent; per 128 output positions, the channel-major x tile and the
//      gate-source z tile by TMA, LN_out(x) and LN_in(z) into UMMA operands, two 128x128x128
//      UMMAs (W_g, W_z), epilogue zo (+)= (W_z x) * sigmoid(W_g z), TMA-stored.
// Reference: opendde/model/triangular/triangular.py:530-567 (maths), :112-139 (orientation).

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

constexpr int CH = 128;    // c_z == c_h on this path
constexpr int TILE = 128;  // positions per projection / output CTA

// ------------------------------------------------------------------ kernel 1: projections
// Persistent, one CTA per SM, an even grid: CTA b projects side b & 1 only (items of the two
// sides of a tile run on neighbouring CTAs at the same time, so a z tile shared by both sides
// is read from DRAM once and from L2 the second time), so it holds one side's [W_p ; W_g]
// (64 KB). That leaves room for a 3-deep ring of z tiles and two output stages: the next z
// tiles stream in while earlier items are normalised, multiplied and stored.
//   warp 0     TMA producer: the side's [W_p ; W_g] once, then z tiles into the ring
//   warp 1     MMA issuer: [p | g] = [W_p ; W_g] LN(z) (N = 256) into the item's warpgroup's 256
//              TMEM columns; the MMA completion frees the ring slot
//   warps 2-9  two warpgroups, alternate items: LN in place in the ring slot; epilogue
//              mask * sigmoid(g) * p (reference order, triangular.py:539-544) transposed into
//              the warpgroup's output stage as [channel][position] and TMA-stored into the
//              channel-major operand a[c][row][k] (or b)
struct ProjSide {
  int64_t n_rows, n_cols;
  pf_mask_view mask;
  int64_t tiles_per_row;
  int64_t ntiles;
};
struct ProjArgs {
  ProjSide side[2];
  const float* ln_w;
  const float* ln_b;
  unsigned int* status;
};

constexpr int P_RING = 3;
constexpr uint32_t P_W = 0, P_TILE = 32768;
constexpr uint32_t P_RING0 = 65536, P_OUT0 = P_RING0 + P_RING * P_TILE;
constexpr uint32_t P_LN = P_OUT0 + 2 * P_TILE, P_BAR = P_LN + 1024;
constexpr uint32_t PROJ_SMEM = P_BAR + 256;
static_assert(PROJ_SMEM + 1024 <= 232448, "dynamic shared memory limit");

__global__ void __launch_bounds__(320, 1) k_trimul_proj(const __grid_constant__ CUtensorMap tz0,
                                                        const __grid_constant__ CUtensorMap tz1,
                                                        const __grid_constant__ CUtensorMap to0,
                                                        const __grid_constant__ CUtensorMap to1,
                                                        const __grid_constant__ CUtensorMap tw0p,
                                                        const __grid_constant__ CUtensorMap tw0g,
                                                        const __grid_constant__ CUtensorMap tw1p,
                                                        const __grid_constant__ CUtensorMap tw1g,
                                                        const ProjArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* g = smem_raw + (base - raw);
  const uint32_t bars = base + P_BAR, wbar = bars;
  // wbar @0, full[3] @8, empty[3] @32, ready[2] @56, done[2] @72, drain @88; TMEM slot @128
  auto full = [&](uint32_t sl) { return bars + 8 + 8 * sl; };
  auto empty = [&](uint32_t sl) { return bars + 32 + 8 * sl; };
  auto ready = [&](int w) { return bars + 56 + 8 * w; };
  auto done = [&](int w) { return bars + 72 + 8 * w; };
  const uint32_t bar_drain = bars + 88;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(g + P_BAR + 128);
  float* lnp = reinterpret_cast<float*>(g + P_LN);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int side = (int)(blockIdx.x & 1);
  const ProjSide& sd = args.side[side];
  const int64_t first = blockIdx.x >> 1, stride = gridDim.x >> 1;  // this side's tiles
  if (tid == 0) {
    mbar_init(wbar, 1);
    for (int sl = 0; sl < P_RING; ++sl) {
      mbar_init(full(sl), 1);
      mbar_init(empty(sl), 1);
    }
    for (int w = 0; w < 2; ++w) {
      mbar_init(ready(w), 1);
      mbar_init(done(w), 1);
    }
    mbar_init(bar_drain, 1);
    fence_barrier_init();
  }
  for (int c = tid; c < CH; c += blockDim.x) {
    lnp[c] = args.ln_w[c];
    lnp[CH + c] = args.ln_b[c];
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const CUtensorMap* tz = side ? &tz1 : &tz0;
      tma_prefetch_desc(tz);
      mbar_arrive_expect_tx(wbar, 65536);
      // atom 0 = [W_p ; W_g] channels 0..63 (32 KB), atom 1 = channels 64..127
      const CUtensorMap* twp = side ? &tw1p : &tw0p;
      const CUtensorMap* twg = side ? &tw1g : &tw0g;
      tma_load_2d(base + P_W, twp, wbar, 0, 0);
      tma_load_2d(base + P_W + 16384, twg, wbar, 0, 0);
      tma_load_2d(base + P_W + 32768, twp, wbar, 64, 0);
      tma_load_2d(base + P_W + 49152, twg, wbar, 64, 0);
      bool ok = true;
      int64_t k = 0;
      for (int64_t t = first; t < sd.ntiles && ok; t += stride, ++k) {
        const uint32_t sl = (uint32_t)(k % P_RING), u = (uint32_t)(k / P_RING);
        if (u > 0) ok = mbar_wait(empty(sl), (u - 1) & 1, args.status) && ok;
        const int r = (int)(t / sd.tiles_per_row);
        const int c0 = (int)((t % sd.tiles_per_row) * TILE);
        const uint32_t st = base + P_RING0 + sl * P_TILE;
        mbar_arrive_expect_tx(full(sl), 32768);
        tma_load_3d(st, tz, full(sl), 0, c0, r);
        tma_load_3d(st + 16384, tz, full(sl), 64, c0, r);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(wbar, 0, args.status);
      int64_t k = 0;
      for (int64_t t = first; t < sd.ntiles && ok; t += stride, ++k) {
        const int w = (int)(k & 1);
        const uint32_t sl = (uint32_t)(k % P_RING);
        ok = mbar_wait(ready(w), (uint32_t)((k >> 1) & 1), args.status) && ok;
        tc_fence_after();
        tile::umma_k128(tmem + w * 256, base + P_RING0 + sl * P_TILE, base + P_W, 32768, idesc_f16(128, 256, true));
        umma_commit(done(w));
        umma_commit(empty(sl));  // the ring slot is free once these MMAs have read it
      }
      umma_commit(bar_drain);  // drain: every MMA complete before TMEM is released
      mbar_wait_drain(bar_drain, 0);
    }
  } else {
    const int wg = (warp - 2) >> 2;
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const bool leader = (warp == 2 + 4 * wg) && lane == 0;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const uint32_t ost = base + P_OUT0 + wg * P_TILE;
    unsigned short* ot = reinterpret_cast<unsigned short*>(g + P_OUT0 + wg * P_TILE);
    int64_t k = 0, mine = 0;
    for (int64_t t = first; t < sd.ntiles; t += stride, ++k) {
      if ((int)(k & 1) != wg) continue;
      const uint32_t sl = (uint32_t)(k % P_RING);
      const int r = (int)(t / sd.tiles_per_row);
      const int c0 = (int)((t % sd.tiles_per_row) * TILE);
      uint8_t* zt = g + P_RING0 + sl * P_TILE;
      mbar_wait(full(sl), (uint32_t)((k / P_RING) & 1), args.status);
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
      float mk = 0.f;
      if (col < sd.n_cols)
        mk = sd.mask.ptr ? sd.mask.ptr[(int64_t)r * sd.mask.row_stride + col * sd.mask.col_stride] : 1.f;
      // the output stage's previous TMA store must have read it before it is overwritten
      if (mine > 0) {
        if (leader) bulk_wait_group_read0();
        named_bar_sync(1 + wg, 128);
      }
      mbar_wait(done(wg), (uint32_t)(mine & 1), args.status);
      tc_fence_after();
      // [channel][position] bf16 tile: 256 B per channel
#pragma unroll
      for (int cc = 0; cc < CH; cc += 16) {
        uint32_t pv[16], gv[16];
        tmem_ld16(tmem + lane_base + wg * 256 + cc, pv);
        tmem_ld16(tmem + lane_base + wg * 256 + 128 + cc, gv);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float v = mk * fast_sigmoid(__uint_as_float(gv[e])) * __uint_as_float(pv[e]);
          ot[(cc + e) * TILE + row] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      named_bar_sync(1 + wg, 128);
      if (leader) {
        tma_store_3d(side ? &to1 : &to0, ost, c0, r, 0);
        bulk_commit_group();
      }
      ++mine;
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

// ------------------------------------------------------------------ kernel 2: contraction
constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr uint32_t A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr uint32_t GEMM_SMEM = STAGES * STAGE_BYTES + 256;

struct GemmArgs {
  int M, N, K;
  int m_tiles, n_tiles;
  int64_t n_work;           // channels * m_tiles * n_tiles
  __nv_bfloat16* out;
  int64_t ldo;
  int64_t out_bstride;
  unsigned int* status;
};

// Persistent: one CTA per SM walks the (channel, m tile, n tile) work list (n fastest, so the
// CTAs running at one time share a channel's a and b in L2). The TMA ring runs across tiles;
// two TMEM accumulators (2 x 256 columns) let the epilogue of one tile overlap the MMAs of
// the next. Warp 0: TMA producer. Warp 1: MMA issuer. Warps 2-5: epilogue (TMEM -> bf16 ->
// global, one output row per thread).
__global__ void __launch_bounds__(192, 1) k_trimul_bgemm(const __grid_constant__ CUtensorMap ta,
                                                         const __grid_constant__ CUtensorMap tb,
                                                         const GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* g = smem_raw + (base - raw);
  const uint32_t bars = base + STAGES * STAGE_BYTES;
  // full[s] @8s, empty[s] @64+8s, acc_full[b] @128+8b, acc_empty[b] @144+8b, drain @160;
  // TMEM slot @192
  auto acc_full = [&](int b) { return bars + 128 + 8 * b; };
  auto acc_empty = [&](int b) { return bars + 144 + 8 * b; };
  const uint32_t bar_drain = bars + 160;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(g + STAGES * STAGE_BYTES + 192);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nk = (args.K + BK - 1) / BK;
  const int64_t G = gridDim.x;
  auto decode = [&](int64_t t, int& ch, int& m0, int& n0) {
    const int nt = (int)(t % args.n_tiles);
    const int64_t r = t / args.n_tiles;
    m0 = (int)(r % args.m_tiles) * BM;
    ch = (int)(r / args.m_tiles);
    n0 = nt * BN;
  };

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bars + 8 * s, 1);
      mbar_init(bars + 64 + 8 * s, 1);
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

  if (warp == 0) {
    if (lane == 0) {
      // TMA producer: one k-block counter across all tiles of this CTA
      uint32_t cnt = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < args.n_work && ok; t += G) {
        int ch, m0, n0;
        decode(t, ch, m0, n0);
        for (int kb = 0; kb < nk; ++kb, ++cnt) {
          const uint32_t s = cnt % STAGES, u = cnt / STAGES;
          if (u > 0) ok = mbar_wait(bars + 64 + 8 * s, (u - 1) & 1, args.status) && ok;
          const uint32_t sa = base + s * STAGE_BYTES, sb = sa + A_BYTES;
          mbar_arrive_expect_tx(bars + 8 * s, STAGE_BYTES);
          tma_load_3d(sa, &ta, bars + 8 * s, kb * BK, m0, ch);
          tma_load_3d(sb, &tb, bars + 8 * s, kb * BK, n0, ch);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(BM, BN, true);
      uint32_t cnt = 0, j = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < args.n_work && ok; t += G, ++j) {
        const uint32_t b = j & 1;
        if (j >= 2) ok = mbar_wait(acc_empty(b), ((j >> 1) - 1) & 1, args.status) && ok;  // epilogue drained it
        tc_fence_after();
        const uint32_t acc = tmem + 256 * b;
        for (int kb = 0; kb < nk; ++kb, ++cnt) {
          const uint32_t s = cnt % STAGES, u = cnt / STAGES;
          ok = mbar_wait(bars + 8 * s, u & 1, args.status) && ok;
          tc_fence_after();
          const uint32_t sa = base + s * STAGE_BYTES, sb = sa + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = sdesc(sa + kk * 32, 1024, SWZ_128B);
            const uint64_t bd = sdesc(sb + kk * 32, 1024, SWZ_128B);
            umma_f16(acc, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(bars + 64 + 8 * s);  // frees the stage when these MMAs finish
        }
        umma_commit(acc_full(b));
      }
      umma_commit(bar_drain);  // drain: every MMA complete before TMEM is released
      mbar_wait_drain(bar_drain, 0);
    }
  } else {
    // epilogue: TMEM -> bf16 -> global
    const int q = warp & 3;
    const int row = q * 32 + lane;
    uint32_t j = 0;
    for (int64_t t = blockIdx.x; t < args.n_work; t += G, ++j) {
      int ch, m0, n0;
      decode(t, ch, m0, n0);
      const uint32_t b = j & 1;
      mbar_wait(acc_full(b), (j >> 1) & 1, args.status);
      tc_fence_after();
      const int gm = m0 + row;
      __nv_bfloat16* orow = args.out + (int64_t)ch * args.out_bstride + (int64_t)gm * args.ldo;
#pragma unroll 1
      for (int cc = 0; cc < BN; cc += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + 256 * b + ((uint32_t)(q * 32) << 16) + cc, v);
        tmem_ld_wait();
        const int gn = n0 + cc;
        if (gm < args.M && gn < args.N) {
          if (gn + 32 <= args.N) {
            uint4* dst = reinterpret_cast<uint4*>(orow + gn);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              uint4 w;
              w.x = pack_bf16(__uint_as_float(v[e * 8 + 0]), __uint_as_float(v[e * 8 + 1]));
              w.y = pack_bf16(__uint_as_float(v[e * 8 + 2]), __uint_as_float(v[e * 8 + 3]));
              w.z = pack_bf16(__uint_as_float(v[e * 8 + 4]), __uint_as_float(v[e * 8 + 5]));
              w.w = pack_bf16(__uint_as_float(v[e * 8 + 6]), __uint_as_float(v[e * 8 + 7]));
              dst[e] = w;
            }
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (gn + e < args.N) orow[gn + e] = __float2bfloat16_rn(__uint_as_float(v[e]));
          }
        }
      }
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

// ------------------------------------------------------------------ kernel 3: output
// Persistent: one CTA per SM walks the output tiles (tile k of the CTA goes to compute
// warpgroup k & 1, which owns shared-memory stage k & 1 and TMEM columns [256 w, 256 w + 256)).
//   warp 0      TMA producer: W_g, W_z once; per tile the z tile (K-major SW128) and the x tile
//               (channel-major box, 128 channels x 128 positions) into the warpgroup's stage
//   warp 1      MMA issuer: gate = W_g LN_in(z) into cols +128, acc = W_z LN_out(x) into cols +0;
//               the MMA completion frees the input stage, so the next tiles load during the
//               epilogue
//   warps 2-9   two warpgroups; thread = position. x column -> registers -> LN_out(x) written
//               K-major into the x buffer; LN_in(z) in place in the z buffer; epilogue
//               acc * sigmoid(gate) (+ residual read back from global, an L2 hit) written into
//               the shared output stage (handed between the warpgroups by out_free), which is
//               then TMA-stored.
struct OutArgs {
  int64_t n_i, n_j, tiles_per_row, n_tiles;
  const float *ln_in_w, *ln_in_b, *ln_out_w, *ln_out_b;
  int resid;                     // 0: none (zo = update), else zo += update
  const __nv_bfloat16* zo;
  int64_t zo_rs, zo_cs;
  unsigned int* status;
};

// W_g, W_z; two input stages (z tile + x tile) freed when their MMAs complete; one output stage
// shared by the two warpgroups (items alternate, so it is handed over by the out_free barrier).
// This fills the 227 KB limit: the launch asks for all of it, and the kernel checks that the
// 1 KB-aligned layout fits in what it got (the dynamic region starts 1 KB-aligned after the
// block's reserved shared memory; if it did not, the kernel reports and returns).
constexpr uint32_t O_WG = 0, O_WZ = 32768, O_STAGE = 65536, O_STAGE_BYTES = 65536;
constexpr uint32_t O_OUT = O_STAGE + 2 * O_STAGE_BYTES;
constexpr uint32_t O_LN = O_OUT + 32768;  // 4 x 128 fp32 LayerNorm parameters
constexpr uint32_t O_BAR = O_LN + 2048;
constexpr uint32_t OUT_SMEM = O_BAR + 256;
constexpr uint32_t OUT_SMEM_ALLOC = 232448;
static_assert(OUT_SMEM <= OUT_SMEM_ALLOC, "dynamic shared memory limit");

__global__ void __launch_bounds__(320, 1) k_trimul_out(const __grid_constant__ CUtensorMap tzg,
                                                       const __grid_constant__ CUtensorMap tx,
                                                       const __grid_constant__ CUtensorMap tzo,
                                                       const __grid_constant__ CUtensorMap twz,
                                                       const __grid_constant__ CUtensorMap twg,
                                                       const OutArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* g = smem_raw + (base - raw);
  const uint32_t bars = base + O_BAR;
  const uint32_t wbar = bars;
  auto full = [&](int w) { return bars + 8 + 8 * w; };
  auto empty = [&](int w) { return bars + 24 + 8 * w; };
  auto ready = [&](int w) { return bars + 40 + 8 * w; };
  auto done = [&](int w) { return bars + 56 + 8 * w; };
  const uint32_t out_free = bars + 80;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(g + O_BAR + 128);
  float* lnp = reinterpret_cast<float*>(g + O_LN);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if ((base - raw) + OUT_SMEM > OUT_SMEM_ALLOC) {  // uniform over the block: nothing was started
    if (tid == 0) atomicOr(args.status, 4u);  // report-only bit: the layout did not fit
    return;
  }

  if (tid == 0) {
    mbar_init(wbar, 1);
    for (int w = 0; w < 2; ++w) {
      mbar_init(full(w), 1);
      mbar_init(empty(w), 1);
      mbar_init(ready(w), 1);
      mbar_init(done(w), 1);
    }
    mbar_init(bars + 72, 1);
    mbar_init(out_free, 1);
    fence_barrier_init();
  }
  for (int c = tid; c < 128; c += blockDim.x) {
    lnp[c] = args.ln_in_w[c];
    lnp[128 + c] = args.ln_in_b[c];
    lnp[256 + c] = args.ln_out_w[c];
    lnp[384 + c] = args.ln_out_b[c];
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
      tma_prefetch_desc(&tzg);
      tma_prefetch_desc(&tx);
      mbar_arrive_expect_tx(wbar, 65536);
      tma_load_2d(base + O_WG, &twg, wbar, 0, 0);
      tma_load_2d(base + O_WG + 16384, &twg, wbar, 64, 0);
      tma_load_2d(base + O_WZ, &twz, wbar, 0, 0);
      tma_load_2d(base + O_WZ + 16384, &twz, wbar, 64, 0);
      for (int64_t k = 0;; ++k) {
        const int64_t t = blockIdx.x + k * G;
        if (t >= args.n_tiles) break;
        const int w = (int)(k & 1);
        const int64_t n = k >> 1;
        if (n > 0) mbar_wait(empty(w), (uint32_t)((n - 1) & 1), args.status);
        const int i = (int)(t / args.tiles_per_row);
        const int j0 = (int)((t % args.tiles_per_row) * TILE);
        const uint32_t st = base + O_STAGE + w * O_STAGE_BYTES;
        mbar_arrive_expect_tx(full(w), 65536);
        tma_load_3d(st, &tzg, full(w), 0, j0, i);
        tma_load_3d(st + 16384, &tzg, full(w), 64, j0, i);
        tma_load_3d(st + 32768, &tx, full(w), j0, i, 0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      mbar_wait(wbar, 0, args.status);
      for (int64_t k = 0;; ++k) {
        const int64_t t = blockIdx.x + k * G;
        if (t >= args.n_tiles) break;
        const int w = (int)(k & 1);
        const uint32_t par = (uint32_t)((k >> 1) & 1);
        const uint32_t sZ = base + O_STAGE + w * O_STAGE_BYTES, sX = sZ + 32768;
        mbar_wait(ready(w), par, args.status);
        tc_fence_after();
        tile::umma_k128(tmem + w * 256 + 128, sZ, base + O_WG, 16384, idesc_f16(128, 128, true));
        tile::umma_k128(tmem + w * 256, sX, base + O_WZ, 16384, idesc_f16(128, 128, true));
        umma_commit(done(w));
        umma_commit(empty(w));  // the stage is free once these MMAs have read it
      }
      umma_commit(bars + 72);  // drain: every MMA complete before TMEM is released
      mbar_wait_drain(bars + 72, 0);
    }
  } else {
    const int wg = (warp - 2) >> 2;
    const int q = warp & 3;             // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;      // position within the tile
    const bool leader = (warp == 2 + 4 * wg) && lane == 0;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    uint8_t* zt = g + O_STAGE + wg * O_STAGE_BYTES;
    uint8_t* xt = zt + 32768;
    for (int64_t k = wg;; k += 2) {
      const int64_t t = blockIdx.x + k * G;
      if (t >= args.n_tiles) break;
      const uint32_t par = (uint32_t)((k >> 1) & 1);
      const int i = (int)(t / args.tiles_per_row);
      const int j0 = (int)((t % args.tiles_per_row) * TILE);
      mbar_wait(full(wg), par, args.status);
      // x(i, j0 + row, :) from the channel-major tile
      uint32_t xr[64];
      {
        const uint16_t* xs = reinterpret_cast<const uint16_t*>(xt);
#pragma unroll
        for (int c = 0; c < 64; ++c)
          xr[c] = (uint32_t)xs[(2 * c) * TILE + row] | ((uint32_t)xs[(2 * c + 1) * TILE + row] << 16);
      }
      named_bar_sync(1 + wg, 128);   // every x column is in registers
      {
        float m, r;
        tile::row_stats(xr, 1e-5f, m, r);
        tile::store_norm_row(xt, row, xr, m, r, lnp + 256, lnp + 384);
      }
      asm volatile("" ::: "memory");  // keep the two row passes apart (register pressure)
      {
        uint32_t zr[64];
        float m, r;
        tile::load_row(zt, row, zr);
        tile::row_stats(zr, 1e-5f, m, r);
        tile::store_norm_row(zt, row, zr, m, r, lnp, lnp + 128);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      named_bar_sync(1 + wg, 128);
      if (leader) mbar_arrive(ready(wg));
      // residual row, fetched while the GEMMs run (zo's old values; an L2 hit when zo is zg)
      const int64_t j = (int64_t)j0 + row;
      const bool valid = j < args.n_j;
      const bool rd = args.resid && valid;
      const uint4* zp = reinterpret_cast<const uint4*>(args.zo + (int64_t)i * args.zo_rs + (valid ? j : 0) * args.zo_cs);
      uint4 old[16];
#pragma unroll
      for (int c = 0; c < 8; ++c) old[c] = rd ? __ldg(zp + c) : make_uint4(0, 0, 0, 0);
      mbar_wait(done(wg), par, args.status);
      tc_fence_after();
#pragma unroll
      for (int c = 8; c < 16; ++c) old[c] = rd ? __ldg(zp + c) : make_uint4(0, 0, 0, 0);
      // the output stage: the previous item's TMA store (the other warpgroup's) has read it
      if (k > 0) mbar_wait(out_free, (uint32_t)((k - 1) & 1), args.status);
#pragma unroll
      for (int cc = 0; cc < CH; cc += 16) {
        uint32_t av[16], gv[16];
        tmem_ld16(tmem + lane_base + wg * 256 + cc, av);
        tmem_ld16(tmem + lane_base + wg * 256 + 128 + cc, gv);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int chunk = (cc >> 3) + e;
          uint4* dst = reinterpret_cast<uint4*>(g + O_OUT + tile::chunk_off(row, chunk));
          float u[8];
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            u[kk] = __uint_as_float(av[e * 8 + kk]) * fast_sigmoid(__uint_as_float(gv[e * 8 + kk]));
          {
            const uint4 o = old[chunk];
            u[0] += bf16lo(o.x); u[1] += bf16hi(o.x); u[2] += bf16lo(o.y); u[3] += bf16hi(o.y);
            u[4] += bf16lo(o.z); u[5] += bf16hi(o.z); u[6] += bf16lo(o.w); u[7] += bf16hi(o.w);
          }
          uint4 wv;
          wv.x = pack_bf16(u[0], u[1]); wv.y = pack_bf16(u[2], u[3]);
          wv.z = pack_bf16(u[4], u[5]); wv.w = pack_bf16(u[6], u[7]);
          *dst = wv;
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      named_bar_sync(1 + wg, 128);
      if (leader) {
        tma_store_3d(&tzo, base + O_OUT, 0, j0, i);
        tma_store_3d(&tzo, base + O_OUT + 16384, 64, j0, i);
        bulk_commit_group();
        bulk_wait_group_read0();
        mbar_arrive(out_free);
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

// ------------------------------------------------------------------ host helpers
int pair_tmap(CUtensorMap* m, const pf_pair_view& v, int64_t n_rows, int64_t n_cols) {
  if (v.row_stride % 8 || v.col_stride % 8)
    return fail(PF_EINVAL_SHAPE, "bf16 pair views need row/col strides that are multiples of 8 elements");
  const uint64_t dims[3] = {(uint64_t)CH, (uint64_t)n_cols, (uint64_t)n_rows};
  const uint64_t str[2] = {(uint64_t)v.col_stride * 2, (uint64_t)v.row_stride * 2};
  const uint32_t box[3] = {64, (uint32_t)TILE, 1};
  return make_tmap(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, v.ptr, dims, str, box,
                   CU_TENSOR_MAP_SWIZZLE_128B);
}

int weight_tmap(CUtensorMap* m, const void* w, int rows, int cols, int box_rows) {
  const uint64_t dims[2] = {(uint64_t)cols, (uint64_t)rows};
  const uint64_t str[1] = {(uint64_t)cols * 2};
  const uint32_t box[2] = {64, (uint32_t)box_rows};
  return make_tmap(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

template <class K>
int set_smem(K kernel, uint32_t bytes) {
  PF_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
  return PF_OK;
}

struct TrimulWs {
  __nv_bfloat16 *a, *b, *x;
  int64_t ld_k, ld_j;
};

void trimul_plan(Arena& ar, int64_t n_i, int64_t n_j, int64_t n_k, TrimulWs& w) {
  w.ld_k = (n_k + 7) / 8 * 8;
  w.ld_j = (n_j + 7) / 8 * 8;
  w.a = ar.take<__nv_bfloat16>((size_t)CH * n_i * w.ld_k);
  w.b = ar.take<__nv_bfloat16>((size_t)CH * n_j * w.ld_k);
  w.x = ar.take<__nv_bfloat16>((size_t)CH * n_i * w.ld_j);
}

}  // namespace

bool trimul_supported(int64_t n_i, int64_t n_j, int64_t n_k, int c_z, int c_h) {
  return c_z == CH && c_h == CH && n_i >= 1 && n_j >= 1 && n_k >= 1 && n_i < (1ll << 31) &&
         n_j < (1ll << 31) && n_k < (1ll << 31);
}

size_t trimul_ws_bytes(int64_t n_i, int64_t n_j, int64_t n_k, int, int) {
  Arena ar(nullptr, 0);
  TrimulWs w;
  trimul_plan(ar, n_i, n_j, n_k, w);
  return ar.used;
}

namespace {

// Dynamic shared-memory limits, set once on every device that runs these kernels.
int ensure_attrs() {
  static std::atomic<unsigned long long> done{0};
  return once_per_device(done, []() -> int {
    PF_TRY(set_smem(k_trimul_proj, PROJ_SMEM + 1024));
    PF_TRY(set_smem(k_trimul_bgemm, GEMM_SMEM + 1024));
    PF_TRY(set_smem(k_trimul_out, OUT_SMEM_ALLOC));
    return PF_OK;
  });
}

// a(ch, i, k) = projection of za(i, k) (i < n_i), b(ch, j, k) of zb(j, k) (j < n_j), stored
// channel-major with row pitch ld (elements, multiple of 8) and plane pitch n * ld.
int launch_proj(const pf_trimul_params* p, pf_pair_view za, pf_pair_view zb, pf_mask_view ma,
                pf_mask_view mb, int64_t n_i, int64_t n_j, int64_t n_k, __nv_bfloat16* a,
                __nv_bfloat16* b, int64_t ld, unsigned int* status, cudaStream_t st) {
  CUtensorMap tz0, tz1, to0, to1, tw0p, tw0g, tw1p, tw1g;
  PF_TRY(pair_tmap(&tz0, za, n_i, n_k));
  PF_TRY(pair_tmap(&tz1, zb, n_j, n_k));
  PF_TRY(weight_tmap(&tw0p, p->w_ap, CH, CH, 128));
  PF_TRY(weight_tmap(&tw0g, p->w_ag, CH, CH, 128));
  PF_TRY(weight_tmap(&tw1p, p->w_bp, CH, CH, 128));
  PF_TRY(weight_tmap(&tw1g, p->w_bg, CH, CH, 128));
  {
    const uint32_t bo[3] = {(uint32_t)TILE, 1, (uint32_t)CH};
    const uint64_t d0[3] = {(uint64_t)n_k, (uint64_t)n_i, (uint64_t)CH};
    const uint64_t s0[2] = {(uint64_t)ld * 2, (uint64_t)n_i * ld * 2};
    PF_TRY(make_tmap(&to0, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a, d0, s0, bo, CU_TENSOR_MAP_SWIZZLE_NONE));
    const uint64_t d1[3] = {(uint64_t)n_k, (uint64_t)n_j, (uint64_t)CH};
    const uint64_t s1[2] = {(uint64_t)ld * 2, (uint64_t)n_j * ld * 2};
    PF_TRY(make_tmap(&to1, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, b, d1, s1, bo, CU_TENSOR_MAP_SWIZZLE_NONE));
  }
  ProjArgs pa;
  const int64_t tpr_k = (n_k + TILE - 1) / TILE;
  pa.side[0] = ProjSide{n_i, n_k, ma, tpr_k, n_i * tpr_k};
  pa.side[1] = ProjSide{n_j, n_k, mb, tpr_k, n_j * tpr_k};
  const int64_t nt = pa.side[0].ntiles > pa.side[1].ntiles ? pa.side[0].ntiles : pa.side[1].ntiles;
  pa.ln_w = p->ln_in_w;
  pa.ln_b = p->ln_in_b;
  pa.status = status;
  {
    // an even grid: CTA b works on side b & 1 (tile b >> 1, then every (grid / 2)-th tile)
    const int64_t half = sm_count() / 2;
    const int64_t grid_p = 2 * (nt < half ? nt : half);
    // read each z view once (once in all when both sides project the same view), write a and b
    const bool same = za.ptr == zb.ptr && za.row_stride == zb.row_stride && za.col_stride == zb.col_stride &&
                      n_i == n_j;
    const double pos_a = (double)n_i * n_k, pos_b = (double)n_j * n_k;
    const double bytes = 2.0 * ((same ? pos_a : pos_a + pos_b) * CH + (pos_a + pos_b) * CH);
    PF_LAUNCH_SCOPE_WORK(st, "k_trimul_proj", bytes, 'b');
    k_trimul_proj<<<(unsigned)grid_p, 320, PROJ_SMEM + 1024, st>>>(tz0, tz1, to0, to1, tw0p, tw0g, tw1p, tw1g, pa);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

// x(ch, i, j) = sum_k a(ch, i, k) b(ch, j, k) into x (row pitch ld_j), then
// zo (+)= (W_z LN_out(x)) * sigmoid(W_g LN_in(zg)).
int launch_contract_out(const pf_trimul_params* p, const __nv_bfloat16* a, int64_t lda,
                        const __nv_bfloat16* b, int64_t ldb, int64_t n_i, int64_t n_j, int64_t n_k,
                        __nv_bfloat16* x, int64_t ld_j, pf_pair_view zg, pf_pair_view zo, int acc,
                        unsigned int* status, cudaStream_t st) {
  PF_TRY(trimul_contract(a, lda, b, ldb, n_i, n_j, n_k, CH, x, ld_j, status, st));
  // LN_out, W_z, gate, residual (persistent, one CTA per SM)
  CUtensorMap tzg, tzo, txm, twz, twg;
  PF_TRY(pair_tmap(&tzg, zg, n_i, n_j));
  PF_TRY(pair_tmap(&tzo, zo, n_i, n_j));
  PF_TRY(weight_tmap(&twz, p->w_z, CH, CH, 128));
  PF_TRY(weight_tmap(&twg, p->w_g, CH, CH, 128));
  {
    const uint64_t dx[3] = {(uint64_t)n_j, (uint64_t)n_i, (uint64_t)CH};
    const uint64_t sx[2] = {(uint64_t)ld_j * 2, (uint64_t)n_i * ld_j * 2};
    const uint32_t bx[3] = {(uint32_t)TILE, 1, (uint32_t)CH};
    PF_TRY(make_tmap(&txm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, x, dx, sx, bx, CU_TENSOR_MAP_SWIZZLE_NONE));
  }
  OutArgs oa;
  oa.n_i = n_i;
  oa.n_j = n_j;
  oa.tiles_per_row = (n_j + TILE - 1) / TILE;
  oa.n_tiles = n_i * oa.tiles_per_row;
  oa.ln_in_w = p->ln_in_w;
  oa.ln_in_b = p->ln_in_b;
  oa.ln_out_w = p->ln_out_w;
  oa.ln_out_b = p->ln_out_b;
  oa.resid = acc ? 1 : 0;
  oa.zo = (const __nv_bfloat16*)zo.ptr;
  oa.zo_rs = zo.row_stride;
  oa.zo_cs = zo.col_stride;
  oa.status = status;
  const int64_t grid_o = oa.n_tiles < sm_count() ? oa.n_tiles : sm_count();
  {
    // read x and the gate source, (read the residual if it is another view), write the output
    const bool resid_apart = acc && (zo.ptr != zg.ptr || zo.row_stride != zg.row_stride);
    const double bytes = 2.0 * (double)n_i * n_j * (CH + CH + (resid_apart ? CH : 0) + CH);
    PF_LAUNCH_SCOPE_WORK(st, "k_trimul_out", bytes, 'b');
    k_trimul_out<<<(unsigned)grid_o, 320, OUT_SMEM_ALLOC, st>>>(tzg, txm, tzo, twz, twg, oa);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

int check_out_view(const pf_pair_view& zo) {
  if (zo.row_stride % 8 || zo.col_stride % 8 || ((uintptr_t)zo.ptr) % 16)
    return fail(PF_EINVAL_SHAPE, "bf16 output view must be 16-byte aligned with strides multiple of 8");
  return PF_OK;
}

int check_cmajor(const void* ptr, int64_t ld, int64_t n_cols, const char* what) {
  if (((uintptr_t)ptr) % 16 || ld % 8 || ld < n_cols)
    return fail(PF_EINVAL_SHAPE, "%s: channel-major bf16 buffer needs a 16-byte aligned base and a row "
                "pitch that is a multiple of 8 elements and >= %lld (got %lld)", what, (long long)n_cols,
                (long long)ld);
  return PF_OK;
}

}  // namespace

int trimul(const pf_trimul_params* p, pf_pair_view za, pf_pair_view zb, pf_mask_view ma,
           pf_mask_view mb, pf_pair_view zg, pf_pair_view zo, int64_t n_i, int64_t n_j, int64_t n_k,
           int, int, int acc, void* ws, size_t ws_bytes, cudaStream_t st) {
  Arena ar(ws, ws_bytes);
  TrimulWs w;
  trimul_plan(ar, n_i, n_j, n_k, w);
  if (!ar.ok()) return fail(PF_EWORKSPACE, "trimul workspace too small");
  PF_TRY(check_out_view(zo));
  unsigned int* status;
  PF_TRY(device_status_ptr(&status));
  PF_TRY(ensure_attrs());
  PF_TRY(launch_proj(p, za, zb, ma, mb, n_i, n_j, n_k, w.a, w.b, w.ld_k, status, st));
  return launch_contract_out(p, w.a, w.ld_k, w.b, w.ld_k, n_i, n_j, n_k, w.x, w.ld_j, zg, zo, acc, status, st);
}

int trimul_project(const pf_trimul_params* p, pf_pair_view z, pf_mask_view m, int64_t n_rows,
                   int64_t n_cols, void* a, void* b, int64_t ld, cudaStream_t st) {
  PF_TRY(check_cmajor(a, ld, n_cols, "a"));
  PF_TRY(check_cmajor(b, ld, n_cols, "b"));
  unsigned int* status;
  PF_TRY(device_status_ptr(&status));
  PF_TRY(ensure_attrs());
  return launch_proj(p, z, z, m, m, n_rows, n_rows, n_cols, (__nv_bfloat16*)a, (__nv_bfloat16*)b, ld,
                     status, st);
}

size_t trimul_combine_ws_bytes(int64_t n_i, int64_t n_j) {
  return (size_t)CH * n_i * ((n_j + 7) / 8 * 8) * 2 + 256;
}

int trimul_combine(const pf_trimul_params* p, const void* a, const void* b, int64_t ld, int64_t n_i,
                   int64_t n_j, int64_t n_k, pf_pair_view zg, pf_pair_view zo, int acc, void* ws,
                   size_t ws_bytes, cudaStream_t st) {
  PF_TRY(check_cmajor(a, ld, n_k, "a"));
  PF_TRY(check_cmajor(b, ld, n_k, "b"));
  PF_TRY(check_out_view(zo));
  Arena ar(ws, ws_bytes);
  const int64_t ld_j = (n_j + 7) / 8 * 8;
  __nv_bfloat16* x = ar.take<__nv_bfloat16>((size_t)CH * n_i * ld_j);
  if (!ar.ok()) return fail(PF_EWORKSPACE, "trimul combine workspace too small");
  unsigned int* status;
  PF_TRY(device_status_ptr(&status));
  PF_TRY(ensure_attrs());
  return launch_contract_out(p, (const __nv_bfloat16*)a, ld, (const __nv_bfloat16*)b, ld, n_i, n_j, n_k, x,
                             ld_j, zg, zo, acc, status, st);
}


// ------------------------------------------------------------------ shared with the general path
int trimul_contract(const __nv_bfloat16* a, int64_t lda, const __nv_bfloat16* b, int64_t ldb, int64_t n_i,
                    int64_t n_j, int64_t n_k, int channels, __nv_bfloat16* x, int64_t ld_j, unsigned int* status,
                    cudaStream_t st) {
  PF_TRY(ensure_attrs());
  CUtensorMap ta, tb;
  {
    const uint64_t da[3] = {(uint64_t)n_k, (uint64_t)n_i, (uint64_t)channels};
    const uint64_t sa[2] = {(uint64_t)lda * 2, (uint64_t)n_i * lda * 2};
    const uint32_t ba[3] = {BK, BM, 1};
    PF_TRY(make_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a, da, sa, ba, CU_TENSOR_MAP_SWIZZLE_128B));
    const uint64_t db[3] = {(uint64_t)n_k, (uint64_t)n_j, (uint64_t)channels};
    const uint64_t sb[2] = {(uint64_t)ldb * 2, (uint64_t)n_j * ldb * 2};
    const uint32_t bb[3] = {BK, BN, 1};
    PF_TRY(make_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, b, db, sb, bb, CU_TENSOR_MAP_SWIZZLE_128B));
  }
  GemmArgs ga;
  ga.M = (int)n_i;
  ga.N = (int)n_j;
  ga.K = (int)n_k;
  ga.m_tiles = (int)((n_i + BM - 1) / BM);
  ga.n_tiles = (int)((n_j + BN - 1) / BN);
  ga.n_work = (int64_t)channels * ga.m_tiles * ga.n_tiles;
  ga.out = x;
  ga.ldo = ld_j;
  ga.out_bstride = (int64_t)n_i * ld_j;
  ga.status = status;
  {
    const int64_t grid_g = ga.n_work < sm_count() ? ga.n_work : sm_count();
    PF_LAUNCH_SCOPE_WORK(st, "k_trimul_bgemm", 2.0 * channels * (double)n_i * n_j * n_k, 'f');
    k_trimul_bgemm<<<(unsigned)grid_g, 192, GEMM_SMEM + 1024, st>>>(ta, tb, ga);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

}  // namespace tc
}  // namespace pf
