// pf_tc_transition.cu -- pair Transition (LN -> SiLU(W_a y) * (W_b y) -> W_out, + residual) on
// tcgen05 tensor cores, c = 128, hidden = 4c = 512, bf16 in / fp32 accumulate.
//
// One CTA = 128 rows. The 512-wide hidden layer never leaves the SM: it is produced and consumed
// in 8 chunks of 64:
//   [a | b](chunk)  = LN(x) [W_a(chunk); W_b(chunk)]^T     UMMA 128x128x128 -> TMEM (2 slots)
//   h(chunk)        = silu(a) * b  -> bf16 -> shared memory (2 slots, SW128 K-major)
//   out            += h(chunk) W_o(:, chunk)^T             UMMA 128x128x64  -> TMEM
// Warps 0-3: LayerNorm prologue, silu epilogue per chunk, final residual epilogue (thread = row).
// Warp 4: MMA issuer. Warp 5: TMA producer for the x tile and the weight-chunk ring (2 slots).
// Reference: opendde/model/modules/primitives.py:182-217.

#include "pf_common.cuh"
#include "pf_prof.h"
#include "pf_sm100.cuh"
#include "pf_tc.h"
#include "pf_tmap.h"

namespace pf {
namespace tc {
using namespace sm100;

namespace {

constexpr int C = 128, HID = 512, CHUNK = 64, NCHUNK = HID / CHUNK, TILE = 128;

// shared memory (offsets from the 1 KB aligned base)
constexpr uint32_t S_A = 0;                 // LN(x): 2 atoms x 128 rows x 128 B = 32 KB
constexpr uint32_t S_W = 32768;             // 2 slots x 48 KB: [W_a;W_b] 2 atoms x 128 rows (32 KB) + W_o 128 rows x 128 B (16 KB)
constexpr uint32_t S_W_SLOT = 49152;
constexpr uint32_t S_H = S_W + 2 * S_W_SLOT;  // 2 slots x 16 KB: h 128 rows x 64 (128 B)
constexpr uint32_t S_BAR = S_H + 2 * 16384;
constexpr uint32_t TR_SMEM = S_BAR + 256;

struct TrArgs {
  int64_t rows;
  __nv_bfloat16* out;
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

__global__ void __launch_bounds__(192, 1) k_transition(const __grid_constant__ CUtensorMap tx,
                                                       const __grid_constant__ CUtensorMap twa,
                                                       const __grid_constant__ CUtensorMap twb,
                                                       const __grid_constant__ CUtensorMap two,
                                                       const TrArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* g = smem_raw + (base - raw);
  const uint32_t bars = base + S_BAR;
  // barriers: x_full @0, a_ready @8, w_full[2] @16, w_empty[2] @32, ab_full[2] @48,
  // ab_empty[2] @64, h_full[2] @80, h_empty[2] @96, out_full @112; TMEM slot @128
  const uint32_t b_x = bars, b_a = bars + 8, b_wf = bars + 16, b_we = bars + 32, b_abf = bars + 48,
                 b_abe = bars + 64, b_hf = bars + 80, b_he = bars + 96, b_out = bars + 112;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(g + S_BAR + 128);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t r0 = (int64_t)blockIdx.x * TILE;

  if (tid == 0) {
    mbar_init(b_x, 1);
    mbar_init(b_a, 4);
    for (int s = 0; s < 2; ++s) {
      mbar_init(b_wf + 8 * s, 1);
      mbar_init(b_we + 8 * s, 1);
      mbar_init(b_abf + 8 * s, 1);
      mbar_init(b_abe + 8 * s, 4);
      mbar_init(b_hf + 8 * s, 4);
      mbar_init(b_he + 8 * s, 1);
    }
    mbar_init(b_out, 1);
    fence_barrier_init();
  }
  if (warp == 4) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // D_ab slots at 0 / 128, D_out at 256

  if (warp == 5) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      mbar_arrive_expect_tx(b_x, 32768);
      tma_load_2d(base + S_A, &tx, b_x, 0, (int)r0);
      tma_load_2d(base + S_A + 16384, &tx, b_x, 64, (int)r0);
      for (int hc = 0; hc < NCHUNK; ++hc) {
        const int s = hc & 1;
        if (hc >= 2 && !mbar_wait(b_we + 8 * s, ((hc - 2) >> 1) & 1, a.status)) break;
        const uint32_t w = base + S_W + s * S_W_SLOT, full = b_wf + 8 * s;
        mbar_arrive_expect_tx(full, S_W_SLOT);
        // atom k (K 64k..64k+63): rows 0..63 = W_a chunk, rows 64..127 = W_b chunk
        tma_load_2d(w, &twa, full, 0, hc * CHUNK);
        tma_load_2d(w + 8192, &twb, full, 0, hc * CHUNK);
        tma_load_2d(w + 16384, &twa, full, 64, hc * CHUNK);
        tma_load_2d(w + 16384 + 8192, &twb, full, 64, hc * CHUNK);
        tma_load_2d(w + 32768, &two, full, hc * CHUNK, 0);  // W_o[:, chunk] 128 rows x 64
      }
    }
  } else if (warp == 4) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_ab = idesc_f16(128, 128, true);
      constexpr uint32_t id_o = idesc_f16(128, 128, true);
      bool ok = mbar_wait(b_a, 0, a.status);  // LN(x) in smem
      auto mma_ab = [&](int hc) {
        const int s = hc & 1;
        const uint32_t w = base + S_W + s * S_W_SLOT;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t atom = kk >> 2, within = (kk & 3) * 32;
          umma_f16(tmem + 128 * s, sdesc(base + S_A + atom * 16384 + within, 1024, SWZ_128B),
                   sdesc(w + atom * 16384 + within, 1024, SWZ_128B), id_ab, kk > 0 ? 1u : 0u);
        }
        umma_commit(b_abf + 8 * s);
      };
      for (int hc = 0; hc < 2 && ok; ++hc) {
        ok = mbar_wait(b_wf + 8 * hc, 0, a.status);
        tc_fence_after();
        mma_ab(hc);
      }
      for (int hc = 0; hc < NCHUNK && ok; ++hc) {
        const int s = hc & 1;
        ok = mbar_wait(b_hf + 8 * s, (hc >> 1) & 1, a.status);
        tc_fence_after();
        const uint32_t hb = base + S_H + s * 16384, w = base + S_W + s * S_W_SLOT + 32768;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          umma_f16(tmem + 256, sdesc(hb + kk * 32, 1024, SWZ_128B), sdesc(w + kk * 32, 1024, SWZ_128B), id_o,
                   (hc > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(b_he + 8 * s);  // h slot s free when this MMA finishes
        umma_commit(b_we + 8 * s);  // weight slot s free (its ab and out MMAs are done)
        if (hc + 2 < NCHUNK) {
          ok = ok && mbar_wait(b_wf + 8 * s, ((hc + 2) >> 1) & 1, a.status);
          ok = ok && mbar_wait(b_abe + 8 * s, (hc >> 1) & 1, a.status);  // D_ab slot read out
          tc_fence_after();
          mma_ab(hc + 2);
        }
      }
      umma_commit(b_out);
    }
  } else {
    // ---------------------------------------------------------------- compute warps (thread = row)
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    mbar_wait(b_x, 0, a.status);
    {
      // LayerNorm in place (two 64-channel SW128 atoms)
      float v[C];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const uint4 q = *reinterpret_cast<const uint4*>(g + S_A + (j >> 3) * 16384 + sw128_off(tid, j & 7));
        v[j * 8 + 0] = bf16lo(q.x); v[j * 8 + 1] = bf16hi(q.x);
        v[j * 8 + 2] = bf16lo(q.y); v[j * 8 + 3] = bf16hi(q.y);
        v[j * 8 + 4] = bf16lo(q.z); v[j * 8 + 5] = bf16hi(q.z);
        v[j * 8 + 6] = bf16lo(q.w); v[j * 8 + 7] = bf16hi(q.w);
      }
      float sm = 0.f;
#pragma unroll
      for (int c = 0; c < C; ++c) sm += v[c];
      const float mean = sm * (1.0f / C);
      float sq = 0.f;
#pragma unroll
      for (int c = 0; c < C; ++c) {
        const float d = v[c] - mean;
        sq += d * d;
      }
      const float rstd = rsqrtf(sq * (1.0f / C) + 1e-5f);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float y[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int c = j * 8 + e;
          y[e] = (v[c] - mean) * rstd * __ldg(a.ln_w + c) + __ldg(a.ln_b + c);
        }
        uint4 q;
        q.x = pack_bf16(y[0], y[1]); q.y = pack_bf16(y[2], y[3]);
        q.z = pack_bf16(y[4], y[5]); q.w = pack_bf16(y[6], y[7]);
        *reinterpret_cast<uint4*>(g + S_A + (j >> 3) * 16384 + sw128_off(tid, j & 7)) = q;
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(b_a);
    for (int hc = 0; hc < NCHUNK; ++hc) {
      const int s = hc & 1;
      mbar_wait(b_abf + 8 * s, (hc >> 1) & 1, a.status);
      tc_fence_after();
      uint32_t av[32], bv[32];
      uint32_t hv[32];  // 64 bf16 of h for this row
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        tmem_ld32(tmem + 128 * s + lane_base + half * 32, av);
        tmem_ld32(tmem + 128 * s + lane_base + 64 + half * 32, bv);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 16; ++e)
          hv[half * 16 + e] = pack_bf16(silu_fast(__uint_as_float(av[2 * e])) * __uint_as_float(bv[2 * e]),
                                        silu_fast(__uint_as_float(av[2 * e + 1])) * __uint_as_float(bv[2 * e + 1]));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(b_abe + 8 * s);  // D_ab slot may be overwritten
      if (hc >= 2) mbar_wait(b_he + 8 * s, ((hc - 2) >> 1) & 1, a.status);
      uint8_t* hb = g + S_H + s * 16384;
#pragma unroll
      for (int ch = 0; ch < 8; ++ch)
        *reinterpret_cast<uint4*>(hb + sw128_off(tid, ch)) =
            make_uint4(hv[ch * 4 + 0], hv[ch * 4 + 1], hv[ch * 4 + 2], hv[ch * 4 + 3]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(b_hf + 8 * s);
    }
    // residual epilogue
    mbar_wait(b_out, 0, a.status);
    tc_fence_after();
    const int64_t row = r0 + tid;
    const bool valid = row < a.rows;
    __nv_bfloat16* op = a.out + (valid ? row : 0) * a.out_stride;
#pragma unroll 1
    for (int cc = 0; cc < C; cc += 32) {
      uint32_t ov[32];
      tmem_ld32(tmem + 256 + lane_base + cc, ov);
      tmem_ld_wait();
      if (valid) {
        uint4* dst = reinterpret_cast<uint4*>(op + cc);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float u[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) u[k] = __uint_as_float(ov[e * 8 + k]);
          if (a.accumulate) {
            const uint4 old = dst[e];
            u[0] += bf16lo(old.x); u[1] += bf16hi(old.x); u[2] += bf16lo(old.y); u[3] += bf16hi(old.y);
            u[4] += bf16lo(old.z); u[5] += bf16hi(old.z); u[6] += bf16lo(old.w); u[7] += bf16hi(old.w);
          }
          uint4 w;
          w.x = pack_bf16(u[0], u[1]); w.y = pack_bf16(u[2], u[3]);
          w.z = pack_bf16(u[4], u[5]); w.w = pack_bf16(u[6], u[7]);
          dst[e] = w;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
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
  static bool attr = false;
  if (!attr) {
    PF_CUDA_TRY(cudaFuncSetAttribute(k_transition, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(TR_SMEM + 1024)));
    attr = true;
  }
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
  TrArgs a{rows, (__nv_bfloat16*)out, os, p->ln_w, p->ln_b, acc, status};
  const int64_t nt = (rows + TILE - 1) / TILE;
  if (nt > 0x7fffffffll) return fail(PF_EUNSUPPORTED, "transition grid too large");
  {
    PF_LAUNCH_SCOPE(st, "k_transition");
    k_transition<<<(unsigned)nt, 192, TR_SMEM + 1024, st>>>(tx, twa, twb, two, a);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

}  // namespace tc
}  // namespace pf
