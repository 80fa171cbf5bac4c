// pf_tc_apb.cu -- AttentionPairBias pair bias on tcgen05: bias(h, r, s) = W_z LN_z(z(r, s)),
// c_z = 128, H = 16 heads (bf16 pair tensor, fp32 bias). One HBM pass over the pair tensor:
// TMA tile of 128 positions -> LayerNorm in place -> UMMA 128 x 16 x 128 -> fp32 stores, one
// head-plane row segment (128 B) per warp per head.
// Reference: opendde/model/modules/transformer.py:599-605 (standard_multihead_attention).

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

constexpr int C = 128, HB = 16, TILE = 128;
// z tile 32 KB, W 4 KB, LayerNorm parameters 1 KB, barriers and the TMEM slot
constexpr uint32_t S_LNP = 36864, S_BAR = S_LNP + 1024;
constexpr uint32_t APB_SMEM = S_BAR + 64;

struct ApbArgs {
  int64_t n_rows, n_cols, tiles_per_row;
  float* bias;
  int64_t hs, rs;
  const float *ln_w, *ln_b;
  unsigned int* status;
};

// The row is held as 64 registers of bf16 pairs (the tile helpers of the fused kernels), so that
// four CTAs fit per SM and their TMA loads, LayerNorms and stores overlap.
__global__ void __launch_bounds__(128, 3) k_apb_bias(const __grid_constant__ CUtensorMap tz,
                                                     const __grid_constant__ CUtensorMap tw, const ApbArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* g = smem_raw + (base - raw);
  const uint32_t sA = base, sB = base + 32768, bar_load = base + S_BAR, bar_mma = bar_load + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(g + S_BAR + 16);
  float* lnp = reinterpret_cast<float*>(g + S_LNP);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int64_t t = blockIdx.x;
  const int64_t r = t / a.tiles_per_row;
  const int64_t c0 = (t % a.tiles_per_row) * TILE;
  if (tid == 0) {
    mbar_init(bar_load, 1);
    mbar_init(bar_mma, 1);
    fence_barrier_init();
  }
  lnp[tid] = a.ln_w ? a.ln_w[tid] : 1.f;
  lnp[C + tid] = a.ln_b ? a.ln_b[tid] : 0.f;
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tid == 0) {
    mbar_arrive_expect_tx(bar_load, 32768 + 4096);
    tma_load_3d(sA, &tz, bar_load, 0, (int)c0, (int)r);
    tma_load_3d(sA + 16384, &tz, bar_load, 64, (int)c0, (int)r);
    tma_load_2d(sB, &tw, bar_load, 0, 0);          // 16 rows x 64 K
    tma_load_2d(sB + 2048, &tw, bar_load, 64, 0);
  }
  mbar_wait(bar_load, 0, a.status);
  {
    uint32_t zr[64];
    float m, rs;
    tile::load_row(g, tid, zr);
    tile::row_stats(zr, 1e-5f, m, rs);
    tile::store_norm_row(g, tid, zr, m, rs, lnp, lnp + C);
  }
  fence_proxy_async_smem();
  __syncthreads();
  if (tid == 0) {
    tc_fence_after();
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const uint32_t atom = kk >> 2, within = (kk & 3) * 32;
      umma_f16(tmem, sdesc(sA + atom * 16384 + within, 1024, SWZ_128B), sdesc(sB + atom * 2048 + within, 1024, SWZ_128B),
               idesc_f16(128, HB, true), kk > 0 ? 1u : 0u);
    }
    umma_commit(bar_mma);
  }
  mbar_wait(bar_mma, 0, a.status);
  tc_fence_after();
  uint32_t bv[16];
  tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16), bv);
  tmem_ld_wait();
  const int64_t col = c0 + tid;
  if (col < a.n_cols) {
#pragma unroll
    for (int h = 0; h < HB; ++h) a.bias[h * a.hs + r * a.rs + col] = __uint_as_float(bv[h]);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 32);
  }
}

}  // namespace

bool apb_pair_bias_supported(int c_z, int heads) { return c_z == C && heads == HB; }

int apb_pair_bias(const pf_apb_params* p, pf_pair_view z, int64_t n_rows, int64_t n_cols, float* bias, int64_t hs,
                  int64_t rs, cudaStream_t st) {
  if (z.row_stride % 8 || z.col_stride % 8 || ((uintptr_t)z.ptr) % 16)
    return fail(PF_EINVAL_SHAPE, "bf16 pair views need 16-byte alignment and strides multiple of 8 elements");
  static std::atomic<unsigned long long> attr_done{0};
  PF_TRY(once_per_device(attr_done, []() -> int {
    PF_CUDA_TRY(cudaFuncSetAttribute(k_apb_bias, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(APB_SMEM + 1024)));
    return PF_OK;
  }));
  unsigned int* status;
  PF_TRY(device_status_ptr(&status));
  CUtensorMap tz, tw;
  {
    const uint64_t dims[3] = {(uint64_t)C, (uint64_t)n_cols, (uint64_t)n_rows};
    const uint64_t str[2] = {(uint64_t)z.col_stride * 2, (uint64_t)z.row_stride * 2};
    const uint32_t box[3] = {64, TILE, 1};
    PF_TRY(make_tmap(&tz, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, z.ptr, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B));
    const uint64_t wd[2] = {(uint64_t)C, (uint64_t)HB};
    const uint64_t ws[1] = {(uint64_t)C * 2};
    const uint32_t wb[2] = {64, HB};
    PF_TRY(make_tmap(&tw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p->w_z, wd, ws, wb, CU_TENSOR_MAP_SWIZZLE_128B));
  }
  ApbArgs a{n_rows, n_cols, (n_cols + TILE - 1) / TILE, bias, hs, rs, p->ln_z_w, p->ln_z_b, status};
  const int64_t nt = n_rows * a.tiles_per_row;
  if (nt > 0x7fffffffll) return fail(PF_EUNSUPPORTED, "pair-bias grid too large");
  {
    // read z (bf16 C channels), write the fp32 bias of HB heads
    PF_LAUNCH_SCOPE_WORK(st, "k_apb_bias", (double)n_rows * n_cols * (2.0 * C + 4.0 * HB), 'b');
    k_apb_bias<<<(unsigned)nt, 128, APB_SMEM + 1024, st>>>(tz, tw, a);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

}  // namespace tc
}  // namespace pf
