// pf_tile_common.cuh -- building blocks of the persistent pair-tile kernels (sm_100a).
//
// A pair tile is 128 positions x 128 bf16 channels. In shared memory it is stored K-major
// with the 128-byte swizzle (two 64-channel atoms of 16 KB, row r of atom a at
// a*16384 + r*128, 16-byte chunks XOR-permuted by r & 7): the layout TMA writes for a box
// {64 channels, 128 positions} and the A-operand layout of a K = 128 UMMA.
//
// LayerNorm over the 128 channels of one position keeps the raw bf16 pairs in 64 registers
// and normalises in fp32 (two-pass mean / biased variance, eps inside the square root), as
// the reference's LayerNorm does (opendde/model/triangular/layers.py:226-269).
#pragma once
#include "pf_sm100.cuh"

namespace pf {
namespace tc {
namespace tile {
using namespace sm100;

constexpr int CH = 128;
constexpr uint32_t ATOM = 16384;   // one 64-channel x 128-position SW128 atom
constexpr uint32_t TILE_BYTES = 2 * ATOM;

__device__ __forceinline__ uint32_t chunk_off(int row, int chunk) {
  return (uint32_t)(chunk >> 3) * ATOM + sw128_off((uint32_t)row, (uint32_t)(chunk & 7));
}

// raw bf16 pairs of one row of a K-major SW128 tile -> r[64]
__device__ __forceinline__ void load_row(const uint8_t* tile, int row, uint32_t (&r)[64]) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const uint4 q = *reinterpret_cast<const uint4*>(tile + chunk_off(row, j));
    r[j * 4 + 0] = q.x; r[j * 4 + 1] = q.y; r[j * 4 + 2] = q.z; r[j * 4 + 3] = q.w;
  }
}

// mean and 1/sqrt(var + eps) of 128 bf16 values held as 64 pairs
__device__ __forceinline__ void row_stats(const uint32_t (&r)[64], float eps, float& mean, float& rstd) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 64; ++i) s += bf16lo(r[i]) + bf16hi(r[i]);
  mean = s * (1.0f / CH);
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < 64; ++i) {
    const float d0 = bf16lo(r[i]) - mean, d1 = bf16hi(r[i]) - mean;
    sq = fmaf(d0, d0, sq);
    sq = fmaf(d1, d1, sq);
  }
  rstd = rsqrtf(sq * (1.0f / CH) + eps);
}

// y = (x - mean) * rstd * g + b for the row, written K-major SW128 into `dst` (bf16).
// g, b: 128 fp32 values in shared memory, 16-byte aligned (b may be null).
__device__ __forceinline__ void store_norm_row(uint8_t* dst, int row, const uint32_t (&r)[64], float mean,
                                               float rstd, const float* g, const float* b) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float4 g0 = *reinterpret_cast<const float4*>(g + j * 8);
    const float4 g1 = *reinterpret_cast<const float4*>(g + j * 8 + 4);
    float4 b0 = make_float4(0.f, 0.f, 0.f, 0.f), b1 = b0;
    if (b) {
      b0 = *reinterpret_cast<const float4*>(b + j * 8);
      b1 = *reinterpret_cast<const float4*>(b + j * 8 + 4);
    }
    const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
    const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    float y[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint32_t w = r[j * 4 + e];
      y[e * 2] = fmaf((bf16lo(w) - mean) * rstd, gg[e * 2], bb[e * 2]);
      y[e * 2 + 1] = fmaf((bf16hi(w) - mean) * rstd, gg[e * 2 + 1], bb[e * 2 + 1]);
    }
    uint4 q;
    q.x = pack_bf16(y[0], y[1]); q.y = pack_bf16(y[2], y[3]);
    q.z = pack_bf16(y[4], y[5]); q.w = pack_bf16(y[6], y[7]);
    *reinterpret_cast<uint4*>(dst + chunk_off(row, j)) = q;
  }
}

// The 8 K-steps (K = 128) of D = A[128 x 128] * B[n x 128]^T from K-major SW128 tiles
// stored as two 64-channel atoms (A atom stride 16 KB, B atom stride b_atom_bytes).
__device__ __forceinline__ void umma_k128(uint32_t d_tmem, uint32_t sA, uint32_t sB, uint32_t b_atom_bytes,
                                          uint32_t idesc) {
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const uint32_t atom = kk >> 2, within = (kk & 3) * 32;
    const uint64_t ad = sdesc(sA + atom * ATOM + within, 1024, SWZ_128B);
    const uint64_t bd = sdesc(sB + atom * b_atom_bytes + within, 1024, SWZ_128B);
    umma_f16(d_tmem, ad, bd, idesc, kk > 0 ? 1u : 0u);
  }
}

}  // namespace tile
}  // namespace tc
}  // namespace pf
