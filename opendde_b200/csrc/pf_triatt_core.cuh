// pf_triatt_core.cuh -- persistent flash-style triangle-attention core for sm_100a (included by
// pf_tc_triatt.cu inside namespace pf::tc::{anon}).
//
// Work item = two rows (i0, i0+1) of the pair plane x one head x 128 queries; one CTA per SM
// walks items w = blockIdx.x, blockIdx.x + gridDim.x, ... and a key-tile "step" stream runs
// through a 3-stage TMA ring continuously across items. The two rows of an item share the
// triangle-bias tile (bias[h][j][k] does not depend on i).
// Warp roles (352 threads):
//   warps 0-3  softmax for row A (thread = query; TMEM lanes 0..127)
//   warps 4-7  softmax for row B
//   warp 8     TMA producer: per step the bias tile, K, V^T and key-mask rows of both rows
//   warp 9     S issuer (one thread) and TMEM owner
//   warp 10    P.V issuer (one thread)
// TMEM (per row R, base 256*R): S [0,128) f16 accumulator (one value per column), P [128,192)
// (f16, two per column), [O | l] [192,240) fp32, Q [240,256) (f16, two per column).
//   S = Q K^T           A = Q (TMEM), B = K tile (smem, 64B swizzle), f16 x f16 -> f16
//   [O | l] += P [V^T; 1]^T   A = P (TMEM), B = V^T tile with a row of ones appended
//                       (smem, 128B swizzle), -> fp32; l is the sum of exactly the P used.
// P has its own columns, so S of the next step is computed while the softmax threads are still
// exponentiating the current one: a softmax thread reads S(t), tells the MMA thread that the S
// columns are free (for the item's last tile, after writing the next item's Q into the Q
// columns), and the MMA thread issues S(t+1) at once; P(t) and PV(t) follow. Per step and row
// the softmax threads therefore wait only for their own previous P.V (before overwriting P or
// rescaling O), not for a P -> PV -> S round trip through the tensor pipe.
// MMA thread, per step t: S_A(t+1), S_B(t+1) (each after its row has read S(t)), then PV_A(t),
// PV_B(t) (each after its row's P(t)), then release of the stage's shared memory.
// Softmax is packed f16x2 on log2-domain logits read straight from TMEM (tcgen05.ld
// .pack::16b): + bias, + key mask (0 / -inf), max, - m, ex2.f16x2. The running max is updated
// lazily (O, L rescaled in TMEM only when a tile's max exceeds it by more than 8).
// Rows without any fully valid key ("uniform" rows) take the reference's limit: logits
// 1e9*(m-1) ~ -1e9 for every key, i.e. a uniform average of V over the existing keys.

struct CoreArgs {
  int64_t n_rows, n_q, n_tiles_k, n_qt, n_items;
  int heads;                // H (d = 32 each); o rows hold heads * 32 channels
  const uint8_t* flags;     // [n_rows][n_tiles_k]  TF_*
  const uint8_t* rowflags;  // [n_rows]  bit 0: uniform row
  const __half* q;          // [(i*heads+h)*n_q + j][D] f16, pre-scaled by log2(e)/sqrt(d)
  __nv_bfloat16* o;         // [(i*n_q + j)][heads*D]
  unsigned int* status;
};

#ifndef PF_CORE_FMA_PAIRS
#define PF_CORE_FMA_PAIRS 4
#endif
constexpr int CORE_THREADS = 352;
constexpr int CORE_STAGES = 3;
// per-stage layout (bytes from the stage base)
constexpr uint32_t CS_KA = 0;                  // 128 x 64 B (SW64) f16
constexpr uint32_t CS_KB = 8192;
constexpr uint32_t CS_VTA = 16384;             // 2 atoms x 48 rows x 128 B (SW128) f16; rows 32..47 = [1; 0]
constexpr uint32_t CS_VTB = 16384 + 12288;
constexpr uint32_t CS_VT_ATOM = 48 * 128;
constexpr uint32_t CS_BIAS = 16384 + 24576;    // 2 atoms x 128 rows x 128 B (SW128) f16
constexpr uint32_t CS_MBA = CS_BIAS + 32768;   // 128 f16
constexpr uint32_t CS_MBB = CS_MBA + 256;
constexpr uint32_t CS_BYTES = 75776;           // 74 KB
constexpr uint32_t CC_BAR = CORE_STAGES * CS_BYTES;
constexpr uint32_t CORE3_SMEM = CC_BAR + 256;
static_assert(CS_BYTES % 1024 == 0 && CS_BIAS % 1024 == 0 && CS_VTB % 1024 == 0, "1 KB alignment");
static_assert(CS_MBB + 256 <= CS_BYTES, "stage overflow");
static_assert(CORE3_SMEM + 1024 <= 227 * 1024, "dynamic shared memory limit");

// TMEM column offsets within a row's 256-column block
constexpr uint32_t T_S = 0, T_P = 128, T_O = 192, T_Q = 240;

__device__ __forceinline__ int next_tile(const uint8_t* fa, const uint8_t* fb, int kt, int n_tiles) {
  while (kt < n_tiles && fa[kt] == TF_SKIP && (fb == nullptr || fb[kt] == TF_SKIP)) ++kt;
  return kt;
}

struct Item {
  int64_t i0;
  int h, jt;
  bool has_b;
  const uint8_t* fa;
  const uint8_t* fb;
};

// NH > 0: the head count as a compile-time constant (the c = 128 path); 0: CoreArgs::heads.
template <int NH>
__device__ __forceinline__ int core_heads(const CoreArgs& a) { return NH > 0 ? NH : a.heads; }

template <int NH>
__device__ __forceinline__ Item decode_item(const CoreArgs& a, int64_t w) {
  const int heads = core_heads<NH>(a);
  Item it;
  it.jt = (int)(w % a.n_qt);
  it.h = (int)((w / a.n_qt) % heads);
  it.i0 = 2 * (w / (a.n_qt * heads));
  it.has_b = it.i0 + 1 < a.n_rows;
  it.fa = a.flags + it.i0 * a.n_tiles_k;
  it.fb = it.has_b ? it.fa + a.n_tiles_k : nullptr;
  return it;
}

__device__ __forceinline__ void tmem_ld32_16b(uint32_t taddr, uint32_t (&r)[32]) {
  // 64 columns of 16-bit values -> 32 registers of packed pairs
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.pack::16b.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// One query row of a 128-key tile in log2 units, packed f16x2: x[p] holds keys (2p, 2p+1).
// BIAS: add the triangle-bias row (SW128 tile in smem); uniform rows (BIAS = false) drop the
// logits entirely. MASK: add the key-mask row (0 / -inf). Returns the packed running max.
// The shared-memory rows are read 32 keys at a time (16 + 16 registers in flight).
template <bool BIAS, bool MASK>
__device__ __forceinline__ uint32_t tile_logits(uint32_t t_s, const uint8_t* brow, const uint8_t* mbrow,
                                                int row_tid, uint32_t (&x)[64]) {
  uint32_t mx = 0xFC00FC00u;  // (-inf, -inf)
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    uint32_t v[32];
    if (BIAS) tmem_ld32_16b(t_s + c * 64, v);  // keys 64c .. 64c+63
#pragma unroll
    for (int hq = 0; hq < 2; ++hq) {
      uint4 b[4], mv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ch = c * 8 + hq * 4 + e;  // 16-byte chunk = 8 keys
        if (BIAS) b[e] = *reinterpret_cast<const uint4*>(brow + (ch >> 3) * 16384 + sw128_off(row_tid, ch & 7));
        if (MASK) mv[e] = reinterpret_cast<const uint4*>(mbrow)[ch];
      }
      if (BIAS && hq == 0) tmem_ld_wait();
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int q = hq * 4 + e, ch = c * 8 + q;
        uint32_t y0 = 0u, y1 = 0u, y2 = 0u, y3 = 0u;
        if (BIAS) {
          y0 = hadd2_u(v[q * 4 + 0], b[e].x);
          y1 = hadd2_u(v[q * 4 + 1], b[e].y);
          y2 = hadd2_u(v[q * 4 + 2], b[e].z);
          y3 = hadd2_u(v[q * 4 + 3], b[e].w);
        }
        if (MASK) {
          y0 = hadd2_u(y0, mv[e].x);
          y1 = hadd2_u(y1, mv[e].y);
          y2 = hadd2_u(y2, mv[e].z);
          y3 = hadd2_u(y3, mv[e].w);
        }
        mx = hmax2_u(mx, hmax2_u(hmax2_u(y0, y1), hmax2_u(y2, y3)));
        x[ch * 4 + 0] = y0;
        x[ch * 4 + 1] = y1;
        x[ch * 4 + 2] = y2;
        x[ch * 4 + 3] = y3;
      }
    }
  }
  return mx;
}

// Softmax thread: copy its query row (32 f16) of item `it`, row r, into the TMEM Q columns.
template <int NH>
__device__ __forceinline__ void load_q_row(const CoreArgs& a, const Item& it, int r, int row_tid,
                                           uint32_t tmem_row, uint32_t lane_base) {
  const int64_t j = (int64_t)it.jt * TILE + row_tid;
  uint32_t qv[16];
  if (j < a.n_q) {
    const uint4* src = reinterpret_cast<const uint4*>(a.q + (((it.i0 + r) * core_heads<NH>(a) + it.h) * a.n_q + j) * D);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint4 u = src[e];
      qv[e * 4 + 0] = u.x; qv[e * 4 + 1] = u.y; qv[e * 4 + 2] = u.z; qv[e * 4 + 3] = u.w;
    }
  } else {
#pragma unroll
    for (int e = 0; e < 16; ++e) qv[e] = 0u;
  }
  tmem_st16(tmem_row + lane_base + T_Q, qv);
}

template <int NH>
__global__ void __launch_bounds__(CORE_THREADS, 1) k_triatt_core(const __grid_constant__ CUtensorMap tk,
                                                                 const __grid_constant__ CUtensorMap tvt,
                                                                 const __grid_constant__ CUtensorMap tb,
                                                                 const __grid_constant__ CUtensorMap tmb,
                                                                 const CoreArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* g = smem_raw + (base - raw);
  const uint32_t bars = base + CC_BAR;
  // barriers: full[3] @0, empty[3] @24, then per row r: s @48+8r (S ready), p @64+8r (P
  // written), o @80+8r (P.V done), sfree @96+8r (S read: its columns are free, and Q is in
  // place for the next S), ofree @112+8r (O read out by the item epilogue); drain @128;
  // TMEM slot @200
  const uint32_t bar_full0 = bars, bar_empty0 = bars + 24;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(g + CC_BAR + 200);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_tiles = (int)a.n_tiles_k;

  if (tid == 0) {
    for (int s = 0; s < CORE_STAGES; ++s) {
      mbar_init(bar_full0 + 8 * s, 1);
      mbar_init(bar_empty0 + 8 * s, 1);
    }
    for (int r = 0; r < 2; ++r) {
      mbar_init(bars + 48 + 8 * r, 1);    // S ready (tcgen05.commit)
      mbar_init(bars + 64 + 8 * r, 4);    // P written (one arrive per softmax warp)
      mbar_init(bars + 80 + 8 * r, 1);    // P.V done (tcgen05.commit)
      mbar_init(bars + 96 + 8 * r, 4);    // S read / Q written
      mbar_init(bars + 112 + 8 * r, 4);   // O/L read out, free for the next item
    }
    mbar_init(bars + 128, 2);             // drain (one commit per MMA issuer)
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  // constant rows 32..47 of every V^T buffer: row 32 = 1.0 (f16), rows 33..47 = 0
  for (int idx = tid; idx < CORE_STAGES * 2 * 2 * 16 * 8; idx += CORE_THREADS) {
    const int ch = idx & 7, rr = 32 + ((idx >> 3) & 15), atom = (idx >> 7) & 1, which = (idx >> 8) & 1,
              st = idx >> 9;
    const uint32_t one2 = (rr == 32) ? 0x3C003C00u : 0u;
    *reinterpret_cast<uint4*>(g + st * CS_BYTES + (which ? CS_VTB : CS_VTA) + atom * CS_VT_ATOM + sw128_off(rr, ch)) =
        make_uint4(one2, one2, one2, one2);
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t step = 0;
      bool ok = true;
      for (int64_t w = blockIdx.x; w < a.n_items && ok; w += gridDim.x) {
        const Item it = decode_item<NH>(a, w);
        const int ihA = (int)(it.i0 * core_heads<NH>(a) + it.h), ihB = ihA + core_heads<NH>(a);
        const uint32_t bytes = 32768 + (8192 + 8192 + 256) * (it.has_b ? 2 : 1);
        for (int kt = next_tile(it.fa, it.fb, 0, n_tiles); kt < n_tiles && ok;
             kt = next_tile(it.fa, it.fb, kt + 1, n_tiles), ++step) {
          const uint32_t s = step % CORE_STAGES, u = step / CORE_STAGES;
          if (u > 0) ok = mbar_wait(bar_empty0 + 8 * s, (u - 1) & 1, a.status);
          if (!ok) break;
          const uint32_t sb = base + s * CS_BYTES, full = bar_full0 + 8 * s;
          const int k0 = kt * TILE;
          mbar_arrive_expect_tx(full, bytes);
          tma_load_3d(sb + CS_BIAS, &tb, full, k0, it.jt * TILE, it.h);
          tma_load_3d(sb + CS_BIAS + 16384, &tb, full, k0 + 64, it.jt * TILE, it.h);
          tma_load_3d(sb + CS_KA, &tk, full, 0, k0, ihA);
          tma_load_3d(sb + CS_VTA, &tvt, full, k0, 0, ihA);
          tma_load_3d(sb + CS_VTA + CS_VT_ATOM, &tvt, full, k0 + 64, 0, ihA);
          tma_load_2d(sb + CS_MBA, &tmb, full, k0, (int)it.i0);
          if (it.has_b) {
            tma_load_3d(sb + CS_KB, &tk, full, 0, k0, ihB);
            tma_load_3d(sb + CS_VTB, &tvt, full, k0, 0, ihB);
            tma_load_3d(sb + CS_VTB + CS_VT_ATOM, &tvt, full, k0 + 64, 0, ihB);
            tma_load_2d(sb + CS_MBB, &tmb, full, k0, (int)(it.i0 + 1));
          }
        }
      }
    }
  } else if (warp == 9 || warp == 10) {
    // ------------------------------------------------------------ MMA issuers
    // warp 9 issues every S = Q K^T, warp 10 every [O | l] += P [V^T; 1]^T; both walk the same
    // step sequence. With S and P.V in separate threads, a row's next S waits only for that
    // row's softmax to read the current S, never for the other row's P (the rows stay
    // decoupled without polling).
    if (lane == 0) {
      const bool s_issuer = warp == 9;
      constexpr uint32_t id_s = idesc_f16_f16acc(128, 128);               // f16 x f16 -> f16
      constexpr uint32_t id_o = idesc_f16(128, 48, false);                // f16 x f16 -> fp32
      uint32_t ns[2] = {0, 0};   // S issued per row (sfree phases)
      uint32_t np[2] = {0, 0};   // P.V issued per row (p phases)
      uint32_t ni[2] = {0, 0};   // items begun per row (ofree phases)
      bool ok = true;
      // Descriptors of stage 0, row A; other stages / row B / K-steps differ only in the start
      // address field (address >> 4), so each MMA's descriptor is one 64-bit add.
      const uint64_t dK0 = sdesc(base + CS_KA, 512, SWZ_64B);
      const uint64_t dV0 = sdesc(base + CS_VTA, 1024, SWZ_128B);
      constexpr uint64_t kStageD = CS_BYTES >> 4, kRowKD = (CS_KB - CS_KA) >> 4, kRowVD = (CS_VTB - CS_VTA) >> 4;
      // S of row r for the step in stage s, once row r's softmax has read its previous S
      auto issue_s = [&](int r, uint32_t s) {
        ok = ok && mbar_wait(bars + 96 + 8 * r, ns[r] & 1, a.status);
        tc_fence_after();
        const uint32_t tb_r = tmem + 256u * r;
        const uint64_t dk = dK0 + s * kStageD + (r ? kRowKD : 0);
        umma_f16_ts(tb_r + T_S, tb_r + T_Q, dk, id_s, 0u);
        umma_f16_ts(tb_r + T_S, tb_r + T_Q + 8, dk + 2, id_s, 1u);  // +32 B
        umma_commit(bars + 48 + 8 * r);
        ns[r] += 1;
      };
      int64_t w = blockIdx.x;
      Item it;
      int kt = n_tiles;
      uint32_t step = 0;
      if (w < a.n_items) {
        it = decode_item<NH>(a, w);
        kt = next_tile(it.fa, it.fb, 0, n_tiles);
        if (s_issuer) {
          ok = mbar_wait(bar_full0, 0, a.status);
          tc_fence_after();
          for (int r = 0; r < (it.has_b ? 2 : 1) && ok; ++r) issue_s(r, 0);
        }
      }
      bool first = true;
      while (w < a.n_items && ok) {
        const uint32_t s = step % CORE_STAGES;
        // the next step (same item or the next one)
        int64_t w2 = w;
        Item it2 = it;
        int kt2 = next_tile(it.fa, it.fb, kt + 1, n_tiles);
        bool first2 = false;
        if (kt2 >= n_tiles) {
          w2 = w + gridDim.x;
          if (w2 < a.n_items) {
            it2 = decode_item<NH>(a, w2);
            kt2 = next_tile(it2.fa, it2.fb, 0, n_tiles);
            first2 = true;
          }
        }
        const bool more = w2 < a.n_items;
        const int nr = it.has_b ? 2 : 1;
        if (s_issuer) {
          // S of the next step, for each row as soon as it has read this step's S
          if (more) {
            const uint32_t s2 = (step + 1) % CORE_STAGES;
            ok = ok && mbar_wait(bar_full0 + 8 * s2, ((step + 1) / CORE_STAGES) & 1, a.status);
            tc_fence_after();
            for (int r = 0; r < (it2.has_b ? 2 : 1) && ok; ++r) issue_s(r, s2);
          }
        } else {
          // P.V of this step, for each row once its P is written
          for (int r = 0; r < nr && ok; ++r) {
            const uint32_t tb_r = tmem + 256u * r;
            ok = mbar_wait(bars + 64 + 8 * r, np[r] & 1, a.status);
            if (first && ni[r] > 0) ok = ok && mbar_wait(bars + 112 + 8 * r, (ni[r] - 1) & 1, a.status);
            tc_fence_after();
            const uint64_t dv = dV0 + s * kStageD + (r ? kRowVD : 0);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              // key step kk: atom kk/4 (6 KB apart), 32 B into the 128 B swizzle row per step
              const uint64_t d = dv + (uint64_t)((kk >> 2) * (CS_VT_ATOM >> 4) + (kk & 3) * 2);
              umma_f16_ts(tb_r + T_O, tb_r + T_P + kk * 8, d, id_o, (!first || kk > 0) ? 1u : 0u);
            }
            umma_commit(bars + 80 + 8 * r);
            np[r] += 1;
            if (first) ni[r] += 1;
          }
          // the stage's K tiles were read by this step's S (done: the softmax read S before
          // writing P) and its V tiles by these P.V MMAs
          umma_commit(bar_empty0 + 8 * s);
        }
        w = w2;
        it = it2;
        kt = kt2;
        first = first2;
        ++step;
      }
      umma_commit(bars + 128);  // drain (count 2): every MMA of both issuers complete
      mbar_wait_drain(bars + 128, 0);
    }
  } else {
    // ------------------------------------------------------------ softmax (row r)
    const int r = warp >> 2;          // 0: row A, 1: row B
    const int q4 = warp & 3;          // TMEM lane quarter
    const int row_tid = tid & 127;    // query within the tile
    const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
    const uint32_t tb_r = tmem + 256u * r;
    const uint32_t bar_s = bars + 48 + 8 * r, bar_p = bars + 64 + 8 * r, bar_o = bars + 80 + 8 * r,
                   bar_sf = bars + 96 + 8 * r, bar_of = bars + 112 + 8 * r;
    uint32_t t = 0;
    bool ok = true;
    // Q of this row's first item, then "S columns free" for the first S
    if (blockIdx.x < a.n_items) {
      const Item it0 = decode_item<NH>(a, blockIdx.x);
      if (r == 0 || it0.has_b) {
        load_q_row<NH>(a, it0, r, row_tid, tb_r, lane_base);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_sf);
      }
    }
    for (int64_t w = blockIdx.x; w < a.n_items && ok; w += gridDim.x) {
      const Item it = decode_item<NH>(a, w);
      if (r == 1 && !it.has_b) break;  // rows B end at the odd last row pair
      const int64_t i = it.i0 + r;
      const uint8_t* fr = r ? it.fb : it.fa;
      const bool uniform = (a.rowflags[i] & 1) != 0;
      float m_run = -INFINITY;
      int it_in = 0;
      for (int kt = next_tile(it.fa, it.fb, 0, n_tiles); kt < n_tiles && ok; ++t, ++it_in) {
        const uint32_t s = t % CORE_STAGES;
        const uint8_t fl = fr[kt];
        const uint8_t* sb = g + s * CS_BYTES;
        ok = __all_sync(0xffffffffu, mbar_wait(bar_full0 + 8 * s, (t / CORE_STAGES) & 1, a.status));
        ok = __all_sync(0xffffffffu, mbar_wait(bar_s, t & 1, a.status)) && ok;
        tc_fence_after();
        uint32_t x[64];
        uint32_t mx;
        // warp-uniform choice of the specialised body: no branch inside the chunk loops, so
        // the shared-memory loads of a 64-key half are issued back to back
        const uint8_t* mbrow = sb + (r ? CS_MBB : CS_MBA);
        const uint8_t* brow = sb + CS_BIAS;
        if (uniform)
          mx = tile_logits<false, true>(tb_r + T_S + lane_base, brow, mbrow, row_tid, x);
        else if (fl != TF_NOADD)
          mx = tile_logits<true, true>(tb_r + T_S + lane_base, brow, mbrow, row_tid, x);
        else
          mx = tile_logits<true, false>(tb_r + T_S + lane_base, brow, mbrow, row_tid, x);
        // S is in registers: its columns are free for the next S. Before the item's last S is
        // released, the next item's Q goes into the Q columns (every S of this item is done).
        kt = next_tile(it.fa, it.fb, kt + 1, n_tiles);
        if (kt >= n_tiles) {
          const int64_t wn = w + gridDim.x;
          if (wn < a.n_items) {
            const Item itn = decode_item<NH>(a, wn);
            if (r == 0 || itn.has_b) {
              load_q_row<NH>(a, itn, r, row_tid, tb_r, lane_base);
              tmem_st_wait();
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_sf);
        const float tmax = fmaxf(f16lo(mx), f16hi(mx));
        const bool need = tmax > m_run + 8.0f;
        // the previous P.V must be done before O is rescaled or P is overwritten (within an
        // item; the item epilogue already waited for the previous item's last one)
        if (it_in > 0) {
          ok = __all_sync(0xffffffffu, mbar_wait(bar_o, (t - 1) & 1, a.status)) && ok;
          tc_fence_after();
        }
        // lazy rescale, warp-collective (tcgen05.ld/st need all lanes)
        if (__any_sync(0xffffffffu, need && m_run != -INFINITY) && it_in > 0) {
          const float alpha = (need && m_run != -INFINITY) ? ex2_approx(m_run - tmax) : 1.0f;
          uint32_t ov[16], lv[16];   // [O | l] columns 0..15 and 32..47 (l in column 32)
          tmem_ld16(tb_r + T_O + lane_base, ov);
          tmem_ld16(tb_r + T_O + 32 + lane_base, lv);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
            lv[e] = __float_as_uint(__uint_as_float(lv[e]) * alpha);
          }
          tmem_st16(tb_r + T_O + lane_base, ov);
          tmem_st16(tb_r + T_O + 32 + lane_base, lv);
          tmem_ld16(tb_r + T_O + 16 + lane_base, ov);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 16; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
          tmem_st16(tb_r + T_O + 16 + lane_base, ov);
        }
        if (need) m_run = tmax;
        const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
        const uint32_t mh = cvt_f16x2(m_use, m_use);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t p[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            // PF_CORE_FMA_PAIRS of every 16 pairs (evenly spread) on the FMA pipe, the rest on MUFU
            const uint32_t y = hsub2_u(x[c * 16 + e], mh);
            p[e] = ((e * PF_CORE_FMA_PAIRS) % 16 < PF_CORE_FMA_PAIRS) ? ex2_poly_f16x2(y) : ex2_f16x2(y);
          }
          tmem_st16(tb_r + T_P + lane_base + c * 16, p);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_p);
      }
      // item epilogue: o = O / l
      ok = __all_sync(0xffffffffu, mbar_wait(bar_o, (t - 1) & 1, a.status)) && ok;
      tc_fence_after();
      uint32_t o0[16], o1[16], lv[16];
      tmem_ld16(tb_r + T_O + lane_base, o0);
      tmem_ld16(tb_r + T_O + 16 + lane_base, o1);
      tmem_ld16(tb_r + T_O + 32 + lane_base, lv);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_of);
      const int64_t j = (int64_t)it.jt * TILE + row_tid;
      // A logit past the f16 range (|q.k| log2(e)/sqrt(d) > 65504) turns the row sum into inf
      // or NaN: report it (status bit 1) instead of returning a silently wrong row.
      if (j < a.n_q && !(__uint_as_float(lv[0]) <= 3.0e38f)) atomicOr(a.status, 2u);
      if (j < a.n_q) {
        const float l = __uint_as_float(lv[0]);
        const float inv = l > 0.f ? 1.0f / l : 0.f;
        uint4* dst = reinterpret_cast<uint4*>(a.o + ((int64_t)i * a.n_q + j) * (core_heads<NH>(a) * D) + it.h * D);
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          uint4 w0;
          w0.x = pack_bf16(__uint_as_float(o0[e * 8 + 0]) * inv, __uint_as_float(o0[e * 8 + 1]) * inv);
          w0.y = pack_bf16(__uint_as_float(o0[e * 8 + 2]) * inv, __uint_as_float(o0[e * 8 + 3]) * inv);
          w0.z = pack_bf16(__uint_as_float(o0[e * 8 + 4]) * inv, __uint_as_float(o0[e * 8 + 5]) * inv);
          w0.w = pack_bf16(__uint_as_float(o0[e * 8 + 6]) * inv, __uint_as_float(o0[e * 8 + 7]) * inv);
          dst[e] = w0;
          uint4 w1;
          w1.x = pack_bf16(__uint_as_float(o1[e * 8 + 0]) * inv, __uint_as_float(o1[e * 8 + 1]) * inv);
          w1.y = pack_bf16(__uint_as_float(o1[e * 8 + 2]) * inv, __uint_as_float(o1[e * 8 + 3]) * inv);
          w1.z = pack_bf16(__uint_as_float(o1[e * 8 + 4]) * inv, __uint_as_float(o1[e * 8 + 5]) * inv);
          w1.w = pack_bf16(__uint_as_float(o1[e * 8 + 6]) * inv, __uint_as_float(o1[e * 8 + 7]) * inv);
          dst[2 + e] = w1;
        }
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
