// clefq: the weight-resident 2-SM INT4 grouped GEMM for short K (at most three 256-code
// stages): the MoE expert down projection (K = intermediate = 768) and small-hidden expert
// gate|up launches.  Included by gemm.cu after gemm2sm.cuh, whose row stores it shares.
//
// With three K stages per tile the two-stage kernel converts a new weight tile into TMEM for
// every token tile, and each stage waits on the round trip commit -> converters -> TMEM
// stores -> leader -> issue (~1.4k cycles against 768 MMA cycles a stage).  Here a cluster
// walks a contiguous range of (pair tile, token tile) work in pair-tile-major order, so
// consecutive tiles usually share one expert's weights.  A run of tiles with the same
// (pair tile, expert) -- a unit -- converts its weights into TMEM once; every token tile of
// the unit reuses them:
//
//   * TMEM: accumulator columns [0, 192) and four 64-column weight slots.  A unit of k
//     stages takes k consecutive slots of the slot ring; with k <= 3 one slot is spare, so
//     the converters prepare the next unit's first stage while the current unit's last tile
//     runs, and its later stages as soon as the MMAs that read a slot complete (a per-slot
//     release barrier, committed after the unit's last tile reads the slot);
//   * SUBN = 192: one 192-token MMA tile per tile-list entry into one accumulator, which the
//     epilogue releases as soon as it is in registers.  SUBN = 96: two 96-token sub-tiles per
//     entry (a second one only if the entry has rows for it) into double-buffered
//     accumulators.  An MMA whose A operand is read from TMEM costs about as much at N = 96
//     as at N = 192, so the narrow form runs the tensor pipe at half rate or less;
//   * twelve epilogue warps (three per TMEM lane quarter) drain the accumulator, release
//     it, and store the BF16 rows through the route permutation.
//
// The producer tells the MMA issuer, per sub-tile, whether it opens a unit, closes a unit or
// is the cluster's last (a word per token slot, published by the slot's barrier), so the
// issuer's chain has no global loads.  Token loads use the .cta_group::2 form without
// multicast; every wait is bounded (mbar_wait_bounded) and every role gives up cleanly.
#pragma once

namespace two_sm_wres {

using two_sm::BMP;
using two_sm::BN2;
using two_sm::KS2;
using two_sm::RowDest;
using two_sm::fetch_row_dest;
using two_sm::store_tile_rows;

// SUBN tokens per sub-tile (MMA N): 192 (one sub-tile per tile-list entry, one accumulator)
// or 96 (two sub-tiles per entry, double-buffered accumulators).
template <int SUBN>
struct WresCfg {
  static_assert(SUBN == 96 || SUBN == 192, "sub-tile width");
  static constexpr int SH = SUBN / 2;                // token rows per CTA and sub-tile
  static constexpr int TOK_B = SH * KS2;             // token bytes per stage and CTA
  static constexpr int NT = SUBN == 96 ? 8 : 5;      // token slots
  static constexpr int NACC = SUBN == 96 ? 2 : 1;    // accumulators
  static constexpr int NSUB = BN2 / SUBN;            // sub-tiles per tile-list entry
  static constexpr int CH = SUBN / 96;               // 32-token chunks per epilogue warp
  static constexpr int EPI_ROWS = SUBN / 12;         // stored token rows per epilogue warp
  static constexpr uint32_t IDESC = idesc_i8(256, SUBN);
  static constexpr int W_OFF = NT * TOK_B;
  static constexpr int RING = NT * TOK_B + 2 * (128 * KS2 / 2);
  static constexpr int STAGING = SUBN * 128 * 2;     // BF16 [token][column]
  static constexpr int SMEM = RING + STAGING + 1024 + 1024;
  static_assert(TOK_B % 2048 == 0, "128-byte swizzle atoms of both K slices stay 1024-byte aligned");
  static_assert(SMEM <= 232448, "shared memory budget");
};
constexpr int NW = 2;                       // int4 weight slots in shared memory
constexpr int W_BYTES = 128 * KS2 / 2;      // 16 KiB: one 128-row x 32-word tile block
constexpr int NSLOT = 4;                    // TMEM weight slots, 64 columns each
constexpr int MAX_KST = NSLOT - 1;          // K stages of a unit (one slot stays spare)
constexpr int WCOL = 192;                   // weight slots after the accumulator columns [0, 192)
constexpr int TMEM_COLS = 512;
constexpr int TMA_W = 4, MMA_W = 5;
constexpr int EPI_W0 = 6;                   // first epilogue warp
constexpr int EPI_WARPS = 12;               // three per TMEM lane quarter
constexpr int THREADS = 32 * (EPI_W0 + EPI_WARPS);
static_assert(WCOL + 64 * NSLOT <= TMEM_COLS, "TMEM budget");

// sub-tile flags, one word per token slot (first K stage of the sub-tile)
constexpr uint32_t kOpens = 1, kCloses = 2, kFinal = 4;

template <int NT>
struct Smem {
  uint64_t tok_full[NT], tok_empty[NT], wsm_full[NW], wsm_empty[NW];
  uint64_t wtm_full[NSLOT], wfree[NSLOT], acc_full[2], acc_empty[2];
  uint32_t sink[4 + EPI_WARPS];  // targets of the follower's asynchronous 4-byte signals
  uint32_t info[NT];
  uint32_t tmem_base;
  int err;
};

// This cluster's work: tiles [begin, end) of the order t = np * n_mt + mt (pair tile np of
// the output columns, tile-list entry mt), split evenly over the clusters.
struct Walk {
  int64_t begin, end;
  int n_mt;
  CQ_DEV void tile(const GemmParams &p, int64_t t, int &np, int &expert, int64_t &row0, int &rows_valid) const {
    np = (int)(t / n_mt);
    const int mt = (int)(t - (int64_t)np * n_mt);
    expert = p.tile_list[1 + 2 * mt];
    row0 = p.tile_list[2 + 2 * mt];
    const int64_t e_end = p.expert_offsets[expert + 1];
    rows_valid = (int)(e_end - row0 < BN2 ? e_end - row0 : BN2);
  }
  CQ_DEV int64_t key(const GemmParams &p, int64_t t) const {
    const int64_t np = t / n_mt;
    return (np << 32) | (uint32_t)p.tile_list[1 + 2 * (t - np * n_mt)];
  }
};

template <int SUBN>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_i4_2sm_wres_kernel(const __grid_constant__ CUtensorMap tok_map, const __grid_constant__ CUtensorMap w_map0,
                            const __grid_constant__ CUtensorMap w_map1, GemmParams p) {
  using C = WresCfg<SUBN>;
  constexpr int SH = C::SH, TOK_B = C::TOK_B, NT = C::NT, NACC = C::NACC, W_OFF = C::W_OFF;
  constexpr int ACC_COLS = SUBN;
  // sub-tiles of a tile-list entry with rows_valid rows (a second 96-row half only if used)
  auto sub_tiles = [](int rows_valid) { return C::NSUB == 2 && rows_valid > SUBN ? 2 : 1; };
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t *ring = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  uint16_t *staging = reinterpret_cast<uint16_t *>(ring + C::RING);
  Smem<NT> &s = *reinterpret_cast<Smem<NT> *>(ring + C::RING + C::STAGING);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;

  // the tile list is the previous kernel's output
  pdl_wait();
  pdl_trigger();
  Walk wk;
  wk.n_mt = p.tile_list[0];
  const int n_pairs = p.n / BMP;
  const int64_t total = (int64_t)n_pairs * wk.n_mt;
  wk.begin = total * cluster / nclusters;
  wk.end = total * (cluster + 1) / nclusters;
  if (wk.begin >= wk.end) return;  // uniform across the pair
  const int k_stages = p.k / KS2;
  const int blocks_k = p.k / 256;  // int4: one 32-word block per K=256 slice

  if (threadIdx.x == 0) {
    for (int i = 0; i < NT; ++i) {
      mbar_init(&s.tok_full[i], 1);
      mbar_init(&s.tok_empty[i], 1);
    }
    for (int i = 0; i < NW; ++i) {
      mbar_init(&s.wsm_full[i], 1);
      mbar_init(&s.wsm_empty[i], 128);
    }
    // wtm_full / acc_empty (used on the leader): local warp arrivals, one of which also
    // expects the follower's 4-byte signals (st.async complete_tx)
    for (int i = 0; i < NSLOT; ++i) {
      mbar_init(&s.wtm_full[i], 4);
      mbar_init(&s.wfree[i], 1);
    }
    for (int i = 0; i < NACC; ++i) {
      mbar_init(&s.acc_full[i], 1);
      mbar_init(&s.acc_empty[i], EPI_WARPS);
    }
    s.err = 0;
    fence_barrier_init();
  }
  if (warp == MMA_W) {
    tmem_alloc2(&s.tmem_base, TMEM_COLS);
    tmem_relinquish2();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  // weight tile of this CTA for pair tile np: 128-row tile 2*np + rank
  auto weight_tile = [&](int np, int expert, int &which, int &w_row_tile) {
    const int nt = 2 * np + (int)rank;
    which = nt / p.n_split;
    w_row_tile = expert * p.n_split + (nt - which * p.n_split);
  };

  if (warp == TMA_W) {
    // ---- TMA producer (both CTAs) -------------------------------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&tok_map);
      tma_prefetch_desc(&w_map0);
      tma_prefetch_desc(&w_map1);
      uint32_t g = 0, w = 0;
      bool ok = true;
      int np, e, rv, nnp = 0, ne = 0, nrv = 0, pnp = -1, pe = -1;
      int64_t r0, nr0 = 0;
      wk.tile(p, wk.begin, np, e, r0, rv);
      for (int64_t t = wk.begin; ok && t < wk.end; ++t) {
        const bool has_next = t + 1 < wk.end;
        if (has_next) wk.tile(p, t + 1, nnp, ne, nr0, nrv);
        const bool opens = np != pnp || e != pe;
        const bool closes = !has_next || nnp != np || ne != e;
        if (opens) {
          int which, w_row_tile;
          weight_tile(np, e, which, w_row_tile);
          const CUtensorMap *w_map = which ? &w_map1 : &w_map0;
          for (int kb = 0; kb < k_stages; ++kb, ++w) {
            const int sw = w % NW;
            if (!(ok = mbar_wait_bounded(&s.wsm_empty[sw], ((w / NW) & 1) ^ 1, &s.err, 1))) break;
            mbar_arrive_expect_tx(&s.wsm_full[sw], W_BYTES);
            tma_load_3d(ring + W_OFF + sw * W_BYTES, w_map, &s.wsm_full[sw], 0, 0, w_row_tile * blocks_k + kb);
          }
        }
        const int nsub = sub_tiles(rv);
        for (int sb = 0; ok && sb < nsub; ++sb) {
          const uint32_t flags = (opens && sb == 0 ? kOpens : 0u) | (closes && sb == nsub - 1 ? kCloses : 0u) |
                                 (!has_next && sb == nsub - 1 ? kFinal : 0u);
          for (int kb = 0; kb < k_stages; ++kb, ++g) {
            const int st = g % NT;
            if (!(ok = mbar_wait_bounded(&s.tok_empty[st], ((g / NT) & 1) ^ 1, &s.err, 1))) break;
            if (rank == 0) {
              if (kb == 0) s.info[st] = flags;
              mbar_arrive_expect_tx(&s.tok_full[st], 2 * TOK_B);
            }
            // x = 128 bytes of a K slice, y = SH rows, z = the stage's two K slices
            tma_load_3d_cg2(ring + st * TOK_B, &tok_map, mapa_shared(smem_u32(&s.tok_full[st]), 0), 0,
                            (int)(r0 + SUBN * sb + SH * (int)rank), 2 * kb);
          }
        }
        pnp = np; pe = e;
        np = nnp; e = ne; r0 = nr0; rv = nrv;
      }
    }
  } else if (warp == MMA_W) {
    // ---- MMA issuer (pair leader only) ---------------------------------------------------
    if (lane == 0 && rank == 0) {
      uint32_t g = 0, unit_w0 = 0;
      int j = 0, units = 0;
      bool ok = true, fin = false;
      while (ok && !fin) {
        const int buf = NACC == 2 ? (j & 1) : 0;
        const uint32_t use = NACC == 2 ? (uint32_t)(j >> 1) : (uint32_t)j;  // earlier uses of the buffer
        if (!(ok = mbar_wait_bounded(&s.acc_empty[buf], (use & 1) ^ 1, &s.err, 7))) break;
        tc_fence_after();
        const uint32_t acc = tmem + ACC_COLS * buf;
        uint32_t flags = 0;
        for (int kb = 0; kb < k_stages; ++kb, ++g) {
          const int st = g % NT;
          if (!(ok = mbar_wait_bounded(&s.tok_full[st], (g / NT) & 1, &s.err, 2))) break;
          if (kb == 0) {
            flags = s.info[st];
            if (flags & kOpens) unit_w0 = (uint32_t)(units++) * (uint32_t)k_stages;
          }
          const uint32_t wst = unit_w0 + kb;
          const int sl = wst % NSLOT;
          if ((flags & kOpens) && !(ok = mbar_wait_bounded(&s.wtm_full[sl], (wst / NSLOT) & 1, &s.err, 3))) break;
          tc_fence_after();
          const uint32_t b_base = smem_u32(ring + st * TOK_B);
#pragma unroll
          for (int jj = 0; jj < KS2 / 32; ++jj) {
            const uint32_t a_col = tmem + WCOL + 64 * sl + 8 * jj;
            const uint32_t b_off = (jj >> 2) * (TOK_B / 2) + 32 * (jj & 3);
            mma_i8_ts2(acc, a_col, smem_desc_sw128(b_base + b_off), C::IDESC, (kb | jj) != 0);
          }
          mma_commit2_mc(&s.tok_empty[st], 3);
          if (flags & kCloses) mma_commit2_mc(&s.wfree[sl], 3);  // the unit's last reader of the slot
        }
        if (!ok) break;
        mma_commit2_mc(&s.acc_full[buf], 3);
        fin = (flags & kFinal) != 0;
        ++j;
      }
      if (j > 0) {
        const int last = NACC == 2 ? ((j - 1) & 1) : 0;
        const uint32_t use = NACC == 2 ? (uint32_t)((j - 1) >> 1) : (uint32_t)(j - 1);
        mbar_wait_bounded(&s.acc_full[last], use & 1, &s.err, 6);
      }
    }
  } else if (warp < 4) {
    // ---- weight converters (both CTAs) -> own TMEM; slot-ready counted on the leader -----
    const int r = warp * 32 + lane;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const uint32_t lead_wtm_full = mapa_shared(smem_u32(&s.wtm_full[0]), 0);
    const uint32_t lead_sink = mapa_shared(smem_u32(&s.sink[warp]), 0);
    // units of this cluster's range: positions whose (pair tile, expert) differs from the
    // previous position's
    int units = 0;
    for (int64_t t0 = wk.begin; t0 < wk.end; t0 += 32) {
      const int64_t t = t0 + lane;
      const bool opens = t < wk.end && (t == wk.begin || wk.key(p, t) != wk.key(p, t - 1));
      units += __popc(__ballot_sync(0xffffffffu, opens));
    }
    const uint32_t n_w = (uint32_t)units * (uint32_t)k_stages;
    bool ok = true;
    for (uint32_t w = 0; ok && w < n_w; ++w) {
      const int st = w % NW;
      const int sl = w % NSLOT;
      bool waited = true;
      if (lane == 0) waited = mbar_wait_bounded(&s.wsm_full[st], (w / NW) & 1, &s.err, 4);
      waited = __shfl_sync(0xffffffffu, waited, 0) != 0;
      if (!(ok = waited)) break;
      const uint32_t wbase = smem_u32(ring + W_OFF + st * W_BYTES);
      // 128-byte rows, 128-byte swizzle: 16-byte chunk c of row r sits at chunk c ^ (r & 7)
      uint32_t wv[32];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 v = lds_v4(wbase + r * 128 + 16 * (c ^ (r & 7)));
        wv[4 * c] = v.x; wv[4 * c + 1] = v.y; wv[4 * c + 2] = v.z; wv[4 * c + 3] = v.w;
      }
      mbar_arrive(&s.wsm_empty[st]);
      // the weights are in registers: wait until the MMAs that read slot sl for the unit
      // before last have completed (its release commit)
      if (lane == 0 && w >= NSLOT) waited = mbar_wait_bounded(&s.wfree[sl], ((w / NSLOT) & 1) ^ 1, &s.err, 4);
      waited = __shfl_sync(0xffffffffu, waited, 0) != 0;
      if (!(ok = waited)) break;
      tc_fence_after();
      // 8 words per 32-code group -> low nibbles then high nibbles (x16)
      uint32_t o[2][32];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int gq = 0; gq < 4; ++gq) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            o[h][8 * gq + q] = nib_lo16(wv[16 * h + 4 * gq + q]);
            o[h][8 * gq + 4 + q] = nib_hi16(wv[16 * h + 4 * gq + q]);
          }
        }
        tmem_st_x32(tmem + lane_base + WCOL + 64 * sl + 32 * h, o[h]);
      }
      tmem_st_wait(o[0]);
      tmem_st_keep(o[1]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0) {
          if (warp == 0) mbar_arrive_expect_tx(&s.wtm_full[sl], 16);
          else mbar_arrive(&s.wtm_full[sl]);
        } else {
          st_async_signal(lead_sink, lead_wtm_full + 8 * sl);
        }
      }
    }
  } else if (warp >= EPI_W0) {
    // ---- epilogue (both CTAs): this CTA's 128 weight rows x SUBN tokens per sub-tile ----
    // Warp e covers TMEM lane quarter (warp & 3) and tokens [TPW*part, TPW*part + TPW).
    constexpr int CH = C::CH, EPI_ROWS = C::EPI_ROWS, TPW = 32 * CH;
    const int quarter = warp & 3;
    const int eidx = warp - EPI_W0;
    const int part = eidx >> 2;
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const uint32_t lead_acc_empty = mapa_shared(smem_u32(&s.acc_empty[0]), 0);
    const uint32_t lead_sink = mapa_shared(smem_u32(&s.sink[4 + eidx]), 0);
    const int m0 = eidx * EPI_ROWS;  // rows this warp stores
    int j = 0;
    bool go = true;
    for (int64_t t = wk.begin; go && t < wk.end; ++t) {
      int np, expert, rv;
      int64_t row0;
      wk.tile(p, t, np, expert, row0, rv);
      int which, w_row_tile;
      weight_tile(np, expert, which, w_row_tile);
      const float ws = p.w_scales[which][(int64_t)w_row_tile * 128 + r];
      const int col0 = (2 * np + (int)rank) * 128;  // first output column of this CTA
      const int nsub = sub_tiles(rv);
      for (int sb = 0; sb < nsub; ++sb, ++j) {
        const int64_t srow0 = row0 + SUBN * sb;
        const int svalid = rv - SUBN * sb;  // may be <= 0: nothing of the sub-tile is stored
        // activation scales of this warp's tokens, and the output rows of its stores,
        // fetched before the accumulator is ready
        float my_scale[CH];
#pragma unroll
        for (int q = 0; q < CH; ++q) {
          my_scale[q] = 0.0f;
          const int mj = TPW * part + 32 * q + lane;
          if (mj < svalid) {
            const int64_t pos = srow0 + mj;
            const int64_t route = p.perm[pos];
            my_scale[q] = p.a_scales[p.scale_mode == 0 ? pos : (p.scale_mode == 1 ? route / p.topk : route)];
          }
        }
        const RowDest dest = fetch_row_dest<true>(p, srow0, svalid, m0, m0 + EPI_ROWS, lane);
        const int buf = NACC == 2 ? (j & 1) : 0;
        const uint32_t use = NACC == 2 ? (uint32_t)(j >> 1) : (uint32_t)j;
        bool have = true;
        if (lane == 0) have = mbar_wait_bounded(&s.acc_full[buf], use & 1, &s.err, 5);
        have = __shfl_sync(0xffffffffu, have, 0) != 0;
        if (!named_barrier_and(2, 32 * EPI_WARPS, have)) {
          go = false;
          break;
        }
        tc_fence_after();
        uint32_t accv[CH][32];
#pragma unroll
        for (int q = 0; q < CH; ++q) tmem_ld_x32(tmem + lane_base + ACC_COLS * buf + TPW * part + 32 * q, accv[q]);
        tmem_ld_wait(accv[0]);
#pragma unroll
        for (int q = 1; q < CH; ++q) tmem_ld_tie(accv[q]);
        // the slice is in registers: release the accumulator
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (rank == 0) {
            if (eidx == 0) mbar_arrive_expect_tx(&s.acc_empty[buf], 4 * EPI_WARPS);
            else mbar_arrive(&s.acc_empty[buf]);
          } else {
            st_async_signal(lead_sink, lead_acc_empty + 8 * buf);
          }
        }
#pragma unroll
        for (int q = 0; q < CH; ++q) {
#pragma unroll
          for (int jj = 0; jj < 32; jj += 2) {
            float y[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const float as = __shfl_sync(0xffffffffu, my_scale[q], jj + u);
              const float a = __int2float_rn((int)accv[q][jj + u] >> 8);
              y[u] = __fmul_rn(a, __fmul_rn(as, ws));
            }
            // two tokens rounded to BF16 (nearest even) by one cvt.rn.bf16x2; a NaN stays a NaN
            uint32_t h2;
            asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(h2) : "f"(y[1]), "f"(y[0]));
            const int c = TPW * part + 32 * q + jj;
            staging[c * 128 + r] = (uint16_t)h2;
            staging[(c + 1) * 128 + r] = (uint16_t)(h2 >> 16);
          }
        }
        named_barrier_sync(1, 32 * EPI_WARPS);
        if (p.store16)
          store_tile_rows<true, 8>(p, staging, srow0, svalid, col0, m0, m0 + EPI_ROWS, lane, dest);
        else
          store_tile_rows<true, 4>(p, staging, srow0, svalid, col0, m0, m0 + EPI_ROWS, lane, dest);
        named_barrier_sync(1, 32 * EPI_WARPS);
      }
    }
  }
  tc_fence_before();
  cluster_sync();  // no CTA leaves while its peer may still signal it
  if (warp == MMA_W) {
    tc_fence_after();
    tmem_dealloc2(tmem, TMEM_COLS);
  }
  if (threadIdx.x == 0 && s.err) atomicCAS(p.err, 0, s.err);
}

}  // namespace two_sm_wres
