// clefq: the 2-SM (cta_group::2) INT4/INT8 GEMM used when every weight matrix has a
// multiple of 256 output rows.  Included by gemm.cu (shares its helpers and epilogue
// arithmetic).
//
// A CTA pair (cluster of 2) computes one 256-weight-row x 192-token tile:
//   * each CTA converts its own 128 weight rows into its TMEM (the MMA's A operand),
//   * each CTA TMA-loads its own 96 token rows (the B operand is split along N between the
//     pair's shared memory); the loads use the .cta_group::2 form so that both halves count
//     on the leader's barrier -- plain loads, no multicast,
//   * the leader issues tcgen05.mma.cta_group::2 (M=256, N=192, K=32) and multicasts one
//     completion (tcgen05.commit) per K stage to both CTAs: it frees the stage's token slot
//     and tells the converters that the TMEM weight stage of two K stages back is free,
//   * both CTAs drain their 128-row slice of the accumulator; accumulators are double
//     buffered (2 x 192 TMEM columns) so a tile's epilogue overlaps the next mainloop.
// Per SM this moves 40 KB of operands per 768 MMA cycles (~53 B/clk), under the ~67 B/clk
// the L2 delivers to one SM, where the 128 x 128 one-CTA tile needs ~96 B/clk.  Each
// K=256 stage is exactly two TMA boxes (a 24 KB 3D token box holding two 128-byte K
// slices, and one contiguous 16 KB weight block): an SM's TMA unit completes about one
// box per ~250 cycles whatever its size up to 16 KB, so small boxes cap the feed rate.
#pragma once

namespace two_sm {

constexpr int BMP = 256;                       // weight rows per pair tile (128 per CTA)
constexpr int BN2 = 192;                       // tokens per pair tile (96 per CTA)
constexpr int HALF = 96;                       // token rows held by one CTA
constexpr int KS2 = 256;                       // codes per stage
constexpr int TOK_B = HALF * KS2;              // 24 KiB: two 12 KiB K-slices of 96 rows
constexpr int NSW = 2;                         // TMEM weight stages (64 columns each)
constexpr int ACC_COLS = 192;
constexpr int WCOL = 2 * ACC_COLS;             // 384: weight stages after both accumulators
constexpr int TMEM2_COLS = 512;
constexpr int THREADS2 = 448;                  // 4 converter, 1 TMA, 1 MMA, 8 epilogue warps
constexpr int EPI_WARPS = 8;                   // two per TMEM lane quarter, 96 tokens each
constexpr int TMA_W = 4, MMA_W = 5;
constexpr uint32_t IDESC2 = idesc_i8(256, BN2);
constexpr int STAGING2 = BN2 * 128 * 2;        // 48 KiB BF16 [token][column]

// Separate rings for the two operands.  Token slots are held until the MMAs that read
// them complete, so their ring must cover the TMA latency (~3k cycles under load) plus a
// stage: 5 slots.  Weight slots are copied into registers by the converters as soon as
// they land (before waiting for a free TMEM stage), so 3 slots keep them ahead.
//
// SUB = 2 (dense int4 only): a pair tile spans two 192-token sub-tiles that share every
// converted weight stage -- per K step the leader issues one MMA into each sub-tile's
// accumulator, twice the tensor work per pass of the converter -> MMA -> commit chain.  The
// two accumulators then fill the TMEM columns that SUB = 1 uses for double buffering, so the
// epilogue of a tile no longer overlaps the next tile's mainloop; token stages hold both
// sub-tiles (48 KiB), 3 of them, and 2 weight slots, to fit shared memory.
template <int BITS, int SUB = 1>
struct Cfg2 {
  static constexpr int TOK_STAGE = SUB * TOK_B;           // token bytes per stage and CTA
  static constexpr int NT = SUB == 2 ? 3 : (BITS == 4 ? 5 : 4);   // token stages
  static constexpr int NW = SUB == 2 ? 2 : (BITS == 4 ? 3 : 2);   // weight stages
  static constexpr int W_BYTES = 128 * KS2 * BITS / 8;
  static constexpr int W_OFF = NT * TOK_STAGE;            // weight ring after the token ring
  static constexpr int RING = NT * TOK_STAGE + NW * W_BYTES;
  static constexpr int SMEM = RING + STAGING2 + 1024 + 1024;
};

template <int NT, int NW>
struct Smem2 {
  uint64_t tok_full[NT], tok_empty[NT], wsm_full[NW], wsm_empty[NW];
  uint64_t wtm_full[NSW], acc_full[2], acc_empty[2];
  uint32_t sink[4 + EPI_WARPS];  // targets of the follower's asynchronous 4-byte signals
  uint32_t tmem_base;
  int err;
};

struct TileMap2 {
  int n_pairs, total;
  int span;  // token rows per pair tile: SUB x BN2 (dense two-stage), BN2 (grouped), or the deep kernel's tile
  CQ_DEV bool get(const GemmParams &p, int t, int64_t &row0, int &rows_valid, int &np, int &expert) const {
    if (t >= total) return false;
    const int mt = t / n_pairs;
    np = t - mt * n_pairs;
    if (p.grouped) {
      expert = p.tile_list[1 + 2 * mt];
      row0 = p.tile_list[2 + 2 * mt];
      const int64_t end = p.expert_offsets[expert + 1];
      rows_valid = (int)(end - row0 < span ? end - row0 : span);
    } else {
      expert = 0;
      row0 = (int64_t)mt * span;
      rows_valid = (int)(p.m - row0 < span ? p.m - row0 : span);
    }
    return true;
  }
};

template <int V> struct StoreVec;
template <> struct StoreVec<4> { using T = uint2; };
template <> struct StoreVec<8> { using T = uint4; };

// Where the rows a warp stores go (grouped mode), read before the tile's accumulator is
// ready so the loads overlap the mainloop instead of sitting in front of every row store:
// lane l holds row m_begin + l's output row (perm).
struct RowDest {
  int orow = 0;
};

template <bool GROUPED>
CQ_DEV RowDest fetch_row_dest(const GemmParams &p, int64_t row0, int rows_valid, int m_begin, int m_end, int lane) {
  RowDest d;
  const int m = m_begin + lane;
  if (GROUPED && m < m_end && m < rows_valid) {
    const int64_t pos = row0 + m;
    d.orow = p.scatter ? p.perm[pos] : (int)pos;
  }
  return d;
}

// Stores token rows [m_begin, m_end) (at most 32) of a CTA's staged BF16 tile (128 columns
// from col0): V columns per lane, so 128 / V lanes per row (V = 8: 16-byte stores, two rows
// per warp instruction).  Dense: optional residual bf16(res + y), and copies to out_peer.
// Grouped: row scatter through perm, with the destinations taken from dest (fetch_row_dest).
template <bool GROUPED, int V>
CQ_DEV void store_tile_rows(const GemmParams &p, const uint16_t *staging, int64_t row0, int rows_valid, int col0,
                            int m_begin, int m_end, int lane, const RowDest &dest) {
  using Vec = typename StoreVec<V>::T;
  constexpr int LPR = 128 / V;  // lanes per row
  constexpr int RPI = 32 / LPR;  // rows per warp iteration
  const int sub = lane / LPR, l = lane % LPR;
  const int iters = (m_end - m_begin + RPI - 1) / RPI;  // the same on every lane
  for (int it = 0; it < iters; ++it) {
    const int mi = it * RPI + sub;  // row within [m_begin, m_end)
    const int m = m_begin + mi;
    int64_t orow = row0 + m;
    // the shuffle runs on every lane (mi < 32), before the row checks
    if (GROUPED) orow = __shfl_sync(0xffffffffu, dest.orow, mi & 31);
    if (m >= m_end || m >= rows_valid) continue;
    const int64_t pos = row0 + m;
    Vec v = *reinterpret_cast<const Vec *>(staging + m * 128 + V * l);
    uint16_t *hv = reinterpret_cast<uint16_t *>(&v);
    if (!GROUPED && p.residual) {
      const Vec rv = *reinterpret_cast<const Vec *>(p.residual + pos * p.ldr + col0 + V * l);
      const uint16_t *hr = reinterpret_cast<const uint16_t *>(&rv);
#pragma unroll
      for (int q = 0; q < V; ++q) hv[q] = f32_to_bf16(__fadd_rn(bf16_to_f32(hr[q]), bf16_to_f32(hv[q])));
    }
    const int64_t off = orow * p.ldo + col0 + V * l;
    *reinterpret_cast<Vec *>(p.out + off) = v;
    if (!GROUPED && p.n_out_peer) {
#pragma unroll
      for (int d = 0; d < kMaxPeers; ++d)
        if (d < p.n_out_peer) *reinterpret_cast<Vec *>(p.out_peer[d] + off) = v;
    }
  }
}

template <bool GROUPED, int BITS, int SUB = 1>
__global__ void __launch_bounds__(THREADS2, 1)
    gemm_i8_2sm_kernel(const __grid_constant__ CUtensorMap tok_map, const __grid_constant__ CUtensorMap w_map0,
                       const __grid_constant__ CUtensorMap w_map1, GemmParams p) {
  static_assert(SUB == 1 || (SUB == 2 && !GROUPED && BITS == 4), "two sub-tiles: dense int4 only");
  using C = Cfg2<BITS, SUB>;
  constexpr int NT = C::NT, NW = C::NW;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t *ring = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  uint16_t *staging = reinterpret_cast<uint16_t *>(ring + C::RING);
  Smem2<NT, NW> &s = *reinterpret_cast<Smem2<NT, NW> *>(ring + C::RING + STAGING2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;

  // grouped: the tile list is the previous kernel's output
  if (GROUPED) {
    pdl_wait();
    pdl_trigger();
  }
  TileMap2 tm;
  tm.n_pairs = p.n / BMP;
  tm.span = SUB * BN2;
  tm.total = (GROUPED ? p.tile_list[0] : (int)((p.m + tm.span - 1) / tm.span)) * tm.n_pairs;
  if (cluster >= tm.total) return;  // uniform across the pair
  const int k_stages = p.k / KS2;
  const int blocks_k = p.k / (32 * (32 / BITS));

  if (threadIdx.x == 0) {
    for (int i = 0; i < NT; ++i) {
      mbar_init(&s.tok_full[i], 1);
      mbar_init(&s.tok_empty[i], 1);
    }
    for (int i = 0; i < NW; ++i) {
      mbar_init(&s.wsm_full[i], 1);
      mbar_init(&s.wsm_empty[i], 128);
    }
    // wtm_full / acc_empty (used on the leader): 4 local warp arrivals, one of which
    // also expects the follower's 4 x 4 signal bytes (st.async complete_tx).
    for (int i = 0; i < NSW; ++i) mbar_init(&s.wtm_full[i], 4);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.acc_full[i], 1);
      mbar_init(&s.acc_empty[i], EPI_WARPS);
    }
    s.err = 0;
    fence_barrier_init();
  }
  if (warp == MMA_W) {
    tmem_alloc2(&s.tmem_base, TMEM2_COLS);
    tmem_relinquish2();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  // dense: the prologue above touches no global memory; tokens, scales, residual and
  // output wait for the previous kernel
  if (!GROUPED) {
    pdl_wait();
    pdl_trigger();
  }

  // Output/weight tile of this CTA for pair tile np: 128-row tile 2*np + rank.
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
      uint32_t g = 0;
      bool ok = true;
      int64_t row0;
      int rows_valid, np, expert;
      for (int t = cluster; ok && tm.get(p, t, row0, rows_valid, np, expert); t += nclusters) {
        int which, w_row_tile;
        weight_tile(np, expert, which, w_row_tile);
        const CUtensorMap *w_map = which ? &w_map1 : &w_map0;
        // Integer accumulation is exact in any order, so each pair tile starts its K sweep
        // at its own offset: pairs sharing a token tile then read different K slices at the
        // same moment instead of hammering the same L2 lines.
        const int k_off = (int)((7u * (uint32_t)t) % (uint32_t)k_stages);
        for (int kk = 0; kk < k_stages; ++kk, ++g) {
          const int kb = kk + k_off < k_stages ? kk + k_off : kk + k_off - k_stages;
          const int sw = g % NW, st = g % NT;
          // weight box first (its slot frees as soon as the converters have read it):
          // whole 128-row x 32-word tiled block(s) of this K=256 slice
          if (!(ok = mbar_wait_bounded(&s.wsm_empty[sw], ((g / NW) & 1) ^ 1, &s.err, 1))) break;
          mbar_arrive_expect_tx(&s.wsm_full[sw], C::W_BYTES);
          tma_load_3d(ring + C::W_OFF + sw * C::W_BYTES, w_map, &s.wsm_full[sw], 0, 0,
                      w_row_tile * blocks_k + kb * (BITS == 4 ? 1 : 2));
          // token box: x = 128 bytes of a K slice, y = 96 rows, z = the stage's two K slices
          if (!(ok = mbar_wait_bounded(&s.tok_empty[st], ((g / NT) & 1) ^ 1, &s.err, 1))) break;
          if (rank == 0) mbar_arrive_expect_tx(&s.tok_full[st], SUB * 2 * TOK_B);
#pragma unroll
          for (int sb = 0; sb < SUB; ++sb)
            tma_load_3d_cg2(ring + st * C::TOK_STAGE + sb * TOK_B, &tok_map,
                            mapa_shared(smem_u32(&s.tok_full[st]), 0), 0, (int)(row0 + sb * BN2 + HALF * rank),
                            2 * kb);
        }
      }
    }
  } else if (warp == MMA_W) {
    // ---- MMA issuer (pair leader only) ---------------------------------------------------
    if (lane == 0 && rank == 0) {
      uint32_t g = 0;
      int i = 0;
      bool ok = true;
      // the issuer needs only the tile count: no tile-list loads on its chain
      for (int t = cluster; ok && t < tm.total; t += nclusters, ++i) {
        // SUB = 1: accumulator buffer i & 1 (double buffered); SUB = 2: both buffers, one
        // per sub-tile, released together by the epilogue
        const int buf = SUB == 1 ? (i & 1) : 0;
        const uint32_t par = SUB == 1 ? (((i >> 1) & 1) ^ 1) : ((i & 1) ^ 1);
        if (!(ok = mbar_wait_bounded(&s.acc_empty[buf], par, &s.err, 7))) break;
        tc_fence_after();
        const uint32_t acc = tmem + ACC_COLS * buf;
        for (int kb = 0; kb < k_stages; ++kb, ++g) {
          const int st = g % NT;
          const int sw = g % NSW;
          if (!(ok = mbar_wait_bounded(&s.tok_full[st], (g / NT) & 1, &s.err, 2) &&
                     mbar_wait_bounded(&s.wtm_full[sw], (g / NSW) & 1, &s.err, 3)))
            break;
          tc_fence_after();
          const uint32_t b_base = smem_u32(ring + st * C::TOK_STAGE);
#pragma unroll
          for (int j = 0; j < KS2 / 32; ++j) {
            const uint32_t a_col = tmem + WCOL + 64 * sw + 8 * j;
            const uint32_t b_off = (j >> 2) * (TOK_B / 2) + 32 * (j & 3);
#pragma unroll
            for (int sb = 0; sb < SUB; ++sb)
              mma_i8_ts2(acc + ACC_COLS * sb, a_col, smem_desc_sw128(b_base + sb * TOK_B + b_off), IDESC2,
                         (kb | j) != 0);
          }
          mma_commit2_mc(&s.tok_empty[st], 3);
        }
        mma_commit2_mc(&s.acc_full[buf], 3);
      }
      if (i > 0) {
        const int last = SUB == 1 ? ((i - 1) & 1) : 0;
        const uint32_t par = SUB == 1 ? (((i - 1) >> 1) & 1) : ((i - 1) & 1);
        mbar_wait_bounded(&s.acc_full[last], par, &s.err, 6);
      }
    }
  } else if (warp < 4) {
    // ---- weight converters (both CTAs) -> own TMEM; stage-ready counted on the leader ----
    const int r = warp * 32 + lane;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const uint32_t lead_wtm_full = mapa_shared(smem_u32(&s.wtm_full[0]), 0);
    const uint32_t lead_sink = mapa_shared(smem_u32(&s.sink[warp]), 0);
    uint32_t g = 0;
    bool ok = true;
    // the converters convert whatever weight block the producer loaded: the tile count is
    // all they need (no tile-list loads on the per-stage chain)
    for (int t = cluster; ok && t < tm.total; t += nclusters) {
      for (int kb = 0; kb < k_stages; ++kb, ++g) {
        const int st = g % NW;
        const int sw = g % NSW;
        bool waited = true;
        if (lane == 0) waited = mbar_wait_bounded(&s.wsm_full[st], (g / NW) & 1, &s.err, 4);
        waited = __shfl_sync(0xffffffffu, waited, 0) != 0;
        if (!(ok = waited)) break;
        const uint32_t wbase = smem_u32(ring + C::W_OFF + st * C::W_BYTES);
        // 128-byte rows, 128-byte swizzle: 16-byte chunk c of row r sits at chunk c ^ (r & 7)
        uint32_t w[32];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 v = lds_v4(wbase + r * 128 + 16 * (c ^ (r & 7)));
          w[4 * c] = v.x; w[4 * c + 1] = v.y; w[4 * c + 2] = v.z; w[4 * c + 3] = v.w;
        }
        uint32_t w2[32];
        if (BITS == 8) {
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint4 v = lds_v4(wbase + 16384 + r * 128 + 16 * (c ^ (r & 7)));
            w2[4 * c] = v.x; w2[4 * c + 1] = v.y; w2[4 * c + 2] = v.z; w2[4 * c + 3] = v.w;
          }
        }
        mbar_arrive(&s.wsm_empty[st]);
        // the weights are in registers: now wait for the TMEM stage the MMA last read, i.e.
        // for the MMAs of stage g - NSW, whose completion the token ring's commit reports
        if (lane == 0 && g >= NSW) {
          const uint32_t gp = g - NSW;
          waited = mbar_wait_bounded(&s.tok_empty[gp % NT], (gp / NT) & 1, &s.err, 4);
        }
        waited = __shfl_sync(0xffffffffu, waited, 0) != 0;
        if (!(ok = waited)) break;
        tc_fence_after();
        if (BITS == 4) {
          // 8 words per 32-code group -> low nibbles then high nibbles (x16)
          uint32_t o[2][32];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int gq = 0; gq < 4; ++gq) {
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                o[h][8 * gq + q] = nib_lo16(w[16 * h + 4 * gq + q]);
                o[h][8 * gq + 4 + q] = nib_hi16(w[16 * h + 4 * gq + q]);
              }
            }
            tmem_st_x32(tmem + lane_base + WCOL + 64 * sw + 32 * h, o[h]);
          }
          tmem_st_wait(o[0]);
          tmem_st_keep(o[1]);
        } else {
          tmem_st_x32(tmem + lane_base + WCOL + 64 * sw, w);
          tmem_st_x32(tmem + lane_base + WCOL + 64 * sw + 32, w2);
          tmem_st_wait(w);
          tmem_st_keep(w2);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (rank == 0) {
            if (warp == 0) mbar_arrive_expect_tx(&s.wtm_full[sw], 16);
            else mbar_arrive(&s.wtm_full[sw]);
          } else {
            st_async_signal(lead_sink, lead_wtm_full + 8 * sw);
          }
        }
      }
    }
  } else {
    // ---- epilogue (warps 6-13, both CTAs): this CTA's 128 weight rows x 192 tokens ------
    // Warp e covers TMEM lane quarter (warp & 3) and tokens [96*half, 96*half + 96).
    // Activation scales (and routes) of the next tile are fetched before its accumulator
    // is ready, so their global-load latency overlaps the mainloop.
    const int quarter = warp & 3;
    const int ehalf = (warp - 6) >> 2;
    const int eidx = warp - 6;
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const uint32_t lead_acc_empty = mapa_shared(smem_u32(&s.acc_empty[0]), 0);
    const uint32_t lead_sink = mapa_shared(smem_u32(&s.sink[4 + eidx]), 0);
    const int shift = BITS == 4 ? 8 : 0;
    const float big = 3.3895313892515355e38f;
    constexpr int CH = (BN2 / 2) / 32;  // 32-token chunks per warp
    int i = 0;
    int64_t row0;
    int rows_valid, np, expert;
    for (int t = cluster; tm.get(p, t, row0, rows_valid, np, expert); t += nclusters, ++i) {
      // SUB = 1: this tile's accumulator is buffer i & 1; SUB = 2: sub-tile sb is buffer sb
      float my_scale[SUB][CH];
#pragma unroll
      for (int sb = 0; sb < SUB; ++sb) {
#pragma unroll
        for (int q = 0; q < CH; ++q) {
          const int mj = sb * BN2 + ehalf * (BN2 / 2) + 32 * q + lane;
          my_scale[sb][q] = 0.0f;
          if (mj < rows_valid) {
            const int64_t pos = row0 + mj;
            if (GROUPED) {
              const int64_t route = p.perm[pos];
              my_scale[sb][q] = p.a_scales[p.scale_mode == 0 ? pos : (p.scale_mode == 1 ? route / p.topk : route)];
            } else {
              my_scale[sb][q] = p.a_scales[pos];
            }
          }
        }
      }
      // each warp stores 24 token rows of every sub-tile, 256 contiguous bytes per row
      const int m0 = eidx * (BN2 / EPI_WARPS);
      const RowDest dest = fetch_row_dest<GROUPED>(p, row0, rows_valid, m0, m0 + BN2 / EPI_WARPS, lane);
      int which, w_row_tile;
      weight_tile(np, expert, which, w_row_tile);
      const float ws = p.w_scales[which][(int64_t)w_row_tile * 128 + r];
      const int col0 = (2 * np + (int)rank) * 128;  // first output column of this CTA
      const int done_buf = SUB == 1 ? (i & 1) : 0;  // the barrier pair of this tile
      bool have = true;
      if (lane == 0)
        have = mbar_wait_bounded(&s.acc_full[done_buf], SUB == 1 ? ((i >> 1) & 1) : (i & 1), &s.err, 5);
      have = __shfl_sync(0xffffffffu, have, 0) != 0;
      if (!named_barrier_and(2, 32 * EPI_WARPS, have)) break;
      tc_fence_after();
#pragma unroll
      for (int sb = 0; sb < SUB; ++sb) {
        const int buf = SUB == 1 ? (i & 1) : sb;
        const int64_t srow0 = row0 + sb * BN2;
        const int svalid = rows_valid - sb * BN2;  // may be <= 0: nothing of the sub-tile is stored
#pragma unroll
        for (int q = 0; q < CH; ++q) {
          const int c = ehalf * (BN2 / 2) + 32 * q;
          uint32_t accv[32];
          tmem_ld_x32(tmem + lane_base + ACC_COLS * buf + c, accv);
          tmem_ld_wait(accv);
          if (q == CH - 1 && sb == SUB - 1) {
            // every accumulator column of the tile is in registers: release the buffer(s)
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
              if (rank == 0) {
                if (eidx == 0) mbar_arrive_expect_tx(&s.acc_empty[done_buf], 4 * EPI_WARPS);
                else mbar_arrive(&s.acc_empty[done_buf]);
              } else {
                st_async_signal(lead_sink, lead_acc_empty + 8 * done_buf);
              }
            }
          }
          if (!GROUPED && p.out_f32) {
            // F32 output: the reference's epilogue value, stored as it is computed
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float as = __shfl_sync(0xffffffffu, my_scale[sb][q], j);
              const float a = __int2float_rn((int)accv[j] >> shift);
              const float y = __fadd_rn(__fmul_rn(__fmul_rn(a, ws), as), 0.0f);
              if (c + j < svalid) p.out_f32[(srow0 + c + j) * p.ldo + col0 + r] = y;
            }
            continue;
          }
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            float y[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const float as = __shfl_sync(0xffffffffu, my_scale[sb][q], j + u);
              const float a = __int2float_rn((int)accv[j + u] >> shift);
              if (GROUPED) {
                y[u] = __fmul_rn(a, __fmul_rn(as, ws));
              } else {
                // finite values saturate to the largest finite BF16; infinities and NaN pass
                const float v = __fadd_rn(__fmul_rn(__fmul_rn(a, ws), as), 0.0f);
                y[u] = fabsf(v) < __int_as_float(0x7f800000) ? maxnum(minnum(v, big), -big) : v;
              }
            }
            // two tokens rounded to BF16 (nearest even) by one cvt.rn.bf16x2; a NaN stays a NaN
            uint32_t h2;
            asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(h2) : "f"(y[1]), "f"(y[0]));
            staging[(c + j) * 128 + r] = (uint16_t)h2;
            staging[(c + j + 1) * 128 + r] = (uint16_t)(h2 >> 16);
          }
        }
        if (GROUPED || !p.out_f32) {
          named_barrier_sync(1, 32 * EPI_WARPS);
          if (p.store16)
            store_tile_rows<GROUPED, 8>(p, staging, srow0, svalid, col0, m0, m0 + BN2 / EPI_WARPS, lane, dest);
          else
            store_tile_rows<GROUPED, 4>(p, staging, srow0, svalid, col0, m0, m0 + BN2 / EPI_WARPS, lane, dest);
          named_barrier_sync(1, 32 * EPI_WARPS);
        }
      }
    }
  }
  // stores into other GPUs' buffers (tensor-parallel output copies) are made visible at
  // system scope by each storing thread before the kernel ends
  if (!GROUPED && p.n_out_peer) __threadfence_system();
  tc_fence_before();
  cluster_sync();  // no CTA leaves while its peer may still signal it
  if (warp == MMA_W) {
    tc_fence_after();
    tmem_dealloc2(tmem, TMEM2_COLS);
  }
  if (threadIdx.x == 0 && s.err) atomicCAS(p.err, 0, s.err);
}

}  // namespace two_sm
