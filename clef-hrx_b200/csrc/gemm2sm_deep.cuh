// clefq: the deep-ring 2-SM (cta_group::2) INT4 GEMM, used for every int4 launch whose
// weight matrices have a multiple of 256 output rows.  Included by gemm.cu after
// gemm2sm.cuh, whose tile map, row-destination prefetch and row stores it shares.
//
// Same division of work as two_sm::gemm_i8_2sm_kernel -- a CTA pair computes a 256-weight-
// row x 192-token tile, weights converted by four warps per CTA into TMEM (the MMA's A
// operand), tokens TMA-loaded into shared memory (B, split between the pair), the leader
// issuing tcgen05.mma.cta_group::2.kind::i8 -- but TMEM is spent differently:
//
//   * one 192-column accumulator instead of two, and five 64-column weight stages instead
//     of two.  A converter may overwrite a weight stage only after the MMAs that read it
//     have completed; with two stages the converters get one stage (768 MMA cycles) of
//     slack, less than the ~1.4k-cycle round trip commit -> converters -> TMEM stores ->
//     leader -> issue, so every K stage waited on that chain.  With five stages the chain
//     has four stages of slack and the MMAs issue back to back;
//   * the accumulator is handed back as soon as it is in registers: twelve epilogue warps
//     (three per TMEM lane quarter, 64 tokens each) load their slice (tcgen05.ld), release
//     the accumulator, and only then apply the epilogue, stage BF16 rows in shared memory
//     and store them while the next tile's MMAs already run.
//
// Rings: 5 token slots of 24 KB (at least as many as TMEM weight stages: a converter
// learns that its stage is free from the token slot's commit of five stages back, which
// must not have been overtaken by a later phase of the same slot) and 3 weight slots of
// 16 KB.  No TMA multicast: token loads use the .cta_group::2 form, only tcgen05.commit
// multicasts.  Every wait is bounded (mbar_wait_bounded) and every role gives up cleanly.
#pragma once

namespace two_sm_deep {

using two_sm::BMP;
using two_sm::KS2;
using two_sm::MMA_W;
using two_sm::RowDest;
using two_sm::TileMap2;
using two_sm::TMA_W;
using two_sm::fetch_row_dest;
using two_sm::store_tile_rows;

// BN tokens per pair tile (BN / 2 per CTA): 192 (grouped launches, whose tile lists are built
// for 192-row tiles) or 256 (dense launches: a third more tensor work per MMA instruction and
// per tile boundary for the same issue and hand-over costs).
template <int BN>
struct DeepCfg {
  static_assert(BN == 192 || BN == 256, "tile width");
  static constexpr int HALF = BN / 2;                  // token rows per CTA
  static constexpr int TOK_B = HALF * KS2;             // token bytes per CTA and stage
  static constexpr int NSW = (512 - BN) / 64;          // TMEM weight stages, 64 columns each
  static constexpr int ACC_COL = 0;                    // accumulator columns [0, BN)
  static constexpr int WCOL = BN;                      // weight stages [BN, 512)
  static constexpr int TMEM_COLS = 512;
  static constexpr int NT = NSW;                       // token slots (>= NSW)
  static constexpr int NW = BN == 256 ? 2 : 3;         // int4 weight slots
  static constexpr int EPI = BN / 16;                  // epilogue warps: BN / 64 per lane quarter
  static constexpr int EPI_TOK = 64;                   // tokens drained per epilogue warp
  static constexpr int EPI_ROWS = BN / EPI;            // 16 stored token rows per epilogue warp
  // Warps 0-3 convert, 4 loads (TMA), 5 issues the MMAs, the epilogue warps follow.  At BN =
  // 256 the 24-warp block (two idle warps complete the second warpgroup) is launched with
  // 80 registers a thread; setmaxnreg then gives the converters 72, the TMA/MMA warpgroup 56
  // and the epilogue warps, which hold 64 accumulator values each, 88: 128 x 72 + 128 x 56 +
  // 512 x 88 = 768 x 80, the block's launch allocation.
  static constexpr int EPI_W0 = BN == 256 ? 8 : 6;     // first epilogue warp
  static constexpr int THREADS = 32 * (EPI_W0 + EPI);
  static constexpr bool REBALANCE = BN == 256;
  static constexpr int REG_CONV = 72, REG_LOW = 56, REG_EPI = 88;
  static constexpr int W_BYTES = 128 * KS2 / 2;        // 16 KB: one 128-row x 32-word tile block
  static constexpr int W_OFF = NT * TOK_B;
  static constexpr int RING = NT * TOK_B + NW * W_BYTES;
  static constexpr int STAGING = BN * 128 * 2;         // BF16 [token][column]
  static constexpr int SMEM = RING + STAGING + 1024 + 1024;
  static constexpr uint32_t IDESC = idesc_i8(256, BN);
  static_assert(NT >= NSW, "token-slot commits double as TMEM-stage releases");
  static_assert(WCOL + 64 * NSW <= TMEM_COLS, "TMEM budget");
  static_assert(SMEM <= 232448, "shared memory budget");
  static_assert(!REBALANCE || (THREADS == 768 && 128 * REG_CONV + 128 * REG_LOW + 32 * EPI * REG_EPI <= THREADS * 80),
                "register split must fit the launch allocation");
};

template <int NT, int NW, int NSW, int EPI>
struct Smem {
  uint64_t tok_full[NT], tok_empty[NT], wsm_full[NW], wsm_empty[NW];
  uint64_t wtm_full[NSW], acc_full, acc_empty;
  uint32_t sink[4 + EPI];  // targets of the follower's asynchronous 4-byte signals
  uint32_t tmem_base;
  int err;
};

template <bool GROUPED, int BN>
__global__ void __launch_bounds__(DeepCfg<BN>::THREADS, 1)
    gemm_i4_2sm_deep_kernel(const __grid_constant__ CUtensorMap tok_map, const __grid_constant__ CUtensorMap w_map0,
                            const __grid_constant__ CUtensorMap w_map1, GemmParams p) {
  using C = DeepCfg<BN>;
  constexpr int HALF = C::HALF, TOK_B = C::TOK_B, NSW = C::NSW, NT = C::NT, NW = C::NW, EPI = C::EPI;
  constexpr int ACC_COL = C::ACC_COL, WCOL = C::WCOL, TMEM_COLS = C::TMEM_COLS, W_BYTES = C::W_BYTES;
  constexpr int W_OFF = C::W_OFF, RING = C::RING, EPI_TOK = C::EPI_TOK, EPI_ROWS = C::EPI_ROWS;
  constexpr uint32_t IDESC = C::IDESC;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t *ring = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  uint16_t *staging = reinterpret_cast<uint16_t *>(ring + RING);
  Smem<NT, NW, NSW, EPI> &s = *reinterpret_cast<Smem<NT, NW, NSW, EPI> *>(ring + RING + C::STAGING);
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
  tm.span = BN;
  tm.total = (GROUPED ? p.tile_list[0] : (int)((p.m + BN - 1) / BN)) * tm.n_pairs;
  if (cluster >= tm.total) return;  // uniform across the pair
  const int k_stages = p.k / KS2;
  const int blocks_k = p.k / 256;   // 32-word (256-code) blocks per weight row

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
    for (int i = 0; i < NSW; ++i) mbar_init(&s.wtm_full[i], 4);
    mbar_init(&s.acc_full, 1);
    mbar_init(&s.acc_empty, EPI);
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
  // dense: the prologue above touches no global memory; tokens, scales, residual and
  // output wait for the previous kernel
  if (!GROUPED) {
    pdl_wait();
    pdl_trigger();
  }

  auto weight_tile = [&](int np, int expert, int &which, int &w_row_tile) {
    const int nt = 2 * np + (int)rank;
    which = nt / p.n_split;
    w_row_tile = expert * p.n_split + (nt - which * p.n_split);
  };

  if (warp == TMA_W) {
    // ---- TMA producer (both CTAs) -------------------------------------------------------
    if (C::REBALANCE) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(C::REG_LOW));
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
        // exact integer accumulation in any order: each tile starts its K sweep at its own
        // offset, so pairs sharing a token tile read different K slices at the same moment
        const int k_off = (int)((7u * (uint32_t)t) % (uint32_t)k_stages);
        for (int kk = 0; kk < k_stages; ++kk, ++g) {
          const int kb = kk + k_off < k_stages ? kk + k_off : kk + k_off - k_stages;
          const int sw = g % NW, st = g % NT;
          if (!(ok = mbar_wait_bounded(&s.wsm_empty[sw], ((g / NW) & 1) ^ 1, &s.err, 1))) break;
          mbar_arrive_expect_tx(&s.wsm_full[sw], W_BYTES);
          if (p.swiglu) {
            // 64 gate rows, then the 64 up rows of the same hidden columns: the converters'
            // rows 0-63 and 64-127 (each box keeps the 128-byte swizzle of its rows)
            const int blk = (expert * p.n_split + np) * blocks_k + kb;
            tma_load_3d(ring + W_OFF + sw * W_BYTES, &w_map0, &s.wsm_full[sw], 0, 64 * (int)rank, blk);
            tma_load_3d(ring + W_OFF + sw * W_BYTES + W_BYTES / 2, &w_map1, &s.wsm_full[sw], 0, 64 * (int)rank, blk);
          } else {
            tma_load_3d(ring + W_OFF + sw * W_BYTES, w_map, &s.wsm_full[sw], 0, 0, w_row_tile * blocks_k + kb);
          }
          if (!(ok = mbar_wait_bounded(&s.tok_empty[st], ((g / NT) & 1) ^ 1, &s.err, 1))) break;
          if (rank == 0) mbar_arrive_expect_tx(&s.tok_full[st], 2 * TOK_B);
          tma_load_3d_cg2(ring + st * TOK_B, &tok_map, mapa_shared(smem_u32(&s.tok_full[st]), 0), 0,
                          (int)(row0 + HALF * rank), 2 * kb);
        }
      }
    }
  } else if (warp == MMA_W) {
    // ---- MMA issuer (pair leader only) ---------------------------------------------------
    if (C::REBALANCE) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(C::REG_LOW));
    // One thread feeds both SMs' tensor pipes, and at N = 192 a stage's eight MMAs are only
    // 768 pipe cycles: the thread's own per-stage path must stay well under that, since it
    // competes for issue slots with the other warps of its SM sub-partition.  So the stage
    // loop is unrolled over the ring slots (NT == NSW: slot, TMEM stage and phase parity are
    // compile-time or flip once per round), every descriptor is computed once, and the next
    // stage's readiness is probed right after this stage's first MMA -- the probes' latency
    // passes while the MMAs queue -- and only waited on if a probe found it not ready.
    if (lane == 0 && rank == 0) {
      const int n_mine = (tm.total - cluster + nclusters - 1) / nclusters;
      const uint32_t total = (uint32_t)n_mine * (uint32_t)k_stages;
      uint64_t bdesc[NT];
#pragma unroll
      for (int q = 0; q < NT; ++q) bdesc[q] = smem_desc_sw128(smem_u32(ring + q * TOK_B));
      const uint32_t acc = tmem + ACC_COL;
      bool ok = mbar_wait_bounded(&s.tok_full[0], 0, &s.err, 2) && mbar_wait_bounded(&s.wtm_full[0], 0, &s.err, 3);
      tc_fence_after();
      uint32_t g = 0, par = 0, tile = 0;
      int kb = 0;
      while (ok && g < total) {
#pragma unroll
        for (int q = 0; q < NT; ++q) {
          if (!ok || g >= total) break;
          const int qn = q + 1 == NT ? 0 : q + 1;
          const uint32_t pn = q + 1 == NT ? par ^ 1 : par;
          const bool more = g + 1 < total;
          const uint32_t ab = tmem + WCOL + 64 * q;
          mma_i8_ts2(acc, ab, bdesc[q], IDESC, kb != 0);
          bool t_ok = true, w_ok = true;
          if (more) {
            t_ok = mbar_try_wait(&s.tok_full[qn], pn);
            w_ok = mbar_try_wait(&s.wtm_full[qn], pn);
          }
#pragma unroll
          for (int j = 1; j < KS2 / 32; ++j)
            mma_i8_ts2(acc, ab + 8 * j, bdesc[q] + (uint64_t)(((j >> 2) * (TOK_B / 2) + 32 * (j & 3)) >> 4), IDESC, 1u);
          // frees the token slot, and tells the converters this stage's TMEM weights are read
          mma_commit2_mc(&s.tok_empty[q], 3);
          ++g;
          if (++kb == k_stages) {
            kb = 0;
            mma_commit2_mc(&s.acc_full, 3);
            ++tile;
            // the epilogue has the finished tile's accumulator in registers
            if (more) ok = mbar_wait_bounded(&s.acc_empty, (tile & 1) ^ 1, &s.err, 7);
          }
          if (more && ok && !t_ok) ok = mbar_wait_bounded(&s.tok_full[qn], pn, &s.err, 2);
          if (more && ok && !w_ok) ok = mbar_wait_bounded(&s.wtm_full[qn], pn, &s.err, 3);
          tc_fence_after();
        }
        par ^= 1;
      }
      if (tile > 0) mbar_wait_bounded(&s.acc_full, (tile - 1) & 1, &s.err, 6);
    }
  } else if (warp < 4) {
    // ---- weight converters (both CTAs) -> own TMEM; stage-ready counted on the leader ----
    if (C::REBALANCE) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(C::REG_CONV));
    const int r = warp * 32 + lane;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const uint32_t lead_wtm_full = mapa_shared(smem_u32(&s.wtm_full[0]), 0);
    const uint32_t lead_sink = mapa_shared(smem_u32(&s.sink[warp]), 0);
    uint32_t g = 0;
    bool ok = true;
    for (int t = cluster; ok && t < tm.total; t += nclusters) {
      for (int kb = 0; kb < k_stages; ++kb, ++g) {
        const int st = g % NW, sw = g % NSW;
        bool waited = true;
        if (lane == 0) waited = mbar_wait_bounded(&s.wsm_full[st], (g / NW) & 1, &s.err, 4);
        waited = __shfl_sync(0xffffffffu, waited, 0) != 0;
        if (!(ok = waited)) break;
        const uint32_t wbase = smem_u32(ring + W_OFF + st * W_BYTES);
        // 128-byte rows, 128-byte swizzle: 16-byte chunk c of row r sits at chunk c ^ (r & 7)
        uint32_t w[32];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 v = lds_v4(wbase + r * 128 + 16 * (c ^ (r & 7)));
          w[4 * c] = v.x; w[4 * c + 1] = v.y; w[4 * c + 2] = v.z; w[4 * c + 3] = v.w;
        }
        mbar_arrive(&s.wsm_empty[st]);
        // TMEM stage sw was last read by the MMAs of stage g - NSW: their commit is the
        // completion of token slot (g - NSW) % NT's phase
        if (lane == 0 && g >= NSW) {
          const uint32_t gp = g - NSW;
          waited = mbar_wait_bounded(&s.tok_empty[gp % NT], (gp / NT) & 1, &s.err, 4);
        }
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
              o[h][8 * gq + q] = nib_lo16(w[16 * h + 4 * gq + q]);
              o[h][8 * gq + 4 + q] = nib_hi16(w[16 * h + 4 * gq + q]);
            }
          }
          tmem_st_x32(tmem + lane_base + WCOL + 64 * sw + 32 * h, o[h]);
        }
        tmem_st_wait(o[0]);
        tmem_st_keep(o[1]);
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
  } else if (warp < C::EPI_W0) {
    // idle warps that complete the TMA/MMA warpgroup for setmaxnreg
    if (C::REBALANCE) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(C::REG_LOW));
  } else {
    // ---- epilogue (both CTAs): this CTA's 128 weight rows x BN tokens -------------------
    if (C::REBALANCE) asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(C::REG_EPI));
    // Warp e reads TMEM lane quarter (warp & 3), tokens [64*part, 64*part + 64); it stores
    // token rows [16*eidx, 16*eidx + 16) of the staged tile.
    const int quarter = warp & 3;
    const int eidx = warp - C::EPI_W0;
    const int part = eidx >> 2;
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const uint32_t lead_acc_empty = mapa_shared(smem_u32(&s.acc_empty), 0);
    const uint32_t lead_sink = mapa_shared(smem_u32(&s.sink[4 + eidx]), 0);
    const float big = 3.3895313892515355e38f;
    const int c0 = part * EPI_TOK;
    const int m0 = eidx * EPI_ROWS;
    int i = 0;
    int64_t row0;
    int rows_valid, np, expert;
    for (int t = cluster; tm.get(p, t, row0, rows_valid, np, expert); t += nclusters, ++i) {
      bool have = true;
      if (lane == 0) have = mbar_wait_bounded(&s.acc_full, i & 1, &s.err, 5);
      have = __shfl_sync(0xffffffffu, have, 0) != 0;
      uint32_t accv[2][32];
      if (have) {
        // each warp drains its slice as soon as it sees the accumulator complete and hands
        // its part back at once; the warps agree on errors only afterwards
        tc_fence_after();
        tmem_ld_x32(tmem + lane_base + ACC_COL + c0, accv[0]);
        tmem_ld_x32(tmem + lane_base + ACC_COL + c0 + 32, accv[1]);
        tmem_ld_wait(accv[0]);
        tmem_ld_tie(accv[1]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (rank == 0) {
            if (eidx == 0) mbar_arrive_expect_tx(&s.acc_empty, 4 * EPI);
            else mbar_arrive(&s.acc_empty);
          } else {
            st_async_signal(lead_sink, lead_acc_empty);
          }
        }
      }
      if (!named_barrier_and(2, 32 * EPI, have)) break;
      // Activation scales, weight scale and row destinations are loaded only now: the next
      // tile's mainloop gives the epilogue plenty of time, and fewer values stay live across
      // the drain (the 64 accumulator registers are what the drain needs).
      float my_scale[2];
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int mj = c0 + 32 * q + lane;
        my_scale[q] = 0.0f;
        if (mj < rows_valid) {
          const int64_t pos = row0 + mj;
          if (GROUPED) {
            const int64_t route = p.perm[pos];
            my_scale[q] = p.a_scales[p.scale_mode == 0 ? pos : (p.scale_mode == 1 ? route / p.topk : route)];
          } else {
            my_scale[q] = p.a_scales[pos];
          }
        }
      }
      float ws;
      int col0;  // first output column of this CTA
      if (p.swiglu) {
        // TMEM lanes 0-63: gate rows, 64-127: up rows of hidden columns col0 .. col0 + 63
        col0 = np * 128 + 64 * (int)rank;
        ws = p.w_scales[r >> 6][(int64_t)expert * p.n_split * 128 + col0 + (r & 63)];
      } else {
        int which, w_row_tile;
        weight_tile(np, expert, which, w_row_tile);
        ws = p.w_scales[which][(int64_t)w_row_tile * 128 + r];
        col0 = (2 * np + (int)rank) * 128;
      }
      if (!GROUPED && p.out_f32) {
        // F32 output: the reference's epilogue value, stored as it is computed
#pragma unroll
        for (int q = 0; q < 2; ++q) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float as = __shfl_sync(0xffffffffu, my_scale[q], j);
            const float a = __int2float_rn((int)accv[q][j] >> 8);
            const float y = __fadd_rn(__fmul_rn(__fmul_rn(a, ws), as), 0.0f);
            const int m = c0 + 32 * q + j;
            if (m < rows_valid) p.out_f32[(row0 + m) * p.ldo + col0 + r] = y;
          }
        }
        continue;
      }
#pragma unroll
      for (int q = 0; q < 2; ++q) {
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          float y[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const float as = __shfl_sync(0xffffffffu, my_scale[q], j + u);
            const float a = __int2float_rn((int)accv[q][j + u] >> 8);
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
          const int m = c0 + 32 * q + j;
          staging[m * 128 + r] = (uint16_t)h2;
          staging[(m + 1) * 128 + r] = (uint16_t)(h2 >> 16);
        }
      }
      if (p.swiglu) {
        // hidden = bf16(bf16(silu(gate)) * up) of the staged BF16 projections (SiLU by
        // silu_bf16_ziv: arithmetic, the table only near rounding midpoints); lane l writes
        // hidden columns col0 + 2l, 2l + 1 of each of its 16 rows (128 bytes per row), at the
        // row's route id when grouped launches scatter
        named_barrier_sync(1, 32 * EPI);
#pragma unroll 2
        for (int mi = 0; mi < EPI_ROWS; ++mi) {
          const int m = m0 + mi;
          if (m >= rows_valid) break;
          const uint32_t gv = *reinterpret_cast<const uint32_t *>(staging + m * 128 + 2 * lane);
          const uint32_t uv = *reinterpret_cast<const uint32_t *>(staging + m * 128 + 64 + 2 * lane);
          const uint32_t s0 = silu_bf16_ziv(gv & 0xffffu, p.silu_tab);
          const uint32_t s1 = silu_bf16_ziv(gv >> 16, p.silu_tab);
          const float h0 = __fmul_rn(__uint_as_float(s0 << 16), __uint_as_float(uv << 16));
          const float h1 = __fmul_rn(__uint_as_float(s1 << 16), __uint_as_float(uv & 0xffff0000u));
          uint32_t h2;
          asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(h2) : "f"(h1), "f"(h0));
          const int64_t orow = (GROUPED && p.scatter) ? (int64_t)p.perm[row0 + m] : row0 + m;
          *reinterpret_cast<uint32_t *>(p.out + orow * p.ldo + col0 + 2 * lane) = h2;
        }
        named_barrier_sync(1, 32 * EPI);  // the staging buffer is free for the next tile
        continue;
      }
      const RowDest dest = fetch_row_dest<GROUPED>(p, row0, rows_valid, m0, m0 + EPI_ROWS, lane);
      named_barrier_sync(1, 32 * EPI);
      if (p.store16)
        store_tile_rows<GROUPED, 8>(p, staging, row0, rows_valid, col0, m0, m0 + EPI_ROWS, lane, dest);
      else
        store_tile_rows<GROUPED, 4>(p, staging, row0, rows_valid, col0, m0, m0 + EPI_ROWS, lane, dest);
      named_barrier_sync(1, 32 * EPI);  // the staging buffer is free for the next tile
    }
  }
  // stores into other GPUs' buffers (tensor-parallel output copies) are made visible at
  // system scope by each storing thread before the kernel ends
  if (!GROUPED && p.n_out_peer) __threadfence_system();
  tc_fence_before();
  cluster_sync();  // no CTA leaves while its peer may still signal it
  if (warp == MMA_W) {
    tc_fence_after();
    tmem_dealloc2(tmem, TMEM_COLS);
  }
  if (threadIdx.x == 0 && s.err) atomicCAS(p.err, 0, s.err);
}

}  // namespace two_sm_deep
