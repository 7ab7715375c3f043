// clefq: INT4/INT8 GEMM on 5th-generation tensor cores (tcgen05, kind::i8), sm_100a.
//
// Computes the reference's h3_gemm_i4_256 / h3_gemm_i8_256 contract
// (kernels/gemm_integer.loom:394-433):
//     acc[m][n] = sum_k a[m][k] * w[n][k]                  (int32, exact)
//     y         = (f32(acc) * ws[n]) * as[m] + 0            BF16 with finite saturation,
//                                                          optional residual / F32 output
// and, in grouped mode, the Omni expert contract (kernels/omni_expert_i4.loom:442-462):
//     y = f32(acc) * (as[x] * ws[e*n + c]) -> BF16, rows gathered/scattered by route.
//
// Data flow per CTA (one 128-weight-row x 128-token output tile):
//   * weights are the MMA "A" operand and live in tensor memory: four converter warps
//     each own 32 weight rows, read the tiled int4 words straight from global memory
//     (each row's 256 codes of a K block are 128 contiguous bytes of the reference's
//     128x32-word tile layout), sign-place each nibble as 16*code in an s8 lane and
//     store 64 TMEM columns per K=256 block with tcgen05.st;
//   * tokens are the MMA "B" operand: TMA streams the s8 operand (same 16*code values,
//     same K permutation) in 128-byte-swizzled K=128 boxes through a 3-stage ring;
//   * one thread issues tcgen05.mma.kind::i8 (M=128 weights, N=128 tokens, K=32) into a
//     TMEM int32 accumulator; tcgen05.commit frees ring slots;
//   * the converter warps then read the accumulator (tcgen05.ld), undo the exact x256
//     (>> 8) and apply the reference epilogue.
// No TMA multicast anywhere (safe in multi-GPU builds).
#include <cuda.h>

#include <atomic>

#include "clefq_internal.h"
#include "cq_common.cuh"

// 1: int4 pair launches take the deep-ring kernel (gemm2sm_deep.cuh); 0: the two-stage
// kernel of gemm2sm.cuh, kept for int8 and for comparison builds.
#ifndef CLEFQ_GEMM_DEEP
#define CLEFQ_GEMM_DEEP 1
#endif
// 1: grouped int4 launches of at most three K stages take the weight-resident kernel
// (gemm2sm_wres.cuh); 0: the two-stage kernel, kept for comparison builds.
#ifndef CLEFQ_GEMM_WRES
#define CLEFQ_GEMM_WRES 1
#endif
// 1: the pair GEMMs and the packing kernels are launched with programmatic stream
// serialization (each waits in-kernel for the previous kernel, griddepcontrol).
#ifndef CLEFQ_PDL
#define CLEFQ_PDL 1
#endif
#ifndef CLEFQ_WRES_SUBN
#define CLEFQ_WRES_SUBN 192   // tokens per MMA of the weight-resident kernel: 192 or 96
#endif

namespace cq {

namespace {

constexpr int BM = 128;                       // weight rows per tile (MMA M)
constexpr int BN = 128;                       // tokens per tile (MMA N)
constexpr int KS = 128;                       // codes per pipeline stage
constexpr int TOK_BYTES = BN * KS;            // 16 KiB: one 128-byte-swizzled TMA box
constexpr int TMEM_COLS = 512;                // 2 accumulators x 128 + weight stages x 32
constexpr int WCOL0 = 256;
constexpr int THREADS = 448;                  // 8 converter, 1 TMA, 1 MMA, 4 epilogue warps
constexpr int CONV_WARPS = 8;                 // two groups of 4: even and odd stages
constexpr int TMA_WARP = 8, MMA_WARP = 9;
constexpr uint32_t IDESC = idesc_i8(BM, BN);

constexpr int STAGING_BYTES = BN * BM * 2;    // one BF16 output tile [token][column]

template <int BITS>
struct Cfg {
  static constexpr int NS = BITS == 4 ? 8 : 6;           // ring depth
  static constexpr int W_BYTES = BM * KS * BITS / 8;     // packed weight bytes per stage
  static constexpr int STAGE = TOK_BYTES + W_BYTES;
  static constexpr int SMEM = NS * STAGE + STAGING_BYTES + 1024 + 512;
};

template <int NS>
struct Smem {
  uint64_t tok_full[NS], tok_empty[NS], wsm_full[NS], wsm_empty[NS], wtm_full[NS], wtm_empty[NS];
  uint64_t acc_full[2], acc_empty[2];
  uint32_t tmem_base;
  int err;
};

// Tile t of this launch -> (token tile row, output column tile, expert); false past the end.
struct TileMap {
  int n_tiles, total;
  CQ_DEV bool get(const GemmParams &p, int t, int64_t &row0, int &rows_valid, int &n_tile, int &expert) const {
    if (t >= total) return false;
    const int mt = t / n_tiles;
    n_tile = t - mt * n_tiles;
    if (p.grouped) {
      expert = p.tile_list[1 + 2 * mt];
      row0 = p.tile_list[2 + 2 * mt];
      const int64_t end = p.expert_offsets[expert + 1];
      rows_valid = (int)(end - row0 < BN ? end - row0 : BN);
    } else {
      expert = 0;
      row0 = (int64_t)mt * BN;
      rows_valid = (int)(p.m - row0 < BN ? p.m - row0 : BN);
    }
    return true;
  }
};

// Persistent: one CTA per SM walks tiles blockIdx.x, blockIdx.x + gridDim.x, ...
// Pipelines (all indexed by a stage counter g that runs across tiles):
//   TMA warp   -> tokens + packed weights into ring slot g % NS
//   converters -> weight slot: swizzled smem -> s8 (16*code) -> TMEM weight stage g % NS;
//                 two groups of four warps take alternate stages
//   MMA thread -> 4 x tcgen05.mma (K=32 each) into accumulator (tile & 1)
//   epilogue   -> drains accumulator (tile & 1) while the next tile accumulates in the other
template <bool GROUPED, int BITS>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tok_map, const __grid_constant__ CUtensorMap w_map0,
                   const __grid_constant__ CUtensorMap w_map1, GemmParams p) {
  using C = Cfg<BITS>;
  constexpr int NS = C::NS;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t *ring = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  uint16_t *staging = reinterpret_cast<uint16_t *>(ring + NS * C::STAGE);
  Smem<NS> &s = *reinterpret_cast<Smem<NS> *>(ring + NS * C::STAGE + STAGING_BYTES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  TileMap tm;
  tm.n_tiles = p.n / BM;
  tm.total = (GROUPED ? p.tile_list[0] : (int)((p.m + BN - 1) / BN)) * tm.n_tiles;
  if ((int)blockIdx.x >= tm.total) return;
  const int k_stages = p.k / KS;
  const int blocks_k = p.k / (32 * (32 / BITS));           // 32-word blocks per weight row

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&s.tok_full[i], 1);
      mbar_init(&s.tok_empty[i], 1);
      mbar_init(&s.wsm_full[i], 1);
      mbar_init(&s.wsm_empty[i], 128);
      mbar_init(&s.wtm_full[i], 128);
      mbar_init(&s.wtm_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.acc_full[i], 1);
      mbar_init(&s.acc_empty[i], 128);
    }
    s.err = 0;
    fence_barrier_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc(&s.tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == TMA_WARP) {
    // ---- TMA producer ------------------------------------------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&tok_map);
      tma_prefetch_desc(&w_map0);
      tma_prefetch_desc(&w_map1);
      uint32_t g = 0;
      bool ok = true;
      int64_t row0;
      int rows_valid, n_tile, expert;
      for (int t = blockIdx.x; ok && tm.get(p, t, row0, rows_valid, n_tile, expert); t += gridDim.x) {
        const int which = n_tile / p.n_split;
        const int w_row_tile = expert * p.n_split + (n_tile - which * p.n_split);
        const CUtensorMap *w_map = which ? &w_map1 : &w_map0;
        // staggered K start per tile (exact integer sums; spreads concurrent L2 reads)
        const int k_off = (int)((7u * (uint32_t)t) % (uint32_t)k_stages);
        for (int kk = 0; kk < k_stages; ++kk, ++g) {
          const int kb = kk + k_off < k_stages ? kk + k_off : kk + k_off - k_stages;
          const int st = g % NS;
          const uint32_t ph = ((g / NS) & 1) ^ 1;
          if (!(ok = mbar_wait_bounded(&s.tok_empty[st], ph, &s.err, 1) &&
                     mbar_wait_bounded(&s.wsm_empty[st], ph, &s.err, 1)))
            break;
          uint8_t *stage = ring + st * C::STAGE;
          mbar_arrive_expect_tx(&s.tok_full[st], TOK_BYTES);
          tma_load_2d(stage, &tok_map, &s.tok_full[st], kb * KS, (int)row0);
          mbar_arrive_expect_tx(&s.wsm_full[st], C::W_BYTES);
          if (BITS == 4)
            tma_load_3d(stage + TOK_BYTES, w_map, &s.wsm_full[st], (kb & 1) * 16, 0,
                        w_row_tile * blocks_k + (kb >> 1));
          else
            tma_load_3d(stage + TOK_BYTES, w_map, &s.wsm_full[st], 0, 0, w_row_tile * blocks_k + kb);
        }
      }
    }
  } else if (warp == MMA_WARP) {
    // ---- MMA issuer ----------------------------------------------------------------------
    if (lane == 0) {
      uint32_t g = 0;
      int i = 0;
      bool ok = true;
      int64_t row0;
      int rows_valid, n_tile, expert;
      for (int t = blockIdx.x; ok && tm.get(p, t, row0, rows_valid, n_tile, expert); t += gridDim.x, ++i) {
        const int buf = i & 1;
        if (!(ok = mbar_wait_bounded(&s.acc_empty[buf], ((i >> 1) & 1) ^ 1, &s.err, 7))) break;
        tc_fence_after();
        const uint32_t acc = tmem + BN * buf;
        for (int kb = 0; kb < k_stages; ++kb, ++g) {
          const int st = g % NS;
          const uint32_t ph = (g / NS) & 1;
          if (!(ok = mbar_wait_bounded(&s.tok_full[st], ph, &s.err, 2) &&
                     mbar_wait_bounded(&s.wtm_full[st], ph, &s.err, 3)))
            break;
          tc_fence_after();
          const uint32_t b_base = smem_u32(ring + st * C::STAGE);
#pragma unroll
          for (int j = 0; j < KS / 32; ++j)
            mma_i8_ts(acc, tmem + WCOL0 + 32 * st + 8 * j, smem_desc_sw128(b_base + 32 * j), IDESC, (kb | j) != 0);
          mma_commit(&s.tok_empty[st]);
          mma_commit(&s.wtm_empty[st]);
        }
        mma_commit(&s.acc_full[buf]);
      }
      // Every issued MMA has finished before TMEM is released, on every path.
      if (i > 0) mbar_wait_bounded(&s.acc_full[(i - 1) & 1], ((i - 1) >> 1) & 1, &s.err, 6);
    }
  } else if (warp < CONV_WARPS) {
    // ---- weight converters (warps 0-7): swizzled smem -> s8 -> TMEM ---------------------
    const int quarter = warp & 3;
    const uint32_t parity_group = warp >> 2;  // this group converts stages g with g % 2 == group
    const int r = quarter * 32 + lane;        // weight row within the tile == TMEM lane
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    uint32_t g = 0;
    bool ok = true;
    int64_t row0;
    int rows_valid, n_tile, expert;
    for (int t = blockIdx.x; ok && tm.get(p, t, row0, rows_valid, n_tile, expert); t += gridDim.x) {
      for (int kb = 0; kb < k_stages; ++kb, ++g) {
        if ((g & 1) != parity_group) continue;
        const int st = g % NS;
        const uint32_t ph = (g / NS) & 1;
        bool waited = true;
        if (lane == 0)
          waited = mbar_wait_bounded(&s.wsm_full[st], ph, &s.err, 4) &&
                   mbar_wait_bounded(&s.wtm_empty[st], ph ^ 1, &s.err, 4);
        waited = __shfl_sync(0xffffffffu, waited, 0) != 0;
        if (!(ok = waited)) break;
        tc_fence_after();
        const uint32_t wbase = smem_u32(ring + st * C::STAGE + TOK_BYTES);
        uint32_t o[32];
        if (BITS == 4) {
          // 64-byte rows, 64-byte swizzle: chunk c of row r sits at chunk c ^ ((r >> 1) & 3)
          uint32_t w[16];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint4 v = lds_v4(wbase + r * 64 + 16 * (c ^ ((r >> 1) & 3)));
            w[4 * c] = v.x; w[4 * c + 1] = v.y; w[4 * c + 2] = v.z; w[4 * c + 3] = v.w;
          }
          mbar_arrive(&s.wsm_empty[st]);
#pragma unroll
          for (int gq = 0; gq < 4; ++gq) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              o[8 * gq + q] = nib_lo16(w[4 * gq + q]);
              o[8 * gq + 4 + q] = nib_hi16(w[4 * gq + q]);
            }
          }
        } else {
          // 128-byte rows, 128-byte swizzle: chunk c of row r sits at chunk c ^ (r & 7)
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint4 v = lds_v4(wbase + r * 128 + 16 * (c ^ (r & 7)));
            o[4 * c] = v.x; o[4 * c + 1] = v.y; o[4 * c + 2] = v.z; o[4 * c + 3] = v.w;
          }
          mbar_arrive(&s.wsm_empty[st]);
        }
        tmem_st_x32(tmem + lane_base + WCOL0 + 32 * st, o);
        tmem_st_wait(o);
        tc_fence_before();
        mbar_arrive(&s.wtm_full[st]);
      }
    }
  } else {
    // ---- epilogue (warps 10-13) ---------------------------------------------------------
    // Phase 1: thread r owns output column r; per 32-token chunk it reads its accumulator
    // lane (tcgen05.ld), takes the token's activation scale from the lane that loaded it
    // (shuffle), applies the reference epilogue and writes BF16 into the staging tile.
    // Phase 2: each warp stores 32 token rows, 256 contiguous bytes per row (residual add
    // and route scatter happen here).
    const int quarter = warp & 3;        // TMEM lanes this warp may access
    const int r = quarter * 32 + lane;   // weight row within the tile
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const int shift = BITS == 4 ? 8 : 0;
    const float big = 3.3895313892515355e38f;
    int i = 0;
    int64_t row0;
    int rows_valid, n_tile, expert;
    for (int t = blockIdx.x; tm.get(p, t, row0, rows_valid, n_tile, expert); t += gridDim.x, ++i) {
      const int buf = i & 1;
      bool have = true;
      if (lane == 0) have = mbar_wait_bounded(&s.acc_full[buf], (i >> 1) & 1, &s.err, 5);
      have = __shfl_sync(0xffffffffu, have, 0) != 0;
      // all four epilogue warps agree before any of them reaches a named barrier
      if (!named_barrier_and(2, 128, have)) break;
      tc_fence_after();
      const int which = n_tile / p.n_split;
      const int64_t w_row = (int64_t)(expert * p.n_split + (n_tile - which * p.n_split)) * BM + r;
      const float ws = p.w_scales[which][w_row];
      const int n_local = n_tile * BM + r;  // output column
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t accv[32];
        tmem_ld_x32(tmem + lane_base + BN * buf + c, accv);
        // lane j fetches what token c + j needs: its activation scale (and route)
        const int mj = c + lane;
        float my_scale = 0.0f;
        if (mj < rows_valid) {
          const int64_t pos = row0 + mj;
          if (GROUPED) {
            const int64_t route = p.perm[pos];
            my_scale = p.a_scales[p.scale_mode == 0 ? pos : (p.scale_mode == 1 ? route / p.topk : route)];
          } else {
            my_scale = p.a_scales[pos];
          }
        }
        tmem_ld_wait(accv);
        if (c + 32 >= BN) {
          tc_fence_before();
          mbar_arrive(&s.acc_empty[buf]);  // accumulator free for tile i + 2
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float as = __shfl_sync(0xffffffffu, my_scale, j);
          const float a = __int2float_rn((int)accv[j] >> shift);
          uint16_t h;
          if (GROUPED) {
            h = f32_to_bf16(__fmul_rn(a, __fmul_rn(as, ws)));
          } else {
            const float y = __fadd_rn(__fmul_rn(__fmul_rn(a, ws), as), 0.0f);
            if (p.out_f32) {
              if (c + j < rows_valid) p.out_f32[(row0 + c + j) * p.ldo + n_local] = y;
              continue;
            }
            const float sat = maxnum(minnum(y, big), -big);
            h = f32_to_bf16(fabsf(y) < __int_as_float(0x7f800000) ? sat : y);
          }
          staging[(c + j) * BM + r] = h;
        }
      }
      if (GROUPED || !p.out_f32) {
        named_barrier_sync(1, 128);
        // phase 2: rows quarter*32 .. quarter*32+31, lane covers columns 4*lane .. 4*lane+3
        for (int m = quarter * 32; m < quarter * 32 + 32 && m < rows_valid; ++m) {
          const int64_t pos = row0 + m;
          int64_t orow = pos;
          if (GROUPED && p.scatter) orow = p.perm[pos];
          uint2 v = *reinterpret_cast<const uint2 *>(staging + m * BM + 4 * lane);
          if (!GROUPED && p.residual) {
            const uint2 rv = *reinterpret_cast<const uint2 *>(p.residual + pos * p.ldr + n_tile * BM + 4 * lane);
            const uint16_t *hv = reinterpret_cast<const uint16_t *>(&v);
            const uint16_t *hr = reinterpret_cast<const uint16_t *>(&rv);
            uint16_t o4[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) o4[q] = f32_to_bf16(__fadd_rn(bf16_to_f32(hr[q]), bf16_to_f32(hv[q])));
            v = *reinterpret_cast<uint2 *>(o4);
          }
          *reinterpret_cast<uint2 *>(p.out + orow * p.ldo + n_tile * BM + 4 * lane) = v;
        }
        named_barrier_sync(1, 128);  // staging is reused by the next tile
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
  if (threadIdx.x == 0 && s.err) atomicCAS(p.err, 0, s.err);
}

#include "gemm2sm.cuh"
#include "gemm2sm_deep.cuh"
#include "gemm2sm_wres.cuh"
#ifndef CLEFQ_DEEP_MIN_KSTAGES
#define CLEFQ_DEEP_MIN_KSTAGES 8   // fewest 256-wide K stages an int4 launch needs for the deep-ring kernel
#endif

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  // a function-local static is initialised once, even with concurrent first callers
  static const EncodeTiledFn fn = [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeTiledFn>(ptr);
    return static_cast<EncodeTiledFn>(nullptr);
  }();
  return fn;
}

}  // namespace

// Weight tiles viewed as a 3D tensor: x = 32 words of one block row, y = 128 rows,
// z = 128x32-word blocks in (row block, k block) order; one box = the K=128 slice of a
// row block (16 words for int4, 32 for int8), swizzled to match the converter reads.
static bool weight_map(EncodeTiledFn enc, CUtensorMap *m, const uint32_t *w, int64_t rows, int k, int bits) {
  const int64_t blocks = rows / 128 * (k / (32 * (32 / bits)));
  cuuint64_t dims[3] = {32, 128, (cuuint64_t)blocks};
  cuuint64_t strides[2] = {128, 16384};
  cuuint32_t box[3] = {(cuuint32_t)(bits == 4 ? 16 : 32), 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint32_t *>(w), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, bits == 4 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The same weight tiles with one box = 64 rows of one block (the SwiGLU epilogue's gate or up
// half of a CTA's 128 weight rows), 8 KB, 128-byte swizzled.
static bool weight_map_half(EncodeTiledFn enc, CUtensorMap *m, const uint32_t *w, int64_t rows, int k) {
  const int64_t blocks = rows / 128 * (k / 256);
  cuuint64_t dims[3] = {32, 128, (cuuint64_t)blocks};
  cuuint64_t strides[2] = {128, 16384};
  cuuint32_t box[3] = {32, 64, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint32_t *>(w), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The same weight tiles with one box = one whole block (int4) or two consecutive blocks
// (int8): 16 or 32 KB contiguous, 128-byte swizzled.
static bool weight_map_blocks(EncodeTiledFn enc, CUtensorMap *m, const uint32_t *w, int64_t rows, int k, int bits) {
  const int64_t blocks = rows / 128 * (k / (32 * (32 / bits)));
  cuuint64_t dims[3] = {32, 128, (cuuint64_t)blocks};
  cuuint64_t strides[2] = {128, 16384};
  cuuint32_t box[3] = {32, 128, (cuuint32_t)(bits == 4 ? 1 : 2)};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint32_t *>(w), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool G, int B>
static void launch_variant(dim3 grid, const CUtensorMap &t, const CUtensorMap &w0, const CUtensorMap &w1,
                           const GemmParams &p, cudaStream_t stream) {
  static std::atomic<bool> attr[64];  // per device: the shared-memory limit is a per-context attribute
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr[dev].load(std::memory_order_acquire)) {
    cudaFuncSetAttribute(gemm_i8_kernel<G, B>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<B>::SMEM);
    if (dev >= 0 && dev < 64) attr[dev].store(true, std::memory_order_release);
  }
  gemm_i8_kernel<G, B><<<grid, THREADS, Cfg<B>::SMEM, stream>>>(t, w0, w1, p);
}

using PairKernel = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, GemmParams);

// Launch a pair kernel on as many co-resident clusters of 2 as the device holds.  KEY
// distinguishes the kernels' per-device caches.
template <int KEY>
static cudaError_t launch_pair_kernel(PairKernel kern, int threads, int smem, int64_t pair_tiles,
                                      const CUtensorMap &t, const CUtensorMap &w0, const CUtensorMap &w1,
                                      const GemmParams &p, cudaStream_t stream) {
  // per device, like the shared-memory attribute; set (release) only after the attribute call
  static std::atomic<int> max_clusters_dev[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::atomic<int> scratch{0};
  std::atomic<int> &slot = (dev >= 0 && dev < 64) ? max_clusters_dev[dev] : scratch;
  int max_clusters = slot.load(std::memory_order_acquire);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (!max_clusters) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    cfg.gridDim = dim3(2 * 74);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) n = device_sms() / 2;
    max_clusters = n;
    slot.store(n, std::memory_order_release);
  }
  const int64_t clusters = pair_tiles < max_clusters ? pair_tiles : max_clusters;
  cfg.gridDim = dim3((unsigned)(2 * clusters));
  // programmatic dependent launch: the pair kernels wait for the previous kernel in-kernel
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = CLEFQ_PDL;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, t, w0, w1, p);
}

template <bool G, int B, int SUB = 1>
static cudaError_t launch_variant_2sm(int64_t pair_tiles, const CUtensorMap &t, const CUtensorMap &w0,
                                      const CUtensorMap &w1, const GemmParams &p, cudaStream_t stream) {
  return launch_pair_kernel<(G ? 1 : 0) + 2 * B + 100 * SUB>(two_sm::gemm_i8_2sm_kernel<G, B, SUB>, two_sm::THREADS2,
                                                             two_sm::Cfg2<B, SUB>::SMEM, pair_tiles, t, w0, w1, p,
                                                             stream);
}

template <bool G, int BN>
static cudaError_t launch_deep_2sm(int64_t pair_tiles, const CUtensorMap &t, const CUtensorMap &w0,
                                   const CUtensorMap &w1, const GemmParams &p, cudaStream_t stream) {
  using C = two_sm_deep::DeepCfg<BN>;
  return launch_pair_kernel<1000 + BN + (G ? 1 : 0)>(two_sm_deep::gemm_i4_2sm_deep_kernel<G, BN>, C::THREADS, C::SMEM,
                                                     pair_tiles, t, w0, w1, p, stream);
}

static cudaError_t launch_wres_2sm(int64_t pair_tiles, const CUtensorMap &t, const CUtensorMap &w0,
                                   const CUtensorMap &w1, const GemmParams &p, cudaStream_t stream) {
  return launch_pair_kernel<2000 + CLEFQ_WRES_SUBN>(two_sm_wres::gemm_i4_2sm_wres_kernel<CLEFQ_WRES_SUBN>,
                                                    two_sm_wres::THREADS, two_sm_wres::WresCfg<CLEFQ_WRES_SUBN>::SMEM,
                                                    pair_tiles, t, w0, w1, p, stream);
}

bool gemm_uses_pairs(const GemmParams &p) { return p.n_split % 2 == 0 && p.n % 256 == 0; }

// Whether launch_gemm can apply the SwiGLU epilogue to a gate|up launch of n_each rows per
// weight matrix and depth k: int4 on the deep-ring kernel.
bool gemm_swiglu_ok(int64_t n_each, int64_t k) {
  return CLEFQ_GEMM_DEEP && n_each % 256 == 0 && k % 256 == 0 && k / 256 >= 8 && silu_table_device() != nullptr;
}
int gemm_tile_rows(int n, int n_split) { return (n_split % 2 == 0 && n % 256 == 0) ? two_sm::BN2 : BN; }

static bool allows_store16(const GemmParams &p) {
  auto al = [](const void *q) { return ((uintptr_t)q & 15) == 0; };
  if (p.ldo % 8 || (p.out && !al(p.out)) || (p.residual && (!al(p.residual) || p.ldr % 8))) return false;
  for (int d = 0; d < p.n_out_peer; ++d)
    if (!al(p.out_peer[d])) return false;
  return true;
}

int launch_gemm(const GemmParams &p0, cudaStream_t stream) {
  GemmParams p = p0;
  p.store16 = allows_store16(p);
  if (p.n % BM || p.k % 256 || p.k <= 0 || p.n <= 0) return CLEFQ_ERR_SHAPE;
  if (!(p.bits == 4 || p.bits == 8)) return CLEFQ_ERR_SHAPE;
  if ((uintptr_t)p.a_op % 16 || p.a_ld % 16 || p.a_ld < p.k) return CLEFQ_ERR_ALIGN;
  const bool two = p.n / BM > p.n_split;
  if (p.n_split <= 0 || (p.n / BM) % p.n_split || p.n / BM > 2 * p.n_split) return CLEFQ_ERR_SHAPE;
  if ((uintptr_t)p.w[0] % 16 || (two && (uintptr_t)p.w[1] % 16)) return CLEFQ_ERR_ALIGN;
  // the epilogue stores 8-byte groups of four BF16 columns
  if (p.out && ((uintptr_t)p.out % 8 || p.ldo % 4)) return CLEFQ_ERR_ALIGN;
  if (p.residual && ((uintptr_t)p.residual % 8 || p.ldr % 4)) return CLEFQ_ERR_ALIGN;
  const bool pairs = gemm_uses_pairs(p);
  if (p.n_out_peer && (!pairs || p.grouped || !p.out || p.n_out_peer > kMaxPeers)) return CLEFQ_ERR_SHAPE;
  if (p.swiglu && (!pairs || p.bits != 4)) return CLEFQ_ERR_SHAPE;
  for (int d = 0; d < p.n_out_peer; ++d)
    if ((uintptr_t)p.out_peer[d] % 8) return CLEFQ_ERR_ALIGN;
  const int tile_rows = pairs ? two_sm::BN2 : BN;
  if (p.grouped && p.tile_rows != tile_rows) return CLEFQ_ERR_SHAPE;  // tile list built for the other kernel
  const int64_t tiles_m = p.grouped ? p.max_tiles : (p.m + tile_rows - 1) / tile_rows;
  if (tiles_m == 0 || p.a_rows == 0) return 0;
  if (tiles_m * (p.n / BM) > 0x7fffffff) return CLEFQ_ERR_SHAPE;
  EncodeTiledFn enc = encode_fn();
  if (!enc) return CLEFQ_ERR_CUDA;
  CUtensorMap tmap, wmap0, wmap1;
  cuuint64_t dims[2] = {(cuuint64_t)p.k, (cuuint64_t)p.a_rows};
  cuuint64_t strides[1] = {(cuuint64_t)p.a_ld};
  cuuint32_t box[2] = {128, (cuuint32_t)(pairs ? two_sm::HALF : BN)};
  cuuint32_t estr[2] = {1, 1};
  CUresult rc = enc(&tmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(p.a_op), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (rc != CUDA_SUCCESS) return CLEFQ_ERR_CUDA;
  const int64_t experts = p.grouped ? p.experts : 1;
  const int64_t wrows = experts * p.n_split * (int64_t)BM;
  if (!weight_map(enc, &wmap0, p.w[0], wrows, p.k, p.bits)) return CLEFQ_ERR_CUDA;
  if (two) {
    if (!weight_map(enc, &wmap1, p.w[1], wrows, p.k, p.bits)) return CLEFQ_ERR_CUDA;
  } else {
    wmap1 = wmap0;
  }
  if (pairs) {
#if CLEFQ_GEMM_DEEP
    // int4 with at least 8 K stages: the deep-ring kernel, 256-token tiles for dense launches
    // and 192 for grouped ones (their tile lists are built for 192 rows).  Shorter K keeps
    // the two-stage kernel, whose double-buffered accumulators hide the tile hand-over that
    // a few K stages cannot amortise.  A dense launch of one 256-token tile or less (C1: 128
    // tokens, 3 pair tiles, 29.6 against 25.6 us per call) is latency-bound and keeps the
    // two-stage kernel, whose set-up is lighter, unless it applies SwiGLU.
    const bool deep = p.bits == 4 && p.k / 256 >= CLEFQ_DEEP_MIN_KSTAGES && (p.grouped || p.swiglu || p.m > 256);
#else
    const bool deep = false;
#endif
    // grouped int4 with at most three K stages (the MoE down projection, K = 768): the
    // weight-resident kernel over the 192-row tile list
    const bool wres = CLEFQ_GEMM_WRES && p.grouped && p.bits == 4 && !p.swiglu && p.k / 256 <= two_sm_wres::MAX_KST;
    const int deep_bn = p.grouped ? 192 : 256;
    const int half = wres ? two_sm_wres::WresCfg<CLEFQ_WRES_SUBN>::SH : (deep ? deep_bn / 2 : two_sm::HALF);
    // token operand as 3D: x = 128 bytes of a K slice, y = rows (pitch a_ld), z = K slices
    cuuint64_t d3[3] = {128, (cuuint64_t)p.a_rows, (cuuint64_t)(p.k / 128)};
    cuuint64_t s3[2] = {(cuuint64_t)p.a_ld, 128};
    cuuint32_t b3[3] = {128, (cuuint32_t)half, 2};
    cuuint32_t e3[3] = {1, 1, 1};
    if (enc(&tmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t *>(p.a_op), d3, s3, b3, e3,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return CLEFQ_ERR_CUDA;
    if (p.swiglu) {
      // the SwiGLU epilogue pairs gate and up rows of the same hidden columns in one CTA
      if (!deep || !two || p.residual || p.out_f32 || p.n_out_peer || (p.scatter && !p.grouped) ||
          !p.out || !p.silu_tab || p.ldo % 2)
        return CLEFQ_ERR_SHAPE;
      if (!weight_map_half(enc, &wmap0, p.w[0], wrows, p.k) || !weight_map_half(enc, &wmap1, p.w[1], wrows, p.k))
        return CLEFQ_ERR_CUDA;
    } else {
      // weights: whole 128-row x 32-word blocks (int8: the two blocks of a K=256 slice)
      if (!weight_map_blocks(enc, &wmap0, p.w[0], wrows, p.k, p.bits)) return CLEFQ_ERR_CUDA;
      if (two) {
        if (!weight_map_blocks(enc, &wmap1, p.w[1], wrows, p.k, p.bits)) return CLEFQ_ERR_CUDA;
      } else {
        wmap1 = wmap0;
      }
    }
    const int64_t pair_tiles = tiles_m * (p.n / two_sm::BMP);
    cudaError_t e;
    if (wres) {
      e = launch_wres_2sm(pair_tiles, tmap, wmap0, wmap1, p, stream);
      return e == cudaSuccess ? 0 : CLEFQ_ERR_CUDA;
    }
    if (deep) {
      if (p.grouped) {
        e = launch_deep_2sm<true, 192>(pair_tiles, tmap, wmap0, wmap1, p, stream);
      } else {
        const int64_t tiles256 = ((p.m + 255) / 256) * (p.n / two_sm::BMP);
        e = launch_deep_2sm<false, 256>(tiles256, tmap, wmap0, wmap1, p, stream);
      }
      return e == cudaSuccess ? 0 : CLEFQ_ERR_CUDA;
    }
    // dense int4 with at least two token tiles: two sub-tiles per pair tile sharing each
    // converted weight stage
    if (!p.grouped && p.bits == 4 && p.m >= 2 * two_sm::BN2) {
      const int64_t pair_tiles2 = ((p.m + 2 * two_sm::BN2 - 1) / (2 * two_sm::BN2)) * (p.n / two_sm::BMP);
      e = launch_variant_2sm<false, 4, 2>(pair_tiles2, tmap, wmap0, wmap1, p, stream);
      return e == cudaSuccess ? 0 : CLEFQ_ERR_CUDA;
    }
    if (p.grouped)
      e = p.bits == 4 ? launch_variant_2sm<true, 4>(pair_tiles, tmap, wmap0, wmap1, p, stream)
                      : launch_variant_2sm<true, 8>(pair_tiles, tmap, wmap0, wmap1, p, stream);
    else
      e = p.bits == 4 ? launch_variant_2sm<false, 4>(pair_tiles, tmap, wmap0, wmap1, p, stream)
                      : launch_variant_2sm<false, 8>(pair_tiles, tmap, wmap0, wmap1, p, stream);
    return e == cudaSuccess ? 0 : CLEFQ_ERR_CUDA;
  }
  // Persistent grid: one CTA per SM (grouped launches do not know their tile count on
  // the host; surplus CTAs exit at once).
  const int64_t total = tiles_m * (p.n / BM);
  const int sms = device_sms();
  dim3 grid((unsigned)(total < sms ? total : sms));
  if (p.grouped) {
    if (p.bits == 4) launch_variant<true, 4>(grid, tmap, wmap0, wmap1, p, stream);
    else launch_variant<true, 8>(grid, tmap, wmap0, wmap1, p, stream);
  } else {
    if (p.bits == 4) launch_variant<false, 4>(grid, tmap, wmap0, wmap1, p, stream);
    else launch_variant<false, 8>(grid, tmap, wmap0, wmap1, p, stream);
  }
  return launch_check();
}

}  // namespace cq
