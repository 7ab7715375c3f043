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

#include "clefq_internal.h"
#include "cq_common.cuh"

namespace cq {

namespace {

constexpr int BM = 128;                       // weight rows per tile (MMA M)
constexpr int BN = 128;                       // tokens per tile (MMA N)
constexpr int KB = 256;                       // codes per K block
constexpr int NS = 3;                         // token ring stages (KB bytes x BN rows each)
constexpr int STAGE_BYTES = BN * KB;          // 32 KiB
constexpr int TMEM_COLS = 256;                // acc 128 + two 64-column weight stages
constexpr int ACC_COL = 0;
constexpr int WCOL0 = 128;
constexpr int THREADS = 192;
constexpr uint32_t IDESC = idesc_i8(BM, BN);
constexpr int SMEM_BYTES = NS * STAGE_BYTES + 1024 /*align slack*/ + 256 /*barriers*/;

struct Smem {
  uint64_t tok_full[NS], tok_empty[NS], w_full[2], w_empty[2], acc_full;
  uint32_t tmem_base;
  int err;
};

// One K=256 block of a weight row (32 packed int4 words) -> 64 TMEM columns of s8
// (16 * code, K-permuted like the token operand), stored as two 32-column halves.
CQ_DEV void store_block_i4(const uint32_t (&w)[32], uint32_t taddr) {
  uint32_t o[32];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
#pragma unroll
    for (int g = 0; g < 4; ++g) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        o[8 * g + i] = nib_lo16(w[16 * h + 4 * g + i]);
        o[8 * g + 4 + i] = nib_hi16(w[16 * h + 4 * g + i]);
      }
    }
    tmem_st_x32(taddr + 32 * h, o);
  }
}

CQ_DEV void load_words(uint32_t (&w)[32], const uint32_t *src) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    uint4 v = ldg_nc_v4(src + 4 * i);
    w[4 * i] = v.x;
    w[4 * i + 1] = v.y;
    w[4 * i + 2] = v.z;
    w[4 * i + 3] = v.w;
  }
}

template <bool GROUPED>
__global__ void __launch_bounds__(THREADS, 2) gemm_i8_kernel(const __grid_constant__ CUtensorMap tmap, GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t *ring = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  Smem &s = *reinterpret_cast<Smem *>(ring + NS * STAGE_BYTES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // ---- tile coordinates ------------------------------------------------------------
  int n_tile = blockIdx.x;                 // weight-row tile
  int64_t row0;                            // first operand row of the token tile
  int rows_valid;                          // token rows of this tile that are real
  int expert = 0;
  if (GROUPED) {
    const int ntiles = p.tile_list[0];
    if ((int)blockIdx.y >= ntiles) return;
    expert = p.tile_list[1 + 2 * blockIdx.y];
    row0 = p.tile_list[2 + 2 * blockIdx.y];
    const int64_t end = p.expert_offsets[expert + 1];
    rows_valid = (int)(end - row0 < BN ? end - row0 : BN);
  } else {
    row0 = (int64_t)blockIdx.y * BN;
    rows_valid = (int)(p.m - row0 < BN ? p.m - row0 : BN);
  }
  const int k_blocks = p.k / KB;
  const int words_per_row_block = 32;                       // 128 bytes of one tiled row
  const int64_t blocks_k = (int64_t)p.k / (32 * (32 / p.bits));
  const int which = n_tile / p.n_split;                    // weight matrix feeding this tile
  const int local_tile = n_tile - which * p.n_split;
  const int64_t w_row_tile = (int64_t)expert * p.n_split + local_tile;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&s.tok_full[i], 1);
      mbar_init(&s.tok_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.w_full[i], 128);
      mbar_init(&s.w_empty[i], 1);
    }
    mbar_init(&s.acc_full, 1);
    s.err = 0;
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(&s.tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == 4) {
    // ---- TMA producer ----------------------------------------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&tmap);
      for (int kb = 0; kb < k_blocks; ++kb) {
        const int st = kb % NS;
        const uint32_t ph = (kb / NS) & 1;
        if (!mbar_wait_bounded(&s.tok_empty[st], ph ^ 1, &s.err, 1)) break;
        mbar_arrive_expect_tx(&s.tok_full[st], STAGE_BYTES);
        uint8_t *dst = ring + st * STAGE_BYTES;
        tma_load_2d(dst, &tmap, &s.tok_full[st], kb * KB, (int)row0);
        tma_load_2d(dst + STAGE_BYTES / 2, &tmap, &s.tok_full[st], kb * KB + 128, (int)row0);
      }
    }
  } else if (warp == 5) {
    // ---- MMA issuer ------------------------------------------------------------------
    if (lane == 0) {
      bool ok = true;
      for (int kb = 0; kb < k_blocks && ok; ++kb) {
        const int st = kb % NS;
        const uint32_t pt = (kb / NS) & 1;
        const int sw = kb & 1;
        const uint32_t pw = (kb >> 1) & 1;
        ok = mbar_wait_bounded(&s.tok_full[st], pt, &s.err, 2) && mbar_wait_bounded(&s.w_full[sw], pw, &s.err, 3);
        if (!ok) break;
        tc_fence_after();
        const uint32_t b_base = smem_u32(ring + st * STAGE_BYTES);
#pragma unroll
        for (int j = 0; j < KB / 32; ++j) {
          const uint32_t b_addr = b_base + (j >> 2) * (STAGE_BYTES / 2) + (j & 3) * 32;
          mma_i8_ts(tmem + ACC_COL, tmem + WCOL0 + 64 * sw + 8 * j, smem_desc_sw128(b_addr), IDESC,
                    (kb | j) != 0);
        }
        mma_commit(&s.tok_empty[st]);
        mma_commit(&s.w_empty[sw]);
      }
      mma_commit(&s.acc_full);
      // Every issued MMA has finished before TMEM is released, on every path.
      mbar_wait_bounded(&s.acc_full, 0, &s.err, 6);
    }
  } else {
    // ---- weight converters (warps 0-3), then epilogue ---------------------------------
    const int r = warp * 32 + lane;  // weight row within the tile == TMEM lane
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const uint32_t *wrow = p.w[which] + (w_row_tile * blocks_k) * 4096 + r * words_per_row_block;
    bool ok = true;
    // Wait for weight stage kb % 2 to be free (warp-uniform), returns false on timeout.
    auto acquire = [&](int kb) -> bool {
      bool waited = true;
      if (lane == 0) waited = mbar_wait_bounded(&s.w_empty[kb & 1], ((kb >> 1) & 1) ^ 1, &s.err, 4);
      waited = __shfl_sync(0xffffffffu, waited, 0) != 0;
      if (waited) tc_fence_after();
      return waited;
    };
    auto release = [&](int kb) {
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&s.w_full[kb & 1]);
    };
    if (p.bits == 4) {
      // Three register buffers: loads run two K blocks ahead of the TMEM stores.
      uint32_t b0[32], b1[32], b2[32];
      auto consume = [&](uint32_t (&b)[32], int kb) -> bool {
        if (!acquire(kb)) return false;
        store_block_i4(b, tmem + lane_base + WCOL0 + 64 * (kb & 1));
        release(kb);
        return true;
      };
      load_words(b0, wrow);
      if (k_blocks > 1) load_words(b1, wrow + 4096);
      for (int kb = 0; kb < k_blocks && ok; kb += 3) {
        if (kb + 2 < k_blocks) load_words(b2, wrow + (int64_t)(kb + 2) * 4096);
        if (!(ok = consume(b0, kb))) break;
        if (kb + 1 >= k_blocks) break;
        if (kb + 3 < k_blocks) load_words(b0, wrow + (int64_t)(kb + 3) * 4096);
        if (!(ok = consume(b1, kb + 1))) break;
        if (kb + 2 >= k_blocks) break;
        if (kb + 4 < k_blocks) load_words(b1, wrow + (int64_t)(kb + 4) * 4096);
        if (!(ok = consume(b2, kb + 2))) break;
      }
    } else {
      // int8 tiles hold 128 codes per block row: two tiled blocks fill one 256-code stage.
      for (int kb = 0; kb < k_blocks; ++kb) {
        uint32_t lo[32], hi[32];
        load_words(lo, wrow + (int64_t)(2 * kb) * 4096);
        load_words(hi, wrow + (int64_t)(2 * kb + 1) * 4096);
        if (!(ok = acquire(kb))) break;
        tmem_st_x32(tmem + lane_base + WCOL0 + 64 * (kb & 1), lo);
        tmem_st_x32(tmem + lane_base + WCOL0 + 64 * (kb & 1) + 32, hi);
        release(kb);
      }
    }
    // ---- epilogue ----------------------------------------------------------------------
    bool have = ok;
    if (lane == 0 && have) have = mbar_wait_bounded(&s.acc_full, 0, &s.err, 5);
    have = __shfl_sync(0xffffffffu, have, 0);
    if (have) {
      tc_fence_after();
      const int n_local = n_tile * BM + r;  // output column
      const float ws = p.w_scales[which][w_row_tile * BM + r];
      const int shift = p.bits == 4 ? 8 : 0;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t acc[32];
        tmem_ld_x32(tmem + lane_base + ACC_COL + c, acc);
        tmem_ld_wait();
#pragma unroll 4
        for (int j = 0; j < 32; ++j) {
          const int mi = c + j;
          if (mi >= rows_valid) break;
          const int64_t pos = row0 + mi;
          const float a = __int2float_rn((int)acc[j] >> shift);
          if (GROUPED) {
            const int64_t route = p.perm[pos];
            const int64_t sidx = p.scale_mode == 0 ? pos : (p.scale_mode == 1 ? route / p.topk : route);
            const int64_t orow = p.scatter ? route : pos;
            const float sc = __fmul_rn(p.a_scales[sidx], ws);
            p.out[orow * p.ldo + n_local] = f32_to_bf16(__fmul_rn(a, sc));
          } else {
            const float y = __fadd_rn(__fmul_rn(__fmul_rn(a, ws), p.a_scales[pos]), 0.0f);
            if (p.out_f32) {
              p.out_f32[pos * p.ldo + n_local] = y;
            } else {
              const float big = 3.3895313892515355e38f;
              const float sat = maxnum(minnum(y, big), -big);
              uint16_t h = f32_to_bf16(fabsf(y) < __int_as_float(0x7f800000) ? sat : y);
              if (p.residual)
                h = f32_to_bf16(__fadd_rn(bf16_to_f32(p.residual[pos * p.ldr + n_local]), bf16_to_f32(h)));
              p.out[pos * p.ldo + n_local] = h;
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
  if (threadIdx.x == 0 && s.err) atomicCAS(p.err, 0, s.err);
}

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

}  // namespace

int launch_gemm(const GemmParams &p, cudaStream_t stream) {
  if (p.n % BM || p.k % KB || p.k <= 0 || p.n <= 0) return CLEFQ_ERR_SHAPE;
  if (!(p.bits == 4 || p.bits == 8)) return CLEFQ_ERR_SHAPE;
  if ((uintptr_t)p.a_op % 16 || p.a_ld % 16 || p.a_ld < p.k) return CLEFQ_ERR_ALIGN;
  if ((uintptr_t)p.w[0] % 16 || (p.n / BM > p.n_split && (uintptr_t)p.w[1] % 16)) return CLEFQ_ERR_ALIGN;
  if (p.n_split <= 0 || (p.n / BM) % p.n_split || p.n / BM > 2 * p.n_split) return CLEFQ_ERR_SHAPE;
  const int64_t tiles_m = p.grouped ? p.max_tiles : (p.m + BN - 1) / BN;
  if (tiles_m == 0 || p.a_rows == 0) return 0;
  if (tiles_m > 65535) return CLEFQ_ERR_SHAPE;
  EncodeTiledFn enc = encode_fn();
  if (!enc) return CLEFQ_ERR_CUDA;
  CUtensorMap tmap;
  cuuint64_t dims[2] = {(cuuint64_t)p.k, (cuuint64_t)p.a_rows};
  cuuint64_t strides[1] = {(cuuint64_t)p.a_ld};
  cuuint32_t box[2] = {128, (cuuint32_t)BN};
  cuuint32_t estr[2] = {1, 1};
  CUresult rc = enc(&tmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(p.a_op), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (rc != CUDA_SUCCESS) return CLEFQ_ERR_CUDA;
  static bool attr_set[2] = {false, false};
  dim3 grid(p.n / BM, (unsigned)tiles_m);
  if (p.grouped) {
    if (!attr_set[1]) {
      cudaFuncSetAttribute(gemm_i8_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
      attr_set[1] = true;
    }
    gemm_i8_kernel<true><<<grid, THREADS, SMEM_BYTES, stream>>>(tmap, p);
  } else {
    if (!attr_set[0]) {
      cudaFuncSetAttribute(gemm_i8_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
      attr_set[0] = true;
    }
    gemm_i8_kernel<false><<<grid, THREADS, SMEM_BYTES, stream>>>(tmap, p);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : CLEFQ_ERR_CUDA;
}

}  // namespace cq
