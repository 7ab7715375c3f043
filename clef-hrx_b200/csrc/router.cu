// clefq: the Omni router linear fused with the router.
//
// The reference computes the router in two steps (src/omni.rs:760-765): a BF16 projection
// of the normalised hidden rows by `mlp.gate` (logits [tokens][experts], BF16, from a GEMM
// with f32 accumulation), then omni_route on those logits.  Here one kernel does both:
//   * a CTA owns 128 tokens; TMA streams their BF16 rows and the BF16 router weight in
//     K=64 slices (128-byte-swizzled boxes) through a 6-stage ring;
//   * one thread issues tcgen05.mma.kind::f16 (BF16 x BF16 -> F32, M=128 tokens, N=experts,
//     K=16) into a TMEM accumulator;
//   * the epilogue thread of token t owns TMEM lane t: it rounds each logit to BF16 (the
//     reference's projection output) and keeps a running top-k list while the columns stream
//     in, then applies the reference router's probabilities (exp relative to the top logit,
//     summed in rank order, BF16-rounded quotient).
// Selection semantics are the reference's repeated arg-max (kernels/omni_route.loom:84-147):
// only logits strictly above -FLT_MAX compete, equal logits rank by ascending expert id, and
// ranks left over once no candidate remains take expert 0 with logit -FLT_MAX.  The logits
// leave the chip only when the caller asks for them.  The f32 accumulation order is this
// kernel's, so logits can differ from another GEMM's by one BF16 rounding step; the routes
// are exactly omni_route of the logits this kernel reports.
#include <cuda.h>

#include <atomic>

#include "clefq_internal.h"
#include "cq_common.cuh"

namespace cq {

namespace {

constexpr float RT_NEG_MAX = -3.402823466e38f;
constexpr int RT_M = 128;                     // tokens per CTA: MMA M, TMEM lanes
constexpr int RT_KS = 64;                     // K elements per stage: one 128-byte row
constexpr int RT_NS = 6;                      // ring stages
constexpr int RT_THREADS = 128;               // warp 0: TMA, warp 1: MMA; all four: epilogue
constexpr int RT_X_BYTES = RT_M * RT_KS * 2;  // 16 KB token box
constexpr int RT_W_MAX = 128 * RT_KS * 2;     // 16 KB router-weight box (128 experts)
constexpr int RT_STAGE = RT_X_BYTES + RT_W_MAX;
constexpr int RT_SMEM = RT_NS * RT_STAGE + 1024 + 256;
constexpr int RT_TOPK = 8;                    // size of the running top list

struct RtSmem {
  uint64_t full[RT_NS], empty[RT_NS], acc_full;
  uint32_t tmem_base;
  int err;
};

struct RouterArgs {
  int64_t tokens;
  int hidden, experts, topk;
  float *routes;         // [tokens][2 * topk]
  uint16_t *logits_out;  // [tokens][experts] BF16, or null
  int *err;
};

// D[tmem] (+)= A[smem desc] x B[smem desc], kind::f16 (BF16 inputs, F32 accumulate), one CTA.
CQ_DEV void mma_bf16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor: kind::f16, D f32, A and B BF16, both K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// Inserts (x, id) into the list sorted by value descending, equal values by id ascending
// (ids arrive in ascending order, so a later equal value goes after the earlier one).
CQ_DEV void top_insert(float (&tv)[RT_TOPK], int (&ti)[RT_TOPK], float x, int id) {
  if (!(x > RT_NEG_MAX && x > tv[RT_TOPK - 1])) return;  // NaN and -inf never compete
#pragma unroll
  for (int q = RT_TOPK - 1; q >= 1; --q) {
    const bool shift = x > tv[q - 1];
    const bool here = !shift && x > tv[q];
    tv[q] = shift ? tv[q - 1] : (here ? x : tv[q]);
    ti[q] = shift ? ti[q - 1] : (here ? id : ti[q]);
  }
  if (x > tv[0]) {
    tv[0] = x;
    ti[0] = id;
  }
}

__global__ void __launch_bounds__(RT_THREADS, 1)
    route_linear_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                        RouterArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t *ring = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  RtSmem &s = *reinterpret_cast<RtSmem *>(ring + RT_NS * RT_STAGE);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row0 = (int64_t)blockIdx.x * RT_M;
  const int stages = a.hidden / RT_KS;
  const int E = a.experts;

  if (threadIdx.x == 0) {
    for (int i = 0; i < RT_NS; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    mbar_init(&s.acc_full, 1);
    s.err = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == 0 && lane == 0) {
    // ---- TMA producer: the CTA's token rows and the router weight, K=64 per stage ----
    tma_prefetch_desc(&xmap);
    tma_prefetch_desc(&wmap);
    const uint32_t bytes = RT_X_BYTES + (uint32_t)E * RT_KS * 2;
    for (int k = 0; k < stages; ++k) {
      const int st = k % RT_NS;
      if (!mbar_wait_bounded(&s.empty[st], ((k / RT_NS) & 1) ^ 1, &s.err, 1)) break;
      mbar_arrive_expect_tx(&s.full[st], bytes);
      tma_load_2d(ring + st * RT_STAGE, &xmap, &s.full[st], k * RT_KS, (int)row0);
      tma_load_2d(ring + st * RT_STAGE + RT_X_BYTES, &wmap, &s.full[st], k * RT_KS, 0);
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer: 4 x (M=128, N=E, K=16) per stage ----------------------------------
    const uint32_t idesc = idesc_bf16(RT_M, E);
    bool ok = true;
    for (int k = 0; k < stages; ++k) {
      const int st = k % RT_NS;
      if (!(ok = mbar_wait_bounded(&s.full[st], (k / RT_NS) & 1, &s.err, 2))) break;
      tc_fence_after();
      const uint32_t xa = smem_u32(ring + st * RT_STAGE), wa = xa + RT_X_BYTES;
#pragma unroll
      for (int j = 0; j < RT_KS / 16; ++j)
        mma_bf16_ss(tmem, smem_desc_sw128(xa + 32 * j), smem_desc_sw128(wa + 32 * j), idesc, (k | j) != 0);
      mma_commit(&s.empty[st]);
    }
    if (ok) mma_commit(&s.acc_full);
  }

  // ---- epilogue: the thread of TMEM lane t routes token row0 + t -----------------------
  bool have = true;
  if (lane == 0) have = mbar_wait_bounded(&s.acc_full, 0, &s.err, 3);
  have = __shfl_sync(0xffffffffu, have, 0) != 0;
  if (have) {
    tc_fence_after();
    const int64_t tok = row0 + warp * 32 + lane;
    const bool live = tok < a.tokens;
    float tv[RT_TOPK];
    int ti[RT_TOPK];
#pragma unroll
    for (int q = 0; q < RT_TOPK; ++q) {
      tv[q] = RT_NEG_MAX;
      ti[q] = 0;
    }
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    for (int c = 0; c < E; c += 32) {
      uint32_t v[32];
      tmem_ld_x32(tmem + lane_base + c, v);
      tmem_ld_wait(v);
      uint32_t packed[16];
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        // the reference's projection writes BF16 logits: round each f32 sum once (RNE)
        const uint16_t lo = f32_to_bf16(__uint_as_float(v[j]));
        const uint16_t hi = f32_to_bf16(__uint_as_float(v[j + 1]));
        packed[j / 2] = (uint32_t)lo | ((uint32_t)hi << 16);
        top_insert(tv, ti, bf16_to_f32(lo), c + j);
        top_insert(tv, ti, bf16_to_f32(hi), c + j + 1);
      }
      if (live && a.logits_out) {
        uint4 *dst = reinterpret_cast<uint4 *>(a.logits_out + tok * E + c);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          dst[q] = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
      }
    }
    if (live) {
      const int K = a.topk;
      float *o = a.routes + tok * 2 * K;
      const float mx = tv[0];
      float p[RT_TOPK];
      float sum = 0.0f;
#pragma unroll
      for (int r = 0; r < RT_TOPK; ++r) {
        p[r] = exp_cw(__fsub_rn(tv[r], mx));
        if (r < K) sum = __fadd_rn(sum, p[r]);
      }
#pragma unroll
      for (int r = 0; r < RT_TOPK; ++r) {
        if (r < K) {
          o[r] = (float)ti[r];
          o[K + r] = bf16r(__fdiv_rn(p[r], sum));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
  if (threadIdx.x == 0 && s.err) atomicCAS(a.err, 0, s.err);
}

using EncodeFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                              const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn router_encode_fn() {
  static const EncodeFn fn = [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeFn>(ptr);
    return static_cast<EncodeFn>(nullptr);
  }();
  return fn;
}

// BF16 [rows][cols] row-major, boxes of 64 columns x box_rows rows, 128-byte swizzle.
bool bf16_map(EncodeFn enc, CUtensorMap *m, const void *base, int64_t rows, int64_t cols, int box_rows) {
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

int launch_route_linear(const void *x, const void *w, int64_t tokens, int hidden, int experts, int topk, float *routes,
                        uint16_t *logits_out, int *err, cudaStream_t stream) {
  if (tokens == 0) return 0;
  EncodeFn enc = router_encode_fn();
  if (!enc) return CLEFQ_ERR_CUDA;
  CUtensorMap xmap, wmap;
  if (!bf16_map(enc, &xmap, x, tokens, hidden, RT_M) || !bf16_map(enc, &wmap, w, experts, hidden, experts))
    return CLEFQ_ERR_CUDA;
  static std::atomic<bool> attr_set[64];  // per device: the shared-memory limit is a per-context attribute
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(route_linear_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, RT_SMEM) != cudaSuccess)
      return launch_check();
    if (dev >= 0 && dev < 64) attr_set[dev].store(true, std::memory_order_release);
  }
  RouterArgs a{};
  a.tokens = tokens;
  a.hidden = hidden;
  a.experts = experts;
  a.topk = topk;
  a.routes = routes;
  a.logits_out = logits_out;
  a.err = err;
  const int64_t grid = (tokens + RT_M - 1) / RT_M;
  route_linear_kernel<<<(unsigned)grid, RT_THREADS, RT_SMEM, stream>>>(xmap, wmap, a);
  return launch_check();
}

}  // namespace cq
