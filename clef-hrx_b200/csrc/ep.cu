// clefq: expert-parallel Omni MoE helpers (routes sharded over GPUs by expert id).
//
// The reference runs the MoE layer on one GPU (src/omni.rs:761-857); these kernels split
// it across ranks so that every rank keeps the experts [rank * E/G, (rank + 1) * E/G):
//
//   home rank:   route -> quantise each token once -> plan (one record per route, grouped
//                by destination rank, in route order) -> pack records
//   all-to-all:  records (int4 codes of the token, its f32 scale, expert id, probability)
//   remote rank: grouped expert GEMMs on the received records -> bf16(value * probability)
//   all-to-all:  per-route products back, in the order they were sent
//   home rank:   the reference's ascending-expert BF16 chain over the returned products
//
// Every step that rounds is the single-GPU step on the same operands (rows are quantised
// and multiplied independently; the chain runs on the home rank in the same order), so
// the result is bit-identical to one GPU.
#include "cq_common.cuh"
#include "clefq_internal.h"

namespace cq {

// Send slots: routes grouped by destination rank (expert / experts_per_rank), stable in
// route order (token-major, then rank k) -- the stable grouping of moe.cu with the rank as
// the key.  counts[d] = routes for rank d.
int launch_ep_plan(const float *routes, int64_t tokens, int topk, int experts, int world, long long *counts,
                   int *slots, int *scratch, cudaStream_t stream) {
  if (world < 1 || world > 64 || experts % world) return CLEFQ_ERR_SHAPE;
  SortArgs a{};
  a.routes = routes;
  a.route_ld = 2 * topk;
  a.tokens = tokens;
  a.topk = topk;
  a.items = tokens * topk;
  a.key_div = experts / world;
  a.keys = world;
  a.dedupe = false;  // one record per route
  a.hist = scratch;
  a.counts64 = counts;
  a.slots = slots;
  return launch_sort(a, stream);
}

// One warp per route: the token's packed code row (hidden/8 words), then scale, expert id
// and probability, at record slots[route] of the send buffer.
__global__ void ep_pack_kernel(const uint32_t *__restrict__ xq, int64_t words_ld, const float *__restrict__ scales,
                               const float *__restrict__ routes, const int *__restrict__ slots, int64_t tokens,
                               int topk, int code_words, int64_t rec_words, uint32_t *__restrict__ send) {
  const int lane = threadIdx.x & 31;
  const int64_t total = tokens * topk;
  const int64_t wstride = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t i = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); i < total; i += wstride) {
    const int64_t t = i / topk;
    const int r = (int)(i % topk);
    uint32_t *rec = send + (int64_t)slots[i] * rec_words;
    const uint32_t *src = xq + t * words_ld;
    for (int w = lane * 4; w < code_words; w += 128)
      *reinterpret_cast<uint4 *>(rec + w) = *reinterpret_cast<const uint4 *>(src + w);
    if (lane == 0) {
      rec[code_words] = __float_as_uint(scales[t]);
      rec[code_words + 1] = (uint32_t)(int)routes[t * 2 * topk + r];
      rec[code_words + 2] = __float_as_uint(routes[t * 2 * topk + topk + r]);
      rec[code_words + 3] = 0u;
    }
  }
}

int launch_ep_pack(const uint32_t *xq, int64_t words_ld, const float *scales, const float *routes, const int *slots,
                   int64_t tokens, int topk, int code_words, int64_t rec_words, uint32_t *send, cudaStream_t stream,
                   int num_sms) {
  const int64_t total = tokens * topk;
  if (total == 0) return 0;
  int64_t blocks = (total + 7) / 8, cap = (int64_t)num_sms * 16;
  ep_pack_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, stream>>>(xq, words_ld, scales, routes, slots,
                                                                              tokens, topk, code_words, rec_words, send);
  return launch_check();
}

// Received records -> contiguous activation scales and one-route-per-record routes
// (local expert id, probability) in the [rows][2] layout the grouping kernels read.
// Records whose expert is not local get id -1 and are left out of every group.
__global__ void ep_unpack_meta_kernel(const uint32_t *__restrict__ recv, int64_t n, int code_words, int64_t rec_words,
                                      int expert_base, int local_experts, float *__restrict__ scales,
                                      float *__restrict__ routes) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t *rec = recv + i * rec_words;
    const int e = (int)rec[code_words + 1] - expert_base;
    scales[i] = __uint_as_float(rec[code_words]);
    routes[2 * i] = (float)(e >= 0 && e < local_experts ? e : -1);
    routes[2 * i + 1] = __uint_as_float(rec[code_words + 2]);
  }
}

int launch_ep_unpack_meta(const uint32_t *recv, int64_t n, int code_words, int64_t rec_words, int expert_base,
                          int local_experts, float *scales, float *routes, cudaStream_t stream, int num_sms) {
  if (n == 0) return 0;
  int64_t blocks = (n + 255) / 256, cap = (int64_t)num_sms * 8;
  ep_unpack_meta_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, stream>>>(
      recv, n, code_words, rec_words, expert_base, local_experts, scales, routes);
  return launch_check();
}

// products[i] = bf16(bf16(values[i]) * probability of record i): the per-route term of the
// reference's combine (src/omni.rs:512-557), eight columns per thread.
__global__ void ep_weigh_kernel(const uint16_t *__restrict__ values, const float *__restrict__ routes, int64_t n,
                                int64_t width, uint16_t *__restrict__ products) {
  const int64_t per_row = width / 8;
  const int64_t total = n * per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / per_row;
    const int64_t c = (i % per_row) * 8;
    const float p = routes[2 * row + 1];
    const uint4 raw = *reinterpret_cast<const uint4 *>(values + row * width + c);
    const uint16_t *h = reinterpret_cast<const uint16_t *>(&raw);
    uint4 o;
    uint16_t *oh = reinterpret_cast<uint16_t *>(&o);
#pragma unroll
    for (int q = 0; q < 8; ++q) oh[q] = f32_to_bf16(__fmul_rn(bf16_to_f32(h[q]), p));
    *reinterpret_cast<uint4 *>(products + row * width + c) = o;
  }
}

int launch_ep_weigh(const uint16_t *values, const float *routes, int64_t n, int64_t width, uint16_t *products,
                    cudaStream_t stream, int num_sms) {
  const int64_t total = n * (width / 8);
  if (total == 0) return 0;
  int64_t blocks = (total + 255) / 256, cap = (int64_t)num_sms * 16;
  ep_weigh_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, stream>>>(values, routes, n, width, products);
  return launch_check();
}

// Home rank: out[t] = the ascending-expert chain s = bf16(s + product) over the token's
// routes, each product found at its send slot (the products come back in send order).
__global__ void ep_combine_kernel(const uint16_t *__restrict__ products, const int *__restrict__ slots,
                                  const float *__restrict__ routes, int64_t tokens, int topk, int64_t width,
                                  uint16_t *__restrict__ out) {
  const int64_t per_tok = width / 8;
  const int64_t total = tokens * per_tok;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / per_tok;
    const int64_t c = (i % per_tok) * 8;
    const float *rt = routes + t * 2 * topk;
    float s[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) s[q] = 0.0f;
    float prev = -1.0f;
    for (int j = 0; j < topk; ++j) {
      // next larger expert id (the reference's combine order; ids are distinct)
      float best = 1000000.0f;
      int r = 0;
      for (int q = 0; q < topk; ++q) {
        const float e = rt[q];
        if (e > prev && e < best) {
          best = e;
          r = q;
        }
      }
      prev = best;
      const uint4 raw = *reinterpret_cast<const uint4 *>(products + (int64_t)slots[t * topk + r] * width + c);
      const uint16_t *h = reinterpret_cast<const uint16_t *>(&raw);
#pragma unroll
      for (int q = 0; q < 8; ++q) s[q] = bf16r(__fadd_rn(s[q], bf16_to_f32(h[q])));
    }
    uint4 o;
    uint16_t *oh = reinterpret_cast<uint16_t *>(&o);
#pragma unroll
    for (int q = 0; q < 8; ++q) oh[q] = f32_to_bf16(s[q]);
    *reinterpret_cast<uint4 *>(out + t * width + c) = o;
  }
}

int launch_ep_combine(const uint16_t *products, const int *slots, const float *routes, int64_t tokens, int topk,
                      int64_t width, uint16_t *out, cudaStream_t stream, int num_sms) {
  const int64_t total = tokens * (width / 8);
  if (total == 0) return 0;
  int64_t blocks = (total + 255) / 256, cap = (int64_t)num_sms * 16;
  ep_combine_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, stream>>>(products, slots, routes, tokens, topk,
                                                                                 width, out);
  return launch_check();
}


// ---- fused expert parallelism over symmetric NVLink buffers ------------------------------
// counts: the G x G matrix in the symmetric region, row s = routes rank s sends to each rank
// (every row is complete once the first barrier of the layer has passed).

// One warp per route: the record goes straight into its destination rank's receive buffer:
// position = (records the lower ranks send to that rank) + (this route's place among the
// routes this rank sends there).  Record: code words, f32 scale, global expert id,
// probability, home route index t * topk + k.
__global__ void ep_dispatch_kernel(EpDispatchArgs a) {
  __shared__ int s_send[kMaxRanks], s_recv[kMaxRanks];
  if (threadIdx.x < (unsigned)a.world) {
    const int g = threadIdx.x;
    int so = 0, ro = 0;
    for (int d = 0; d < g; ++d) so += a.counts[a.rank * a.world + d];
    for (int src = 0; src < a.rank; ++src) ro += a.counts[src * a.world + g];
    s_send[g] = so;
    s_recv[g] = ro;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t total = a.tokens * a.topk;
  const int64_t wstride = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t i = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); i < total; i += wstride) {
    const int64_t t = i / a.topk;
    const int r = (int)(i % a.topk);
    const int e = (int)a.routes[t * 2 * a.topk + r];
    const int d = e >= 0 ? e / a.per_rank : a.world;
    if (d >= a.world) continue;
    const int64_t pos = (int64_t)s_recv[d] + (a.slots[i] - s_send[d]);
    if (pos < 0 || pos >= a.recv_cap) {
      if (lane == 0) atomicCAS(a.err, 0, kSiteEpCapacity);
      continue;
    }
    uint32_t *rec = a.recv[d] + pos * a.rec_words;
    const uint32_t *src = a.xq + t * a.words_ld;
    for (int w = lane * 4; w < a.code_words; w += 128)
      *reinterpret_cast<uint4 *>(rec + w) = *reinterpret_cast<const uint4 *>(src + w);
    if (lane == 0)
      *reinterpret_cast<uint4 *>(rec + a.code_words) =
          make_uint4(__float_as_uint(a.scales[t]), (uint32_t)e,
                     __float_as_uint(a.routes[t * 2 * a.topk + a.topk + r]), (uint32_t)i);
  }
  // every thread makes its own stores into peers visible at system scope before the kernel
  // ends; the barrier kernel's single-thread fence does not cover other threads' stores
  __threadfence_system();
}

// Received records -> per-record activation scale, (local expert, probability) route rows,
// and where the product goes back: home rank (from the record's position) and home route.
// n_dev = records received (the matrix column of this rank).
__global__ void ep_receive_kernel(EpReceiveArgs a) {
  __shared__ int s_off[kMaxRanks + 1];
  if (threadIdx.x == 0) {
    int run = 0;
    for (int src = 0; src < a.world; ++src) {
      s_off[src] = run;
      run += a.counts[src * a.world + a.rank];
    }
    s_off[a.world] = run;
    if (blockIdx.x == 0) {
      *a.n_dev = run < a.recv_cap ? run : a.recv_cap;
      if (run > a.recv_cap) atomicCAS(a.err, 0, kSiteEpCapacity);
    }
  }
  __syncthreads();
  const int64_t n = s_off[a.world] < a.recv_cap ? s_off[a.world] : a.recv_cap;
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < n; p += (int64_t)gridDim.x * blockDim.x) {
    const uint4 meta = *reinterpret_cast<const uint4 *>(a.recv + p * a.rec_words + a.code_words);
    const int e = (int)meta.y - a.expert_base;
    int src = 0;
    while (src + 1 < a.world && s_off[src + 1] <= p) ++src;
    a.scales[p] = __uint_as_float(meta.x);
    a.routes[2 * p] = (float)(e >= 0 && e < a.local_experts ? e : -1);
    a.routes[2 * p + 1] = __uint_as_float(meta.z);
    a.ret_prob[p] = __uint_as_float(meta.z);
    a.ret_rank[p] = src;
    a.ret_row[p] = (int)meta.w;
  }
}

// One warp per received route: its product row goes home scaled by the route's probability,
// bf16(value * prob), the same rounding as the single-GPU combine's product; 16-byte loads
// and stores, eight columns per lane and step.
__global__ void ep_return_kernel(EpReturnArgs a) {
  const int64_t d = *a.n_dev;
  const int64_t n = d < 0 ? 0 : (d < a.cap ? d : a.cap);
  const int lane = threadIdx.x & 31;
  const int chunks = a.hidden / 8;
  const int64_t wstride = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t p = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); p < n; p += wstride) {
    const float pr = a.prob[p];
    const uint4 *src = reinterpret_cast<const uint4 *>(a.values + p * a.hidden);
    uint4 *dst = reinterpret_cast<uint4 *>(a.base[a.rank[p]] + (int64_t)a.row[p] * a.hidden);
    for (int c = lane; c < chunks; c += 32) {
      uint4 v = __ldcs(src + c);
      uint16_t *h = reinterpret_cast<uint16_t *>(&v);
#pragma unroll
      for (int q = 0; q < 8; ++q) h[q] = f32_to_bf16(__fmul_rn(bf16_to_f32(h[q]), pr));
      dst[c] = v;
    }
  }
  // stores into peers are made visible at system scope before the kernel ends
  __threadfence_system();
}

int launch_ep_return(const EpReturnArgs &a, cudaStream_t stream, int num_sms) {
  if (a.cap <= 0) return 0;
  int64_t blocks = (a.cap + 7) / 8, cap = (int64_t)num_sms * 16;
  ep_return_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, stream>>>(a);
  return launch_check();
}

int launch_ep_dispatch(const EpDispatchArgs &a, cudaStream_t stream, int num_sms) {
  const int64_t total = a.tokens * a.topk;
  if (total == 0) return 0;
  int64_t blocks = (total + 7) / 8, cap = (int64_t)num_sms * 16;
  ep_dispatch_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, stream>>>(a);
  return launch_check();
}

int launch_ep_receive(const EpReceiveArgs &a, cudaStream_t stream, int num_sms) {
  int64_t blocks = (a.recv_cap + 255) / 256, cap = (int64_t)num_sms * 8;
  if (blocks < 1) blocks = 1;
  ep_receive_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, stream>>>(a);
  return launch_check();
}

}  // namespace cq
