// clefq: Omni MoE routing operators for sm_100a.
//
//   route     kernels/omni_route.loom:84-147 with the serial semantics of
//             benches/kernels/omni_route_serial.loom: top-k by repeated strict '>' scans
//             in ascending expert id from (-3.402823466e38, id 0); p_j = exp(l_j - l_0)
//             summed in rank order, p_j / sum rounded to BF16.
//   group     kernels/omni_group_routes{,_ordered}.loom: per expert the route ids
//             t*topk + rank in ascending token order, and order[t][j] = the rank holding
//             the j-th smallest expert id.  Also the expert-sorted permutation, the
//             per-expert row offsets and the 128-row GEMM tile list used internally.
//   tasks     kernels/omni_expert_tasks.loom:30-61 (16-row task list, reference format).
//   combine   kernels/omni_combine_ordered.loom:51-79 / omni_combine.loom:40-72.
//   gather    rows of the s8 operand into expert-sorted order (internal).
#include "clefq_internal.h"
#include "cq_common.cuh"

namespace cq {

constexpr float NEG_MAX = -3.402823466e38f;

// One warp per token; lane l holds experts l, l+32, l+64, l+96.
__global__ void route_kernel(const void *__restrict__ logits, int is_f32, int64_t tokens, int experts, int topk,
                             float *__restrict__ routes) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= tokens) return;
  float v[4];
  bool used[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int e = lane + 32 * j;
    used[j] = e >= experts;
    v[j] = NEG_MAX;
    if (e < experts)
      v[j] = is_f32 ? static_cast<const float *>(logits)[t * experts + e]
                    : bf16_to_f32(static_cast<const uint16_t *>(logits)[t * experts + e]);
  }
  float *o = routes + t * 2 * topk;
  float my_val = 0.0f;  // lane r keeps the value selected at rank r
  for (int r = 0; r < topk; ++r) {
    float bv = NEG_MAX;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (!used[j] && v[j] > bv) {
        bv = v[j];
        bi = lane + 32 * j;
      }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (ov > bv || (!(ov < bv) && ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (bi == 0x7fffffff) {  // nothing above the floor: the serial scan keeps id 0
      bi = 0;
      bv = NEG_MAX;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (lane + 32 * j == bi) used[j] = true;
    if (lane == r) my_val = bv;
    if (lane == 0) o[r] = (float)bi;
  }
  const float mx = __shfl_sync(0xffffffffu, my_val, 0);
  const float p = exp_cw(__fsub_rn(my_val, mx));
  float sum = 0.0f;
  for (int j = 0; j < topk; ++j) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, p, j));
  if (lane < topk) o[topk + lane] = bf16r(__fdiv_rn(p, sum));
}

int launch_route(const void *logits, int is_f32, int64_t tokens, int experts, int topk, float *routes,
                 cudaStream_t stream) {
  if (tokens <= 0) return 0;
  const int warps = 8;
  route_kernel<<<(unsigned)((tokens + warps - 1) / warps), warps * 32, 0, stream>>>(logits, is_f32, tokens, experts,
                                                                                     topk, routes);
  return cudaGetLastError() == cudaSuccess ? 0 : CLEFQ_ERR_CUDA;
}

// Counts of routes per expert (ids read from the f32 route table).
__global__ void count_kernel(const float *__restrict__ routes, int64_t tokens, int topk, int experts,
                             int *__restrict__ counts) {
  const int64_t total = tokens * topk;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / topk;
    const int r = (int)(i % topk);
    const float *rt = routes + t * 2 * topk;
    const int e = (int)rt[r];
    // A token that repeats an expert id is grouped once, at its last matching rank, as
    // the fill pass does.
    bool last = true;
    for (int q = r + 1; q < topk; ++q) last = last && (int)rt[q] != e;
    if (last && e >= 0 && e < experts) atomicAdd(&counts[e], 1);
  }
}

// Single CTA: offsets (exclusive prefix), GEMM tile list (128-row tiles), and optionally
// the reference-format counts groups[e][0] and 16-row task list.
__global__ void scan_kernel(const int *__restrict__ counts, int experts, int64_t tokens, int tile_rows,
                            int *__restrict__ offsets, int *__restrict__ tile_list, float *__restrict__ groups,
                            float *__restrict__ tasks) {
  __shared__ int s_off[1025], s_tiles[1025], s_tasks[1025];
  const int e = threadIdx.x;
  const int c = e < experts ? counts[e] : 0;
  if (threadIdx.x == 0) {
    int run = 0, trun = 0, krun = 0;
    for (int i = 0; i < experts; ++i) {
      const int ci = counts[i];
      s_off[i] = run;
      s_tiles[i] = trun;
      s_tasks[i] = krun;
      run += ci;
      trun += (ci + tile_rows - 1) / tile_rows;
      krun += (ci + 15) / 16;
    }
    s_off[experts] = run;
    s_tiles[experts] = trun;
    s_tasks[experts] = krun;
  }
  __syncthreads();
  if (e < experts) {
    offsets[e] = s_off[e];
    for (int i = 0; i < (c + tile_rows - 1) / tile_rows; ++i) {
      tile_list[1 + 2 * (s_tiles[e] + i)] = e;
      tile_list[2 + 2 * (s_tiles[e] + i)] = s_off[e] + tile_rows * i;
    }
    if (groups) groups[(int64_t)e * (tokens + 1)] = (float)c;
    if (tasks) {
      for (int i = 0; i < (c + 15) / 16; ++i) {
        tasks[1 + 2 * (s_tasks[e] + i)] = (float)e;
        tasks[2 + 2 * (s_tasks[e] + i)] = (float)(16 * i);
      }
    }
  }
  if (threadIdx.x == 0) {
    offsets[experts] = s_off[experts];
    tile_list[0] = s_tiles[experts];
    if (tasks) tasks[0] = (float)s_tasks[experts];
  }
}

// One CTA (256 threads) per expert: stable compaction in token order.
__global__ void __launch_bounds__(256) fill_kernel(const float *__restrict__ routes, int64_t tokens, int topk,
                                                   const int *__restrict__ offsets, float *__restrict__ groups,
                                                   float *__restrict__ order, int *__restrict__ perm) {
  __shared__ int warp_tot[8];
  const int e = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int base = offsets[e];
  const float ef = (float)e;
  int count0 = 0;
  for (int64_t t0 = 0; t0 < tokens; t0 += 256) {
    const int64_t t = t0 + threadIdx.x;
    int rank = topk, less = 0;
    if (t < tokens) {
      const float *rt = routes + t * 2 * topk;
      for (int r = 0; r < topk; ++r) {
        const float id = rt[r];
        if ((int)id == e) rank = r;
        if (id < ef) ++less;
      }
    }
    const bool match = rank < topk;
    const unsigned ballot = __ballot_sync(0xffffffffu, match);
    const int in_warp = __popc(ballot & ((1u << lane) - 1u));
    if (lane == 0) warp_tot[warp] = __popc(ballot);
    __syncthreads();
    int before = 0, total = 0;
    for (int w = 0; w < 8; ++w) {
      const int n = warp_tot[w];
      if (w < warp) before += n;
      total += n;
    }
    if (match) {
      const int ordinal = count0 + before + in_warp;
      const int route = (int)(t * topk + rank);
      if (groups) groups[(int64_t)e * (tokens + 1) + 1 + ordinal] = (float)route;
      if (perm) perm[base + ordinal] = route;
      if (order) order[t * topk + less] = (float)rank;
    }
    count0 += total;
    __syncthreads();
  }
}

int launch_group(const float *routes, int64_t tokens, int topk, int experts, int tile_rows, int *counts, int *offsets,
                 int *tile_list, int *perm, float *groups, float *order, float *tasks, cudaStream_t stream,
                 int num_sms) {
  if (experts > 1024 || topk <= 0) return CLEFQ_ERR_SHAPE;
  cudaMemsetAsync(counts, 0, sizeof(int) * experts, stream);
  if (tokens > 0) {
    const int64_t total = tokens * topk;
    int64_t blocks = (total + 255) / 256, cap = (int64_t)num_sms * 8;
    count_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, stream>>>(routes, tokens, topk, experts, counts);
  }
  scan_kernel<<<1, experts <= 32 ? 32 : ((experts + 31) / 32) * 32, 0, stream>>>(counts, experts, tokens, tile_rows,
                                                                                 offsets, tile_list, groups, tasks);
  if (tokens > 0)
    fill_kernel<<<experts, 256, 0, stream>>>(routes, tokens, topk, offsets, groups, order, perm);
  return cudaGetLastError() == cudaSuccess ? 0 : CLEFQ_ERR_CUDA;
}

// Reference-format task list from a reference-format groups buffer (counts in groups[e][0]).
__global__ void tasks_kernel(const float *__restrict__ groups, int64_t tokens, int experts, float *__restrict__ tasks) {
  __shared__ int s_pref[1025];
  if (threadIdx.x == 0) {
    int run = 0;
    for (int e = 0; e < experts; ++e) {
      s_pref[e] = run;
      run += ((int)groups[(int64_t)e * (tokens + 1)] + 15) / 16;
    }
    s_pref[experts] = run;
    tasks[0] = (float)run;
  }
  __syncthreads();
  const int e = threadIdx.x;
  if (e < experts) {
    const int c = (int)groups[(int64_t)e * (tokens + 1)];
    for (int i = 0; i < (c + 15) / 16; ++i) {
      tasks[1 + 2 * (s_pref[e] + i)] = (float)e;
      tasks[2 + 2 * (s_pref[e] + i)] = (float)(16 * i);
    }
  }
}

int launch_tasks(const float *groups, int64_t tokens, int experts, float *tasks, cudaStream_t stream) {
  if (experts > 1024) return CLEFQ_ERR_SHAPE;
  tasks_kernel<<<1, ((experts + 31) / 32) * 32, 0, stream>>>(groups, tokens, experts, tasks);
  return cudaGetLastError() == cudaSuccess ? 0 : CLEFQ_ERR_CUDA;
}

// Sorted-layout tables from a reference-format groups buffer: offsets, perm, tile list.
__global__ void groups_to_sorted_kernel(const float *__restrict__ groups, int64_t tokens, int topk, int experts,
                                        int tile_rows, int *__restrict__ offsets, int *__restrict__ perm,
                                        int *__restrict__ tile_list) {
  const int cap = (int)(tokens * topk);
  __shared__ int s_off[1025], s_tiles[1025], s_cnt[1024];
  if (threadIdx.x == 0) {
    // Counts come from the caller: clamp each to [0, tokens] and the total to
    // tokens*topk so that no later index leaves its buffer.
    int run = 0, trun = 0;
    for (int e = 0; e < experts; ++e) {
      int c = (int)groups[(int64_t)e * (tokens + 1)];
      c = c < 0 ? 0 : (c > tokens ? (int)tokens : c);
      c = run + c > cap ? cap - run : c;
      s_cnt[e] = c;
      s_off[e] = run;
      s_tiles[e] = trun;
      run += c;
      trun += (c + tile_rows - 1) / tile_rows;
    }
    s_off[experts] = run;
    s_tiles[experts] = trun;
    tile_list[0] = trun;
    offsets[experts] = run;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < experts; e += blockDim.x) {
    const int c = s_cnt[e];
    offsets[e] = s_off[e];
    for (int i = 0; i < (c + tile_rows - 1) / tile_rows; ++i) {
      tile_list[1 + 2 * (s_tiles[e] + i)] = e;
      tile_list[2 + 2 * (s_tiles[e] + i)] = s_off[e] + tile_rows * i;
    }
  }
  __syncthreads();
  for (int e = 0; e < experts; ++e) {
    const int c = s_cnt[e];
    for (int i = threadIdx.x; i < c; i += blockDim.x) {
      int r = (int)groups[(int64_t)e * (tokens + 1) + 1 + i];
      perm[s_off[e] + i] = r < 0 ? 0 : (r >= cap ? cap - 1 : r);
    }
  }
}

int launch_groups_to_sorted(const float *groups, int64_t tokens, int topk, int experts, int tile_rows, int *offsets,
                            int *perm, int *tile_list, cudaStream_t stream) {
  if (experts > 1024) return CLEFQ_ERR_SHAPE;
  groups_to_sorted_kernel<<<1, 256, 0, stream>>>(groups, tokens, topk, experts, tile_rows, offsets, perm, tile_list);
  return cudaGetLastError() == cudaSuccess ? 0 : CLEFQ_ERR_CUDA;
}

// dst[p][:] = src[row(p)][:], row(p) = perm[p] / div (16-byte vectors).
__global__ void gather_rows_kernel(const uint8_t *__restrict__ src, int64_t src_ld, const int *__restrict__ perm,
                                   int div, int64_t rows, int64_t row_bytes, uint8_t *__restrict__ dst, int64_t dst_ld) {
  const int64_t v_per_row = row_bytes / 16;
  const int64_t total = rows * v_per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = i / v_per_row, v = i % v_per_row;
    const int64_t srow = perm[p] / div;
    reinterpret_cast<uint4 *>(dst + p * dst_ld)[v] = reinterpret_cast<const uint4 *>(src + srow * src_ld)[v];
  }
}

int launch_gather(const uint8_t *src, int64_t src_ld, const int *perm, int div, int64_t rows, int64_t row_bytes,
                  uint8_t *dst, int64_t dst_ld, cudaStream_t stream, int num_sms) {
  if (rows <= 0) return 0;
  if (row_bytes % 16 || src_ld % 16 || dst_ld % 16 || (uintptr_t)src % 16 || (uintptr_t)dst % 16) return CLEFQ_ERR_ALIGN;
  const int64_t total = rows * (row_bytes / 16);
  int64_t blocks = (total + 255) / 256, cap = (int64_t)num_sms * 16;
  gather_rows_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, stream>>>(src, src_ld, perm, div, rows,
                                                                                  row_bytes, dst, dst_ld);
  return cudaGetLastError() == cudaSuccess ? 0 : CLEFQ_ERR_CUDA;
}

// Weighted combine in ascending expert order with BF16 rounding at every step; eight
// columns per thread.  order == nullptr: find the ascending order per token like
// omni_combine.loom (prev/best scan).
__global__ void combine_kernel(const uint16_t *__restrict__ values, const float *__restrict__ routes,
                               const float *__restrict__ order, int64_t tokens, int topk, int64_t width,
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
      int r;
      if (order) {
        r = (int)order[t * topk + j];
        r = r < 0 ? 0 : (r >= topk ? topk - 1 : r);
      } else {
        float best = 1000000.0f;
        r = 0;
        for (int q = 0; q < topk; ++q) {
          const float e = rt[q];
          if (e > prev && e < best) {
            best = e;
            r = q;
          }
        }
        prev = best;
      }
      const float p = rt[topk + r];
      const uint4 raw = *reinterpret_cast<const uint4 *>(values + (t * topk + r) * width + c);
      const uint16_t *h = reinterpret_cast<const uint16_t *>(&raw);
#pragma unroll
      for (int q = 0; q < 8; ++q) s[q] = bf16r(__fadd_rn(s[q], bf16r(__fmul_rn(bf16_to_f32(h[q]), p))));
    }
    uint4 o;
    uint16_t *oh = reinterpret_cast<uint16_t *>(&o);
#pragma unroll
    for (int q = 0; q < 8; ++q) oh[q] = f32_to_bf16(s[q]);
    *reinterpret_cast<uint4 *>(out + t * width + c) = o;
  }
}

// Rounds two floats to BF16 with one cvt.rn.bf16x2 and widens them back to F32.
CQ_DEV void bf16r2_inplace(float &lo, float &hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  lo = __uint_as_float(r << 16);
  hi = __uint_as_float(r & 0xffff0000u);
}

// The same combine with topk fixed at compile time: the K route rows' 16-byte chunks are all
// loaded before the ordered chain consumes them, so a thread has K loads in flight instead
// of one.  Identical arithmetic and order to combine_kernel.
template <int K>
__global__ void combine_k_kernel(const uint16_t *__restrict__ values, const float *__restrict__ routes,
                                 const float *__restrict__ order, int64_t tokens, int64_t width,
                                 uint16_t *__restrict__ out) {
  const int64_t per_tok = width / 8;
  const int64_t total = tokens * per_tok;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / per_tok;
    const int64_t c = (i % per_tok) * 8;
    const float *rt = routes + t * 2 * K;
    int rank[K];
    if (order) {
#pragma unroll
      for (int j = 0; j < K; ++j) {
        const int r = (int)order[t * K + j];
        rank[j] = r < 0 ? 0 : (r >= K ? K - 1 : r);
      }
    } else {
      float prev = -1.0f;
#pragma unroll
      for (int j = 0; j < K; ++j) {
        float best = 1000000.0f;
        int r = 0;
#pragma unroll
        for (int q = 0; q < K; ++q) {
          const float e = rt[q];
          if (e > prev && e < best) {
            best = e;
            r = q;
          }
        }
        prev = best;
        rank[j] = r;
      }
    }
    uint4 raw[K];
#pragma unroll
    for (int j = 0; j < K; ++j) raw[j] = *reinterpret_cast<const uint4 *>(values + (t * K + rank[j]) * width + c);
    // s = bf16(s + bf16(v * p)) with both roundings done two lanes at a time by
    // cvt.rn.bf16x2 (round to nearest even, as f32_to_bf16 for every finite value and
    // for infinities; a NaN stays a NaN).
    float s[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) s[q] = 0.0f;
#pragma unroll
    for (int j = 0; j < K; ++j) {
      const float p = rt[K + rank[j]];
      const uint32_t *hw = reinterpret_cast<const uint32_t *>(&raw[j]);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float lo = __fmul_rn(__uint_as_float(hw[q] << 16), p);
        float hi = __fmul_rn(__uint_as_float(hw[q] & 0xffff0000u), p);
        bf16r2_inplace(lo, hi);
        lo = __fadd_rn(s[2 * q], lo);
        hi = __fadd_rn(s[2 * q + 1], hi);
        bf16r2_inplace(lo, hi);
        s[2 * q] = lo;
        s[2 * q + 1] = hi;
      }
    }
    uint4 o;
    uint32_t *ow = reinterpret_cast<uint32_t *>(&o);
#pragma unroll
    for (int q = 0; q < 4; ++q)  // the sums are BF16 values already: keep their top halves
      ow[q] = __byte_perm(__float_as_uint(s[2 * q]), __float_as_uint(s[2 * q + 1]), 0x7632);
    *reinterpret_cast<uint4 *>(out + t * width + c) = o;
  }
}

int launch_combine(const uint16_t *values, const float *routes, const float *order, int64_t tokens, int topk,
                   int64_t width, uint16_t *out, cudaStream_t stream, int num_sms) {
  if (width % 8) return CLEFQ_ERR_SHAPE;
  if ((uintptr_t)values % 16 || (uintptr_t)out % 16) return CLEFQ_ERR_ALIGN;
  const int64_t total = tokens * (width / 8);
  if (total == 0) return 0;
  int64_t blocks = (total + 255) / 256, cap = (int64_t)num_sms * 16;
  const unsigned grid = (unsigned)(blocks < cap ? blocks : cap);
  switch (topk) {
    case 8: combine_k_kernel<8><<<grid, 256, 0, stream>>>(values, routes, order, tokens, width, out); break;
    case 4: combine_k_kernel<4><<<grid, 256, 0, stream>>>(values, routes, order, tokens, width, out); break;
    case 2: combine_k_kernel<2><<<grid, 256, 0, stream>>>(values, routes, order, tokens, width, out); break;
    default: combine_kernel<<<grid, 256, 0, stream>>>(values, routes, order, tokens, topk, width, out); break;
  }
  return cudaGetLastError() == cudaSuccess ? 0 : CLEFQ_ERR_CUDA;
}


// dst[p][:] = s8 operand of packed int4 row perm[p] / div (unpack fused with the gather).
__global__ void gather_unpack_i4_kernel(const uint32_t *__restrict__ a, int64_t a_ld, const int *__restrict__ perm,
                                        int div, int64_t rows, int k, uint8_t *__restrict__ dst, int64_t dst_ld) {
  const int groups = k / 32;
  const int64_t total = rows * groups;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = i / groups;
    const int gq = (int)(i % groups);
    const uint32_t *src = a + (int64_t)(perm[p] / div) * a_ld + gq * 4;
    uint32_t w0, w1, w2, w3;
    if ((a_ld & 3) == 0) {
      const uint4 v = *reinterpret_cast<const uint4 *>(src);
      w0 = v.x; w1 = v.y; w2 = v.z; w3 = v.w;
    } else {
      w0 = src[0]; w1 = src[1]; w2 = src[2]; w3 = src[3];
    }
    uint4 *out = reinterpret_cast<uint4 *>(dst + p * dst_ld + gq * 32);
    out[0] = make_uint4(nib_lo16(w0), nib_lo16(w1), nib_lo16(w2), nib_lo16(w3));
    out[1] = make_uint4(nib_hi16(w0), nib_hi16(w1), nib_hi16(w2), nib_hi16(w3));
  }
}

int launch_gather_unpack_i4(const uint32_t *a, int64_t a_ld, const int *perm, int div, int64_t rows, int k,
                            uint8_t *dst, int64_t dst_ld, cudaStream_t stream, int num_sms) {
  const int64_t total = rows * (k / 32);
  if (total <= 0) return 0;
  if ((uintptr_t)dst % 16 || dst_ld % 16) return CLEFQ_ERR_ALIGN;
  int64_t blocks = (total + 255) / 256, cap = (int64_t)num_sms * 16;
  gather_unpack_i4_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, stream>>>(a, a_ld, perm, div, rows, k,
                                                                                       dst, dst_ld);
  return cudaGetLastError() == cudaSuccess ? 0 : CLEFQ_ERR_CUDA;
}

}  // namespace cq
