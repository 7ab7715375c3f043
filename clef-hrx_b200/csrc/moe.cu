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
  return launch_check();
}

// ---- stable grouping: a three-phase counting sort of route items by key ----------------
// Item i = t * topk + r is route r of token t; its key is expert / key_div (an expert id,
// or the rank owning it).  With dedupe, a token that repeats an expert id is grouped once,
// at its last matching rank.  The items of each key keep ascending item order, which is the
// reference's ascending route order within each expert group.
//   hist:    one CTA per chunk of items: per-key counts of the chunk
//   scan:    one CTA: per-key totals, offsets, tile list; each chunk's base per key
//   scatter: one CTA per chunk: stable positions (per-warp sub-ranges in order, lanes of one
//            key ranked with match.any), written as perm / slots / groups / order
CQ_DEV int64_t sort_items(const SortArgs &a) {
  if (!a.items_dev) return a.items;
  const int64_t n = *a.items_dev;
  return n < a.items ? (n > 0 ? n : 0) : a.items;
}

CQ_DEV int item_key(const SortArgs &a, int64_t i) {
  const int64_t t = i / a.topk;
  const int r = (int)(i % a.topk);
  const float *rt = a.routes + t * a.route_ld;
  const int e = (int)rt[r];
  if (a.dedupe)
    for (int q = r + 1; q < a.topk; ++q)
      if ((int)rt[q] == e) return -1;
  if (e < 0) return -1;
  const int k = e / a.key_div;
  return k < a.keys ? k : -1;
}

__global__ void __launch_bounds__(256) sort_hist_kernel(SortArgs a) {
  extern __shared__ int sh_count[];
  for (int k = threadIdx.x; k < a.keys; k += blockDim.x) sh_count[k] = 0;
  __syncthreads();
  const int64_t n = sort_items(a);
  const int64_t lo = (int64_t)blockIdx.x * a.chunk;
  const int64_t hi = lo + a.chunk < n ? lo + a.chunk : n;
  for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const int k = item_key(a, i);
    if (k >= 0) atomicAdd(&sh_count[k], 1);
  }
  __syncthreads();
  for (int k = threadIdx.x; k < a.keys; k += blockDim.x) a.hist[(int64_t)k * gridDim.x + blockIdx.x] = sh_count[k];
}

// Exclusive block-wide prefix sum of one value per thread (1024 threads at most); returns
// (prefix, block total).
CQ_DEV int2 block_exclusive_scan(int v, int *warp_sums) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = (blockDim.x + 31) >> 5;
  int x = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, off);
    if (lane >= off) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nwarps ? warp_sums[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, off);
      if (lane >= off) w += y;
    }
    warp_sums[lane] = w;  // inclusive prefix over warps
  }
  __syncthreads();
  const int total = warp_sums[nwarps - 1];
  const int before = warp == 0 ? 0 : warp_sums[warp - 1];
  __syncthreads();
  return make_int2(before + x - v, total);
}

// hist is key-major ([keys][chunks]).  Warps sum each key's chunk counts, each thread scans
// two adjacent keys (2t and 2t+1), and warps turn each key's chunk counts into the chunks'
// first positions; every warp issues its loads of a key at once (chunks <= 320).
constexpr int kSortChunkRegs = (kSortChunksMax + 31) / 32;
__global__ void __launch_bounds__(512, 1) sort_scan_kernel(const __grid_constant__ SortArgs a, int chunks) {
  __shared__ int warp_sums[32];
  __shared__ int s_key[1024];  // per-key totals, then offsets
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  for (int e = warp; e < a.keys; e += nwarps) {
    const int *h = a.hist + (int64_t)e * chunks;
    int c = 0;
#pragma unroll
    for (int j = 0; j < kSortChunkRegs; ++j) {
      const int q = lane + 32 * j;
      if (q < chunks) c += h[q];
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) c += __shfl_xor_sync(0xffffffffu, c, off);
    if (lane == 0) s_key[e] = c;
  }
  __syncthreads();
  const int e0 = 2 * threadIdx.x;
  int c[2], off[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) c[j] = e0 + j < a.keys ? s_key[e0 + j] : 0;
  const int2 r0 = block_exclusive_scan(c[0] + c[1], warp_sums);
  off[0] = r0.x;
  off[1] = off[0] + c[0];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int e = e0 + j;
    if (e >= a.keys) continue;
    if (a.counts) a.counts[e] = c[j];
    if (a.counts64) a.counts64[e] = c[j];
    if (a.offsets) a.offsets[e] = off[j];
    if (a.groups) a.groups[(int64_t)e * (a.tokens + 1)] = (float)c[j];
    s_key[e] = off[j];
  }
  if (threadIdx.x == 0 && a.offsets) a.offsets[a.keys] = r0.y;
  if (a.tile_list) {
    const int t0 = (c[0] + a.tile_rows - 1) / a.tile_rows, t1 = (c[1] + a.tile_rows - 1) / a.tile_rows;
    const int2 r = block_exclusive_scan(t0 + t1, warp_sums);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int n = j ? t1 : t0, base = j ? r.x + t0 : r.x;
      for (int i = 0; i < n; ++i) {
        a.tile_list[1 + 2 * (base + i)] = e0 + j;
        a.tile_list[2 + 2 * (base + i)] = off[j] + a.tile_rows * i;
      }
    }
    if (threadIdx.x == 0) a.tile_list[0] = r.y;
  }
  if (a.tasks) {
    const int k0 = (c[0] + 15) / 16, k1 = (c[1] + 15) / 16;
    const int2 r = block_exclusive_scan(k0 + k1, warp_sums);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int n = j ? k1 : k0, base = j ? r.x + k0 : r.x;
      for (int i = 0; i < n; ++i) {
        a.tasks[1 + 2 * (base + i)] = (float)(e0 + j);
        a.tasks[2 + 2 * (base + i)] = (float)(16 * i);
      }
    }
    if (threadIdx.x == 0) a.tasks[0] = (float)r.y;
  }
  __syncthreads();
  // hist[e][q] := first position of key e's items in chunk q
  for (int e = warp; e < a.keys; e += nwarps) {
    int *h = a.hist + (int64_t)e * chunks;
    int v[kSortChunkRegs];
#pragma unroll
    for (int j = 0; j < kSortChunkRegs; ++j) {
      const int q = lane + 32 * j;
      v[j] = q < chunks ? h[q] : 0;
    }
    int carry = s_key[e];
#pragma unroll
    for (int j = 0; j < kSortChunkRegs; ++j) {
      int x = v[j];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      const int q = lane + 32 * j;
      if (q < chunks) h[q] = carry + x - v[j];
      carry += __shfl_sync(0xffffffffu, x, 31);
    }
  }
}

__global__ void __launch_bounds__(256) sort_scatter_kernel(SortArgs a) {
  extern __shared__ int sh_base[];  // [8 warps][keys]: next position per key for each warp
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int j = threadIdx.x; j < 8 * a.keys; j += blockDim.x) sh_base[j] = 0;
  __syncthreads();
  const int64_t n = sort_items(a);
  const int64_t lo = (int64_t)blockIdx.x * a.chunk;
  const int64_t hi = lo + a.chunk < n ? lo + a.chunk : n;
  const int per_warp = a.chunk / 8;
  const int64_t wlo = lo + (int64_t)warp * per_warp;
  const int64_t whi = wlo + per_warp < hi ? wlo + per_warp : hi;
  int *mine = sh_base + warp * a.keys;
  for (int64_t i = wlo + lane; i < whi; i += 32) {
    const int k = item_key(a, i);
    if (k >= 0) atomicAdd(&mine[k], 1);
  }
  __syncthreads();
  for (int k = threadIdx.x; k < a.keys; k += blockDim.x) {
    int run = a.hist[(int64_t)k * gridDim.x + blockIdx.x];
    for (int w = 0; w < 8; ++w) {
      const int c = sh_base[w * a.keys + k];
      sh_base[w * a.keys + k] = run;
      run += c;
    }
  }
  __syncthreads();
  const unsigned lt = (1u << lane) - 1u;
  for (int64_t i0 = wlo; i0 < whi; i0 += 32) {
    const int64_t i = i0 + lane;
    const int k = i < whi ? item_key(a, i) : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, k);
    const int rank = __popc(peers & lt);
    const int pos = k >= 0 ? mine[k] + rank : -1;
    __syncwarp();
    if (k >= 0 && rank == 0) mine[k] += __popc(peers);
    __syncwarp();
    if (k < 0) continue;
    if (a.perm) a.perm[pos] = (int)i;
    if (a.slots) a.slots[i] = pos;
    if (a.groups) a.groups[(int64_t)k * (a.tokens + 1) + 1 + (pos - a.offsets[k])] = (float)i;
    if (a.order) {
      // order[t][j] = the rank holding the token's j-th smallest expert id
      const int64_t t = i / a.topk;
      const float *rt = a.routes + t * a.route_ld;
      const float id = rt[i % a.topk];
      int less = 0;
      for (int q = 0; q < a.topk; ++q) less += rt[q] < id;
      a.order[t * a.topk + less] = (float)(i % a.topk);
    }
  }
}

int64_t sort_scratch_ints(int keys) { return (int64_t)kSortChunksMax * keys; }

int launch_sort(SortArgs a, cudaStream_t stream) {
  if (a.keys < 1 || a.keys > 1024 || a.topk < 1 || a.key_div < 1 || !a.hist) return CLEFQ_ERR_SHAPE;
  // chunks of whole 256-item rounds, at most kSortChunksMax of them
  int64_t chunk = (a.items + kSortChunksMax - 1) / kSortChunksMax;
  chunk = ((chunk + 255) / 256) * 256;
  if (chunk < 256) chunk = 256;
  if (chunk > 0x7fffffff) return CLEFQ_ERR_SHAPE;
  a.chunk = (int)chunk;
  const int chunks = a.items > 0 ? (int)((a.items + chunk - 1) / chunk) : 0;
  if (chunks > 0)
    sort_hist_kernel<<<chunks, 256, sizeof(int) * a.keys, stream>>>(a);
  sort_scan_kernel<<<1, 512, 0, stream>>>(a, chunks);
  if (chunks > 0)
    sort_scatter_kernel<<<chunks, 256, sizeof(int) * 8 * a.keys, stream>>>(a);
  return launch_check();
}

int launch_group(const float *routes, int64_t tokens, int topk, int experts, int tile_rows, int *counts, int *offsets,
                 int *tile_list, int *perm, float *groups, float *order, float *tasks, cudaStream_t stream,
                 int num_sms) {
  (void)num_sms;
  if (experts > 1024 || topk <= 0) return CLEFQ_ERR_SHAPE;
  SortArgs a{};
  a.routes = routes;
  a.route_ld = 2 * topk;
  a.tokens = tokens;
  a.topk = topk;
  a.items = tokens * topk;
  a.key_div = 1;
  a.keys = experts;
  a.dedupe = true;
  a.hist = counts + experts;
  a.counts = counts;
  a.offsets = offsets;
  a.tile_list = tile_list;
  a.tile_rows = tile_rows;
  a.perm = perm;
  a.groups = groups;
  a.order = order;
  a.tasks = tasks;
  return launch_sort(a, stream);
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
  return launch_check();
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
  return launch_check();
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
  return launch_check();
}

// Weighted combine in ascending expert order with BF16 rounding at every step; eight
// columns per thread.  order == nullptr: find the ascending order per token like
// omni_combine.loom (prev/best scan).
// weighted: values already hold bf16(v * p) (the expert-parallel products), so only the
// chain's additions remain.
__global__ void combine_kernel(const uint16_t *__restrict__ values, const float *__restrict__ routes,
                               const float *__restrict__ order, int64_t tokens, int topk, int64_t width,
                               uint16_t *__restrict__ out, bool weighted) {
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
      for (int q = 0; q < 8; ++q)
        s[q] = bf16r(__fadd_rn(s[q], weighted ? bf16_to_f32(h[q]) : bf16r(__fmul_rn(bf16_to_f32(h[q]), p))));
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
// loaded before the ordered chain consumes them, so a thread has K x CPT / 8 loads in flight
// instead of one.  CPT = 16 columns per thread (two chunks per route row) when the width
// allows it.  The route rows are read once, so their loads stream past the caches (ld.cs);
// measured on the C4 combine this took 62.5 -> 55.6 us.  Identical arithmetic and order to
// combine_kernel.
template <int K, bool WEIGHTED, int CPT>
__global__ void combine_k_kernel(const uint16_t *__restrict__ values, const float *__restrict__ routes,
                                 const float *__restrict__ order, int64_t tokens, int64_t width,
                                 uint16_t *__restrict__ out) {
  constexpr int NV = CPT / 8;  // 16-byte chunks per route row and thread
  const int64_t per_tok = width / CPT;
  const int64_t total = tokens * per_tok;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / per_tok;
    const int64_t c = (i % per_tok) * CPT;
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
    uint4 raw[K][NV];
#pragma unroll
    for (int j = 0; j < K; ++j)
#pragma unroll
      for (int v = 0; v < NV; ++v)
        raw[j][v] = __ldcs(reinterpret_cast<const uint4 *>(values + (t * K + rank[j]) * width + c + 8 * v));
    // s = bf16(s + bf16(v * p)) with both roundings done two lanes at a time by
    // cvt.rn.bf16x2 (round to nearest even, as f32_to_bf16 for every finite value and
    // for infinities; a NaN stays a NaN).
    float s[CPT];
#pragma unroll
    for (int q = 0; q < CPT; ++q) s[q] = 0.0f;
#pragma unroll
    for (int j = 0; j < K; ++j) {
      const float p = rt[K + rank[j]];
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        const uint32_t *hw = reinterpret_cast<const uint32_t *>(&raw[j][v]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float lo = __uint_as_float(hw[q] << 16);
          float hi = __uint_as_float(hw[q] & 0xffff0000u);
          if (!WEIGHTED) {
            lo = __fmul_rn(lo, p);
            hi = __fmul_rn(hi, p);
            bf16r2_inplace(lo, hi);
          }
          float &s0 = s[8 * v + 2 * q], &s1 = s[8 * v + 2 * q + 1];
          lo = __fadd_rn(s0, lo);
          hi = __fadd_rn(s1, hi);
          bf16r2_inplace(lo, hi);
          s0 = lo;
          s1 = hi;
        }
      }
    }
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      uint4 o;
      uint32_t *ow = reinterpret_cast<uint32_t *>(&o);
#pragma unroll
      for (int q = 0; q < 4; ++q)  // the sums are BF16 values already: keep their top halves
        ow[q] = __byte_perm(__float_as_uint(s[8 * v + 2 * q]), __float_as_uint(s[8 * v + 2 * q + 1]), 0x7632);
      *reinterpret_cast<uint4 *>(out + t * width + c + 8 * v) = o;
    }
  }
}

int launch_combine(const uint16_t *values, const float *routes, const float *order, int64_t tokens, int topk,
                   int64_t width, uint16_t *out, cudaStream_t stream, int num_sms, bool weighted) {
  if (width % 8) return CLEFQ_ERR_SHAPE;
  if ((uintptr_t)values % 16 || (uintptr_t)out % 16) return CLEFQ_ERR_ALIGN;
  const int64_t total = tokens * (width / 8);
  if (total == 0) return 0;
  int64_t blocks = (total + 255) / 256, cap = (int64_t)num_sms * 16;
  const unsigned grid = (unsigned)(blocks < cap ? blocks : cap);
  if (topk == 8 && width % 16 == 0) {
    // 16 columns per thread, 128 threads per block, one block per 2048 columns of a token
    const int64_t b16 = (tokens * (width / 16) + 127) / 128, cap16 = (int64_t)num_sms * 64;
    const unsigned g16 = (unsigned)(b16 < cap16 ? b16 : cap16);
    if (weighted) combine_k_kernel<8, true, 16><<<g16, 128, 0, stream>>>(values, routes, order, tokens, width, out);
    else combine_k_kernel<8, false, 16><<<g16, 128, 0, stream>>>(values, routes, order, tokens, width, out);
    return launch_check();
  }
#define CQ_COMBINE_K(K)                                                                            \
  (weighted ? combine_k_kernel<K, true, 8><<<grid, 256, 0, stream>>>(values, routes, order, tokens, width, out) \
            : combine_k_kernel<K, false, 8><<<grid, 256, 0, stream>>>(values, routes, order, tokens, width, out))
  switch (topk) {
    case 8: CQ_COMBINE_K(8); break;
    case 4: CQ_COMBINE_K(4); break;
    case 2: CQ_COMBINE_K(2); break;
    default: combine_kernel<<<grid, 256, 0, stream>>>(values, routes, order, tokens, topk, width, out, weighted); break;
  }
#undef CQ_COMBINE_K
  return launch_check();
}


// dst[p][:] = s8 operand of packed int4 row perm[p] / div (unpack fused with the gather).
__global__ void gather_unpack_i4_kernel(const uint32_t *__restrict__ a, int64_t a_ld, const int *__restrict__ perm,
                                        int div, int64_t rows, const int64_t *rows_dev, int k,
                                        uint8_t *__restrict__ dst, int64_t dst_ld) {
  const int groups = k / 32;
  if (rows_dev) {
    const int64_t d = *rows_dev;
    rows = d < 0 ? 0 : (d < rows ? d : rows);
  }
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
                            uint8_t *dst, int64_t dst_ld, cudaStream_t stream, int num_sms, const int64_t *rows_dev) {
  const int64_t total = rows * (k / 32);
  if (total <= 0) return 0;
  if ((uintptr_t)dst % 16 || dst_ld % 16) return CLEFQ_ERR_ALIGN;
  int64_t blocks = (total + 255) / 256, cap = (int64_t)num_sms * 16;
  gather_unpack_i4_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, stream>>>(a, a_ld, perm, div, rows,
                                                                                       rows_dev, k, dst, dst_ld);
  return launch_check();
}

}  // namespace cq
