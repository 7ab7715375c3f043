// clefq: internal launch interfaces shared by the .cu files (not part of the C ABI).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/clefq.h"

namespace cq {

constexpr int kMaxRanks = 8;              // ranks of a tensor-parallel group (one node)
constexpr int kMaxPeers = kMaxRanks - 1;  // extra store destinations of a fused collective
constexpr int kMaxDup = 8;                // operand rows one packed row can be written to

struct PrepareArgs {
  const uint16_t *x;
  int64_t x_ld;
  const uint16_t *aux;  // SwiGLU up [rows][aux_ld], attention q_gate [rows][aux_ld], norm weight [width]
  int64_t aux_ld;
  int64_t rows;
  int width;
  int stride;
  int bits;
  int mode;
  uint32_t *out;        // codes then scales
  uint8_t *op8;         // optional s8 operand [rows][op_ld] (int4 only)
  int64_t op_ld;
  uint16_t *norm_out;   // MODE_NORM_STORE: bf16 [rows][norm_ld]
  int64_t norm_ld;
  int team_warps;       // warps per row (set by launch_prepare)
  int rows_per_block;
  int stages;           // cp.async stages per thread (GEMM-input packing kernel)
  float *rowmax_out;    // if set: write each row's |Hadamard| maximum (NaN/inf -> +inf) only
  const float *rowmax_in;  // if set: quantise with this row maximum instead of the row's own
  // GEMM-input packing only: every code word (row, w) is also stored at
  // code_dst[d][row * code_ld + w], e.g. into the ranks' symmetric buffers over NVLink
  uint32_t *code_dst[kMaxRanks];
  int64_t code_ld;
  int n_code_dst;
  // GEMM-input packing only: when set, only the first *rows_dev rows (<= rows) are packed;
  // the storage layout still spans `rows`
  const int64_t *rows_dev;
  // plain int4 GEMM-input packing only: the s8 operand of input row r is stored at operand
  // rows dup_rows[r * dup + d] (d < dup <= kMaxDup; negative entries skipped) instead of row r
  const int *dup_rows;
  int dup;
  int narrow;           // set by the launcher: GEMM-input rows of 1..3 groups, one team per group
};
int launch_prepare(const PrepareArgs &a, cudaStream_t stream);
const uint16_t *silu_table_device();  // the BF16 SiLU table on the current device
int launch_swiglu(const uint16_t *g, const uint16_t *u, uint16_t *out, int64_t n, cudaStream_t stream, int num_sms);
int launch_silu(const uint16_t *x, uint16_t *out, int64_t n, cudaStream_t stream, int num_sms);
int launch_retile(const uint32_t *codes, int64_t rows, int64_t in_words, int64_t words, uint32_t *out,
                  cudaStream_t stream, int num_sms);
int launch_unpack_i4(const uint32_t *a, int64_t a_ld, int64_t rows, int k, uint8_t *op, int64_t op_ld,
                     cudaStream_t stream, int num_sms);

// Dense / grouped tcgen05 GEMM over an s8 token operand and tiled int4/int8 weights.
struct GemmParams {
  const uint8_t *a_op;      // s8 token operand [rows][a_ld bytes]
  int64_t a_rows;           // rows of the operand tensor (TMA bound)
  int64_t a_ld;             // bytes
  const float *a_scales;
  const uint32_t *w[2];     // tiled codes: one matrix, or two stacked along the output
  const float *w_scales[2]; //   columns (e.g. gate then up), each n_split*128 rows per expert
  int n_split;              // 128-row weight tiles per matrix per expert
  int64_t m;                // dense: token rows
  int n;                    // output columns (both matrices; per expert when grouped)
  int k;
  int bits;
  uint16_t *out;            // bf16 [.][ldo]
  float *out_f32;           // optional f32 output (dense)
  int64_t ldo;
  const uint16_t *residual; // optional bf16 residual [m][ldr] (dense)
  int64_t ldr;
  // grouped (MoE) mode
  int grouped;
  const int *tile_list;     // [1 + 2*max_tiles]: count, then (expert, sorted_row0)
  const int *expert_offsets;// [experts + 1] sorted-row offsets
  const int *perm;          // sorted position -> route id
  int max_tiles;
  int experts;              // experts whose weights are stacked in w[] (grouped)
  int tile_rows;            // token rows per tile-list entry (gemm_tile_rows)
  int topk;
  int scale_mode;           // a_scales index: 0 -> p, 1 -> perm[p] / topk, 2 -> perm[p]
  int scatter;              // output row: 1 -> perm[p], 0 -> p
  int *err;                 // device status word
  // dense 2-SM kernel only: every output row is also stored at these bases (same offsets
  // as from out), e.g. peers' symmetric buffers over NVLink
  uint16_t *out_peer[kMaxPeers];
  int n_out_peer;
  int store16;              // set by launch_gemm: every output address allows 16-byte stores
  // SwiGLU epilogue (int4, two weight maps: gate in w[0], up in w[1]; deep-ring kernel only):
  // each CTA computes 64 gate and the matching 64 up rows of one hidden-column slab and stores
  // bf16(bf16(silu(gate)) * up) -- the reference's SwiGLU of the two BF16 projections -- as
  // hidden [rows][ldo] BF16, n / 2 columns; silu_tab is the BF16 SiLU table of every input.
  int swiglu;
  const uint16_t *silu_tab;
};
int launch_gemm(const GemmParams &p, cudaStream_t stream);
bool gemm_swiglu_ok(int64_t n_each, int64_t k);  // the SwiGLU epilogue serves this gate|up shape
// Token rows per tile of the kernel launch_gemm picks for this output shape (grouped
// callers build their tile lists with it).
int gemm_tile_rows(int n, int n_split);

// Bump allocator over a caller workspace (256-byte aligned sections); with a null base it
// only measures.
struct Arena {
  uint8_t *base;
  int64_t cap, used = 0;
  bool ok = true;
  template <class T>
  T *take(int64_t count) {
    int64_t off = (used + 255) & ~int64_t(255);
    int64_t bytes = count * (int64_t)sizeof(T);
    if (off + bytes > cap) {
      ok = false;
      return nullptr;
    }
    used = off + bytes;
    return base ? reinterpret_cast<T *>(base + off) : nullptr;
  }
};
inline int64_t aligned_total(const Arena &a) { return (a.used + 255) & ~int64_t(255); }

// One rank's view of the symmetric regions of a node-local group (comm.cu).
constexpr int64_t kCommHeader = 4096;  // flags and the epoch counter precede the caller's bytes

struct CommBarrierArgs {
  uint32_t *flags;                  // this rank's flags[world]
  uint32_t *peer_flags[kMaxRanks];  // rank g's flags as mapped here (null for this rank)
  uint32_t *counter;                // this rank's epoch counter
  int rank, world;
  int64_t timeout_ns;
  const uint32_t *src;              // optional: `words` 4-byte words stored at dst[g] of every peer
  uint32_t *dst[kMaxRanks];
  int64_t words;
  const float *maxes;               // optional, after the wait: mx[i] = max_g maxes[g * m + i]
  float *mx;
  int64_t m;
  int *err;
};
int launch_comm_barrier(const CommBarrierArgs &a, cudaStream_t stream);

// Stable grouping of route items by key (moe.cu): item i = t * topk + r, key = (int)
// routes[t * route_ld + r] / key_div; ascending item order within each key.
constexpr int kSortChunksMax = 296;  // item chunks per sort (two per SM)
struct SortArgs {
  const float *routes;
  int64_t route_ld;          // floats per token row of routes
  int64_t tokens;            // token rows (the groups layout's row count)
  int topk;
  int64_t items;             // item bound (tokens * topk)
  const int64_t *items_dev;  // optional: actual item count on the device (<= items)
  int key_div, keys;
  bool dedupe;               // a token's repeated expert id is grouped once, at its last rank
  int chunk;                 // set by launch_sort
  int *hist;                 // scratch [sort_scratch_ints(keys)]
  int *counts;               // optional outputs
  long long *counts64;
  int *offsets;              // [keys + 1]
  int *tile_list;            // [1 + 2 * tiles]: count, then (key, first position) per tile
  int tile_rows;
  int *perm;                 // position -> item
  int *slots;                // item -> position
  float *groups;             // reference layout [keys][tokens + 1]
  float *order;              // [tokens][topk]
  float *tasks;              // reference 16-row task list
};
int64_t sort_scratch_ints(int keys);
int launch_sort(SortArgs a, cudaStream_t stream);

// Fused expert parallelism (ep.cu).
constexpr int kSiteEpCapacity = 9;  // status site: more records than the receive capacity
struct EpDispatchArgs {
  const uint32_t *xq;        // packed token rows [tokens][words_ld]
  int64_t words_ld;
  const float *scales;       // [tokens]
  const float *routes;       // [tokens][2 * topk]
  const int *slots;          // send slot per route (grouped by destination rank)
  int64_t tokens;
  int topk, per_rank;
  const int *counts;         // [world][world] in the symmetric region
  int rank, world;
  int code_words;
  int64_t rec_words;
  uint32_t *recv[kMaxRanks]; // every rank's receive buffer as mapped here
  int64_t recv_cap;          // records each receive buffer holds
  int *err;
};
struct EpReceiveArgs {
  const uint32_t *recv;      // this rank's receive buffer
  const int *counts;         // [world][world]
  int rank, world;
  int code_words;
  int64_t rec_words, recv_cap;
  int expert_base, local_experts;
  float *scales, *routes;    // [cap], [cap][2]
  int *ret_rank, *ret_row;
  float *ret_prob;
  int64_t *n_dev;
  int *err;
};
int launch_ep_dispatch(const EpDispatchArgs &a, cudaStream_t stream, int num_sms);
// Expert-parallel return: product row p (p < *n_dev) of values [cap][hidden] goes home as
// bf16(value * prob[p]) to base[rank[p]] + row[p] * hidden (a peer's buffer over NVLink).
struct EpReturnArgs {
  const uint16_t *values;
  const int64_t *n_dev;
  int64_t cap;
  int hidden;
  const int *rank, *row;
  const float *prob;
  uint16_t *base[kMaxRanks];
};
int launch_ep_return(const EpReturnArgs &a, cudaStream_t stream, int num_sms);
int launch_ep_receive(const EpReceiveArgs &a, cudaStream_t stream, int num_sms);

int device_sms();
int report_error(int code, const char *msg);  // sets clefq_last_error()
// After a kernel launch: 0, or CLEFQ_ERR_CUDA with CUDA's error kept for this thread, so
// the caller's message (last_launch_error) can name it although the error state is cleared.
int launch_check();
cudaError_t last_launch_error();
int *device_status_word();  // per-device zero-initialised status word used by bounded waits

}  // namespace cq

struct clefq_comm {
  int rank, world, device;
  int64_t bytes;                      // caller bytes of every region (after the header)
  uint8_t *base;                      // this rank's region
  uint8_t *peer[cq::kMaxRanks];       // every rank's region as mapped here (peer[rank] = base)
  bool opened[cq::kMaxRanks];         // peer[g] was opened from an IPC handle
  int64_t timeout_ns;                 // bound of each barrier wait
};

namespace cq {
CommBarrierArgs comm_barrier_args(clefq_comm *c, int *err);
}  // namespace cq
