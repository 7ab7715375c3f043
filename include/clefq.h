/*
 * clefq -- C ABI of the B200 (sm_100a) implementation of clef-hrx's INT4 quantized
 * matmul path: activation/weight packing, the dense INT4 GEMM and SwiGLU MLP, and the
 * Omni MoE expert pipeline (route, group, grouped expert GEMMs, combine).
 *
 * Conventions (all entry points):
 *   - Every call is asynchronous and stream-ordered on `stream` (a cudaStream_t; NULL is
 *     the legacy default stream).  Buffers are caller-owned DEVICE pointers; no entry
 *     point allocates device memory (the status word of clefq_status is a static
 *     __device__ variable of the library).
 *   - Calls that need scratch take a caller-provided `workspace` and have a
 *     *_workspace_size query.
 *   - Return value: CLEFQ_OK (0) or a negative clefq_status_t.  Shape checks mirror the
 *     reference's `ensure!` conditions; clefq_last_error() describes the last failure of
 *     the calling thread.
 *   - Layouts are the reference's: BF16 as uint16 bit patterns; packed codes + scales in
 *     one buffer (codes[rows][stride/P] u32, then f32 scales[rows]); weights in
 *     128-row x 32-word tiles; routes/groups/order/tasks as f32 index buffers.
 *   - Calls are reentrant on different streams.
 *
 * Reference citations are paths within the clef-hrx project.
 */
#ifndef CLEFQ_H
#define CLEFQ_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CLEFQ_API __attribute__((visibility("default")))

typedef enum {
  CLEFQ_OK = 0,
  CLEFQ_ERR_SHAPE = -1,   /* a shape/dtype/argument check failed (reference: ensure!) */
  CLEFQ_ERR_ALIGN = -2,   /* a pointer or pitch is not 16-byte aligned */
  CLEFQ_ERR_CUDA = -3,    /* a CUDA launch or runtime call failed */
  CLEFQ_ERR_NCCL = -4,    /* a collective failed */
  CLEFQ_ERR_TIMEOUT = -5, /* a bounded device-side wait gave up (see clefq_status) */
  CLEFQ_ERR_WORKSPACE = -6 /* workspace missing or too small */
} clefq_status_t;

/* Packing pre-ops (src/quantized.rs:574-776; kernels/prepare_integer_register.loom). */
typedef enum {
  CLEFQ_PREP_PLAIN = 0,     /* h3_prepare_plain_tiled_i{4,8} */
  CLEFQ_PREP_SWIGLU = 1,    /* h3_prepare_swiglu_i*: x = gate, aux = up (same shape) */
  CLEFQ_PREP_ATTN_GATE = 2, /* h3_prepare_attention_gate_i*: aux = q_gate [rows][2*width] */
  CLEFQ_PREP_NORM = 3,      /* h3_prepare_norm_i*: aux = RMSNorm weight [width], +1 offset, eps 1e-6 */
  CLEFQ_PREP_NORM_STORE = 4 /* h3_prepare_norm_store_i*: also writes the BF16 normalized rows */
} clefq_prep_kind_t;

typedef enum {
  CLEFQ_BF16 = 0,
  CLEFQ_F32 = 1,
  /* MoE blocks only (clefq_moe, clefq_moe_ep_layer): the `logits` argument is the router weight
   * BF16 [experts][hidden]; the blocks then route with clefq_route_linear's fused kernel on x */
  CLEFQ_ROUTER_WEIGHT_BF16 = 2
} clefq_dtype_t;

CLEFQ_API const char *clefq_last_error(void);
CLEFQ_API int clefq_version(void);

/*
 * Synchronizes `stream`, then reads and clears this device's status word, which the
 * tcgen05 kernels set when a bounded wait gives up.  Returns CLEFQ_OK or
 * CLEFQ_ERR_TIMEOUT (or CLEFQ_ERR_CUDA if the stream itself failed).
 */
CLEFQ_API int clefq_status(void *stream);

/*
 * Rotate (Hadamard-256) and quantize rows; replaces prepare / prepare_with_source /
 * prepare_with_inputs / prepare_attention_gate_with_source / prepare_norm*_with_source
 * (src/quantized.rs:574-776) and their kernels (kernels/prepare_integer*.loom).
 *   x        BF16 [rows][x_ld]          (width used)
 *   aux      see clefq_prep_kind_t      (aux_ld in elements)
 *   out      u32 codes[rows][stride/P] then f32 scales[rows]   (P = 32/bits)
 *   operand  optional s8 GEMM operand [rows][operand_ld bytes] of the same codes
 *            (bits 4 only; the tcgen05 GEMM's input format, 16*code, K-permuted)
 *   norm_out BF16 [rows][norm_ld] normalized rows (CLEFQ_PREP_NORM_STORE only)
 * Checks (src/quantized.rs:621-640): bits 4|8; 256 <= width <= 32768, width % 256 == 0;
 * 1 <= rows <= 1048576; width <= stride <= 65536, stride % (512/bits) == 0.
 * The RMSNorm pre-op accepts any width (the reference fixes 5120 and divides by 5120).
 */
CLEFQ_API int clefq_prepare(void *stream, int kind, int bits, const void *x, int64_t x_ld, const void *aux,
                            int64_t aux_ld, int64_t rows, int64_t width, int64_t stride, void *out, void *operand,
                            int64_t operand_ld, void *norm_out, int64_t norm_ld);

/*
 * Permute packed weight words into 128-row x 32-word blocks, dropping stride padding;
 * replaces retile_codes (src/quantized.rs:542-572, kernels/retile_codes.loom).
 *   codes u32 [rows][in_words] -> out u32 [rows * cols / (32/bits)] tiled.
 * Checks: rows % 128 == 0, (cols/(32/bits)) % 32 == 0, in_words >= cols/(32/bits).
 */
CLEFQ_API int clefq_retile(void *stream, const void *codes, int64_t rows, int64_t cols, int bits, int64_t in_words,
                           void *out);

/*
 * Weight loading (src/quantized.rs:147-234 load_quantized_weight, after its precision policy):
 * BF16 [rows][cols] -> prepare with stride cols (+512/bits when cols % 1024 == 0) -> retile.
 * tiled != 0: src is in the checkpoint's tiled256x64 layout (src/checkpoint.rs:20-100,
 * [rows/256][cols/64][256][64]) and is restored to rows on the device.  Outputs the tiled codes
 * (rows*cols*bits/8 bytes) and the f32 scale row.  rows and cols must be multiples of 256
 * (the reference's ensure!).
 */
CLEFQ_API int clefq_untile_bf16(void *stream, const void *src, int64_t rows, int64_t cols, void *dst);
CLEFQ_API int64_t clefq_load_weight_workspace_size(int64_t rows, int64_t cols, int bits, int tiled);
CLEFQ_API int clefq_load_weight(void *stream, const void *src, int64_t rows, int64_t cols, int bits, int tiled,
                                void *codes_tiled, float *scales, void *workspace, int64_t workspace_bytes);

/*
 * Dense quantized projection; replaces project_prepared + h3_gemm_i{4,8}_256[_residual]
 * (src/quantized.rs:470-537, kernels/gemm_integer.loom:394-433):
 *   y = (f32(sum_k a*w) * w_scales[n]) * a_scales[m] + 0
 *   BF16 out: finite values saturate to +-3.3895e38; with residual: bf16(res + bf16(y)).
 *   F32 out: y.
 *   a_codes  packed codes [m][a_ld_words] (as written by clefq_prepare), a_scales f32 [m]
 *   w_tiled  tiled codes of the [n][k] weight, w_scales f32 [n]
 *   residual BF16 [m][residual_ld] or NULL (BF16 output only)
 *   out      [m][out_ld] of out_dtype
 * bits 4 needs workspace >= clefq_gemm_workspace_size(m, k, 4) (the s8 operand);
 * bits 8 reads the packed codes directly (a_ld_words*4 must be a multiple of 16).
 * Checks: n % 128 == 0, k % 256 == 0, k <= a_ld_words * (32/bits).
 */
CLEFQ_API int64_t clefq_gemm_workspace_size(int64_t m, int64_t k, int bits);
CLEFQ_API int clefq_gemm(void *stream, int bits, const void *a_codes, int64_t a_ld_words, const float *a_scales,
                         int64_t m, const void *w_tiled, const float *w_scales, int64_t n, int64_t k,
                         const void *residual, int64_t residual_ld, int out_dtype, void *out, int64_t out_ld,
                         void *workspace, int64_t workspace_bytes);
/*
 * The same projection as clefq_gemm (bits 4 only) for callers that cannot allocate device
 * memory and so cannot pass a workspace: for example a host runtime that reserves all of
 * device memory for its own allocator at start-up and gives a plugin nothing but each
 * call's inputs and outputs, or an FFI binding with no workspace argument.  It has no
 * counterpart in the reference (whose engine owns every allocation).
 * The s8 operand scratch is a fixed 64 MiB array inside this library's device image:
 *   - m * k must be <= CLEFQ_GEMM_NOALLOC_MAX_BYTES, else CLEFQ_ERR_WORKSPACE;
 *   - with the CUDA runtime's default lazy module loading (CUDA 12.2 and later) the
 *     64 MiB are taken on a device by the first call there and kept until the process
 *     exits; with CUDA_MODULE_LOADING=EAGER every device on which this library has a
 *     context holds them, whether or not it calls this function;
 *   - the first call on a device resolves the array's address with that device current,
 *     which is what loads it.  A call with m == 0 does only that: a host whose allocator
 *     reserves all device memory makes one m == 0 call on each device first, otherwise
 *     the first real call may fail with CLEFQ_ERR_CUDA (out of memory);
 *   - all calls on a device share the array, so calls that overlap on the GPU (other
 *     streams or host threads) race on it -- the caller must serialise them.
 * Nothing here calls cudaMalloc, cudaFree or any allocating library routine.
 */
#define CLEFQ_GEMM_NOALLOC_MAX_BYTES (64ll << 20)
CLEFQ_API int clefq_gemm_noalloc(void *stream, const void *a_codes, int64_t a_ld_words, const float *a_scales,
                                 int64_t m, const void *w_tiled, const float *w_scales, int64_t n, int64_t k,
                                 const void *residual, int64_t residual_ld, int out_dtype, void *out, int64_t out_ld);

/* Same projection from an s8 operand written by clefq_prepare (no unpack pass). */
CLEFQ_API int clefq_gemm_s8(void *stream, int bits, const void *operand, int64_t operand_ld, const float *a_scales,
                            int64_t m, const void *w_tiled, const float *w_scales, int64_t n, int64_t k,
                            const void *residual, int64_t residual_ld, int out_dtype, void *out, int64_t out_ld);

/*
 * Two projections of one prepared input in one launch, the way a SwiGLU MLP's gate and up
 * projections share their packed activation (src/backbone.rs:880-894 calls project(gate) and
 * project(up) on one input; src/quantized.rs:254-280 reuses its packed codes):
 *   out[:, 0:n] = projection by w0, out[:, n:2n] = projection by w1, BF16 (as clefq_gemm_s8).
 * Checks: n % 128 == 0, k % 256 == 0, out_ld >= 2n.
 */
CLEFQ_API int clefq_gemm_pair_s8(void *stream, const void *operand, int64_t operand_ld, const float *a_scales,
                                 int64_t m, const void *w0_tiled, const float *w0_scales, const void *w1_tiled,
                                 const float *w1_scales, int64_t n, int64_t k, void *out, int64_t out_ld);

/*
 * Gate and up of one packed int4 input in one launch with SwiGLU in the epilogue, the gate|up
 * step of clefq_mlp: out BF16 [m][n] = bf16(bf16(silu(g)) * u) with g, u the BF16 projections
 * x.gate and x.up, bit-identical to project_quantized by gate and by up, then swiglu (src/quantized.rs:235-253,
 * src/ops.rs:9-29).  Checks: n % 256 == 0, k % 256 == 0, k >= 2048, out_ld even and >= n.
 */
CLEFQ_API int clefq_gemm_swiglu_s8(void *stream, const void *operand, int64_t operand_ld, const float *a_scales,
                                   int64_t m, const void *gate_tiled, const float *gate_scales, const void *up_tiled,
                                   const float *up_scales, int64_t n, int64_t k, void *out, int64_t out_ld);

/* SwiGLU bf16(bf16(g/(1+exp(-g))) * u); replaces Engine::swiglu (src/ops.rs:9-29,
 * kernels/swiglu.loom:41-50).  n elements, BF16. */
CLEFQ_API int clefq_swiglu(void *stream, const void *gate, const void *up, int64_t n, void *out);

/* SiLU bf16(g/(1+exp(-g))) of n BF16 values, the activation half of SwiGLU
 * (kernels/swiglu.loom:41-50), computed exactly as the SwiGLU GEMM epilogue computes it. */
CLEFQ_API int clefq_silu(void *stream, const void *x, int64_t n, void *out);

/*
 * Router; replaces omni_route (src/omni.rs:170-190, kernels/omni_route.loom:84-147):
 * routes f32 [tokens][2*topk] = selected ids (as f32) || BF16-rounded probabilities.
 * Checks: 0 < topk <= experts <= 128 and topk <= 32.  logits_dtype CLEFQ_BF16|CLEFQ_F32.
 */
CLEFQ_API int clefq_route(void *stream, const void *logits, int logits_dtype, int64_t tokens, int experts, int topk,
                          float *routes);

/*
 * Router linear and router in one kernel; replaces the two steps of the MoE block
 * (src/omni.rs:760-765): logits = project(norm, "mlp.gate") (BF16 GEMM, f32 accumulation,
 * BF16 output) followed by omni_route(logits, topk).
 *   x              BF16 [tokens][hidden] (the normalised hidden rows)
 *   router_weight  BF16 [experts][hidden], row-major
 *   routes         f32 [tokens][2*topk], as clefq_route
 *   logits_out     BF16 [tokens][experts] or NULL: the logits the routes were chosen from
 * The logits' f32 accumulation order is this kernel's (a tcgen05 BF16 GEMM), so they can
 * differ from another GEMM's by one BF16 rounding; routes are always exactly clefq_route of
 * logits_out.  Checks: hidden % 64 == 0; experts in 32..128, a multiple of 32; topk 1..8.
 */
CLEFQ_API int clefq_route_linear(void *stream, const void *x, const void *router_weight, int64_t tokens,
                                 int64_t hidden, int experts, int topk, float *routes, void *logits_out);

/*
 * Stable grouping; replaces omni_group_routes / omni_group_routes_ordered
 * (src/omni.rs:192-245, kernels/omni_group_routes{,_ordered}.loom):
 *   groups f32 [experts][tokens+1] = count, then route ids t*topk+rank in token order
 *   order  f32 [tokens][topk] (nullable) = rank of the j-th smallest expert id
 * workspace >= clefq_group_workspace_size(tokens, topk, experts).
 */
CLEFQ_API int64_t clefq_group_workspace_size(int64_t tokens, int topk, int experts);
CLEFQ_API int clefq_group_routes(void *stream, const float *routes, int64_t tokens, int topk, int experts,
                                 float *groups, float *order, void *workspace, int64_t workspace_bytes);

/* Task list [total, (expert, row0) per 16-row tile]; replaces omni_expert_tasks
 * (src/omni.rs:126-169, kernels/omni_expert_tasks.loom:30-61). tasks f32 of length
 * 1 + 2*(ceil(tokens*topk/16) + experts - 1). */
CLEFQ_API int clefq_expert_tasks(void *stream, const float *groups, int64_t tokens, int experts, float *tasks);

/*
 * Grouped INT4 expert projection; replaces omni_expert_impl with groups
 * (src/omni.rs:289-534; kernels/omni_expert_i4.loom, _compact, _k128_down):
 *   for expert e, route r in groups[e]: x = input_routed ? r : r / topk
 *   out[r][c] = bf16(f32(sum_k a[x][k] * w[e*n + c][k]) * (a_scales[x] * w_scales[e*n + c]))
 *   a_codes packed int4 [rows][a_ld_words] + a_scales, rows = tokens (or tokens*topk routed)
 *   w_tiled tiled [experts*n][k], w_scales [experts*n]; out BF16 [tokens*topk][n]
 * Checks: n % 128 == 0 (the reference needs n % 256), k % 256 == 0.
 * workspace >= clefq_expert_workspace_size(tokens, topk, experts, k).
 */
CLEFQ_API int64_t clefq_expert_workspace_size(int64_t tokens, int topk, int experts, int64_t k);
CLEFQ_API int clefq_expert(void *stream, const void *a_codes, int64_t a_ld_words, const float *a_scales,
                           const void *w_tiled, const float *w_scales, const float *groups, int64_t tokens, int topk,
                           int experts, int64_t k, int64_t n, int input_routed, void *out, void *workspace,
                           int64_t workspace_bytes);

/*
 * Gate and up experts with SwiGLU in the GEMM epilogue, one launch; replaces the reference's
 * fused gate/up experts omni_gate_up (src/omni.rs:302-373,
 * benches/kernels/omni_gate_up_i4.loom):
 *   out[r][c] = bf16(bf16(silu(g)) * u), g and u the BF16 expert projections of clefq_expert
 *   (input_routed = 0) by gate_tiled and up_tiled, for route r of groups; out BF16
 *   [tokens*topk][n], rows in route order.
 * Each CTA of the pair holds 64 gate and the matching 64 up weight rows, so both operands of
 * every SwiGLU meet in one accumulator.  Checks: n % 256 == 0, k % 256 == 0, k >= 2048.
 * workspace >= clefq_expert_workspace_size(tokens, topk, experts, k).
 */
CLEFQ_API int clefq_expert_gate_up(void *stream, const void *a_codes, int64_t a_ld_words, const float *a_scales,
                                   const void *gate_tiled, const float *gate_scales, const void *up_tiled,
                                   const float *up_scales, const float *groups, int64_t tokens, int topk, int experts,
                                   int64_t k, int64_t n, void *out, void *workspace, int64_t workspace_bytes);

/*
 * Weighted combine in ascending expert order with BF16 rounding at each step; replaces
 * omni_combine_ordered (order != NULL) and omni_combine (order == NULL)
 * (src/omni.rs:246-278,535-556; kernels/omni_combine{,_ordered}.loom).
 *   values BF16 [tokens*topk][width], routes f32 [tokens][2*topk] -> out BF16 [tokens][width]
 * Checks: width % 8 == 0.
 */
CLEFQ_API int clefq_combine(void *stream, const void *values, const float *routes, const float *order,
                            int64_t tokens, int topk, int64_t width, void *out);

/*
 * Dense INT4 SwiGLU MLP block; replaces mlp() = project(gate), project(up),
 * project_swiglu(gate, up, down, residual) (src/backbone.rs:880-894,
 * src/quantized.rs:406-439), bit-identical to those separate steps:
 *   prepare(x) -> gate, up projections -> SwiGLU -> prepare -> down projection (+ residual)
 * With hidden >= 4096 and inter % 256 == 0 the gate|up launch applies SwiGLU in its epilogue
 * and writes the hidden rows; otherwise SwiGLU is fused into their packing (same outputs).
 *   x BF16 [m][hidden]; gate/up tiled [inter][hidden] + scales; down tiled [hidden][inter]
 *   out BF16 [m][hidden]; residual BF16 [m][hidden] or NULL
 * workspace >= clefq_mlp_workspace_size(m, hidden, inter).
 */
CLEFQ_API int64_t clefq_mlp_workspace_size(int64_t m, int64_t hidden, int64_t inter);
CLEFQ_API int clefq_mlp(void *stream, const void *x, int64_t m, int64_t hidden, int64_t inter, const void *gate_tiled,
                        const float *gate_scales, const void *up_tiled, const float *up_scales, const void *down_tiled,
                        const float *down_scales, const void *residual, void *out, void *workspace,
                        int64_t workspace_bytes);
/*
 * Pre-norm MLP block with the input as residual; replaces normalized_mlp
 * (src/quantized.rs:348-404): RMSNorm (weight + 1 offset, eps 1e-6, mean over `hidden`)
 * fused into the packing of x (prepare_norm_with_source, src/quantized.rs:615-640), gate and
 * up projections of the shared codes, SwiGLU (in the gate|up epilogue or the packing of the
 * hidden rows, as clefq_mlp chooses), and the down projection with x itself as residual:
 *   out = bf16(x + bf16(down(swiglu(gate(norm(x)), up(norm(x))))))
 * norm_weight BF16 [hidden].  out may be x (each element is read before it is overwritten).
 * The reference takes this path only at width 5120 and 17408 intermediate rows; any width
 * that is a multiple of 256 works here.  workspace >= clefq_mlp_workspace_size(m, hidden, inter).
 */
CLEFQ_API int clefq_normalized_mlp(void *stream, const void *x, int64_t m, int64_t hidden, int64_t inter,
                                   const void *norm_weight, const void *gate_tiled, const float *gate_scales,
                                   const void *up_tiled, const float *up_scales, const void *down_tiled,
                                   const float *down_scales, void *out, void *workspace, int64_t workspace_bytes);
/*
 * clefq_mlp from host memory to host memory: x, residual (nullable) and out are host
 * buffers [m][hidden] (pinned for the copies to overlap).  The rows run in chunks of
 * chunk_rows; each chunk's host->device copy, kernels and device->host copy overlap those of
 * its neighbours (library-owned copy streams).  Rows are independent, so the output equals
 * clefq_mlp's.
 *   flags: CLEFQ_HOST_STREAMING lets this call's input copies start before earlier work on
 *          `stream` finishes (the next call of a stream of calls then overlaps this one); the
 *          workspace must then be used by these calls only.  0: the call starts after
 *          earlier work on `stream`.
 *   done_event: a cudaEvent_t recorded after the call's last output copy (out is complete
 *          once it has fired); NULL makes `stream` wait for that copy instead.
 * workspace >= clefq_mlp_host_workspace_size(chunk_rows, hidden, inter, residual != NULL).
 */
#define CLEFQ_HOST_STREAMING 1
CLEFQ_API int64_t clefq_mlp_host_workspace_size(int64_t chunk_rows, int64_t hidden, int64_t inter, int with_residual);
CLEFQ_API int clefq_mlp_host(void *stream, const void *x_host, int64_t m, int64_t hidden, int64_t inter,
                             const void *gate_tiled, const float *gate_scales, const void *up_tiled,
                             const float *up_scales, const void *down_tiled, const float *down_scales,
                             const void *residual_host, void *out_host, int64_t chunk_rows, int flags,
                             void *done_event, void *workspace, int64_t workspace_bytes);

/*
 * Omni INT4 MoE block; replaces the expert part of forward_layers_cached
 * (src/omni.rs:761-857, fast defaults): route(logits) -> ordered groups -> gate, up
 * experts on the shared packed input -> SwiGLU -> down experts -> ordered combine.
 *   x BF16 [tokens][hidden] (normalized input), logits [tokens][experts] (logits_dtype), or
 *   with CLEFQ_ROUTER_WEIGHT_BF16 the router weight [experts][hidden] (router linear fused in)
 *   gate/up tiled [experts*inter][hidden] + scales; down tiled [experts*hidden][inter]
 *   out BF16 [tokens][hidden]; routes_out f32 [tokens][2*topk] (nullable)
 * workspace >= clefq_moe_workspace_size(tokens, hidden, inter, experts, topk).
 */
CLEFQ_API int64_t clefq_moe_workspace_size(int64_t tokens, int64_t hidden, int64_t inter, int experts, int topk);
CLEFQ_API int clefq_moe(void *stream, const void *x, const void *logits, int logits_dtype, int64_t tokens,
                        int64_t hidden, int64_t inter, int experts, int topk, const void *gate_tiled,
                        const float *gate_scales, const void *up_tiled, const float *up_scales,
                        const void *down_tiled, const float *down_scales, void *out, float *routes_out,
                        void *workspace, int64_t workspace_bytes);

/*
 * Expert-parallel Omni MoE.  No counterpart in the reference, which runs the MoE block on
 * one GPU (src/omni.rs:761-857); these are the pieces around the two all-to-all exchanges
 * of a host that shards the experts over `world` ranks (rank r owns experts
 * [r*experts/world, (r+1)*experts/world)).  Per layer, on every rank:
 *   1. clefq_route + clefq_prepare(x, int4, no operand)              (home tokens)
 *   2. clefq_moe_ep_plan  -> send_counts[world] (int64, device) and send_slots[tokens*topk]
 *   3. exchange counts; clefq_moe_ep_pack -> one record per route, grouped by destination
 *   4. all-to-all of the records (clefq_moe_ep_record_bytes(hidden) bytes each)
 *   5. clefq_moe_ep_experts on the received records -> BF16 products bf16(value * prob)
 *   6. all-to-all of the products back (hidden BF16 each, same order as sent)
 *   7. clefq_moe_ep_combine -> the reference's ascending-expert BF16 chain per token.
 * The result is bit-identical to clefq_moe on one GPU.
 */
CLEFQ_API int64_t clefq_moe_ep_record_bytes(int64_t hidden);
/* routes f32 [tokens][2*topk] from clefq_route; send_counts int64 [world]; send_slots int32 [tokens*topk];
 * workspace of clefq_moe_ep_plan_workspace_size(world) bytes */
CLEFQ_API int64_t clefq_moe_ep_plan_workspace_size(int world);
CLEFQ_API int clefq_moe_ep_plan(void *stream, const float *routes, int64_t tokens, int topk, int experts, int world,
                                int64_t *send_counts, int32_t *send_slots, void *workspace, int64_t workspace_bytes);
/* a_codes/a_ld_words/a_scales: packed int4 rows of the tokens (clefq_prepare storage) */
CLEFQ_API int clefq_moe_ep_pack(void *stream, const void *a_codes, int64_t a_ld_words, const float *a_scales,
                                int64_t tokens, int64_t hidden, const float *routes, int topk,
                                const int32_t *send_slots, void *send_records);
/* records [n][record_bytes] received from all ranks; local expert weights as in clefq_moe with
 * experts = local_experts; products BF16 [n][hidden] in record order. */
CLEFQ_API int64_t clefq_moe_ep_experts_workspace_size(int64_t records, int64_t hidden, int64_t inter,
                                                      int local_experts);
CLEFQ_API int clefq_moe_ep_experts(void *stream, const void *records, int64_t n, int64_t hidden, int64_t inter,
                                   int expert_base, int local_experts, const void *gate_tiled, const float *gate_scales,
                                   const void *up_tiled, const float *up_scales, const void *down_tiled,
                                   const float *down_scales, void *products, void *workspace,
                                   int64_t workspace_bytes);
/* products BF16 [sum(send_counts)][hidden] in send order; out BF16 [tokens][hidden] */
CLEFQ_API int clefq_moe_ep_combine(void *stream, const void *products, const int32_t *send_slots, const float *routes,
                                   int64_t tokens, int topk, int64_t hidden, void *out);

/*
 * Split packing and tensor-parallel MLP helpers.  No counterpart in the reference, which runs
 * the MLP block on one GPU (src/backbone.rs:880-894); these serve a host that shards the
 * intermediate dimension over `world` ranks (rank r: gate/up rows [r*I/G, (r+1)*I/G), down rows
 * [r*H/G, (r+1)*H/G)).  Per MLP block, on every rank:
 *   1. clefq_prepare(x) (replicated) and the gate|up GEMM of the rank's intermediate rows
 *   2. clefq_prepare_rowmax(SwiGLU shard) -> f32 [rows]; all-reduce MAX over the ranks
 *   3. clefq_prepare_scaled(SwiGLU shard, the reduced maxima) -> int4 codes of the shard,
 *      with the scales of the full row (identical on every rank)
 *   4. all-gather the code shards; clefq_tp_gather_unpack -> the full s8 operand
 *   5. the down GEMM of the rank's output rows; all-gather; clefq_tp_interleave -> [rows][H]
 * The result is bit-identical to clefq_mlp on one GPU.
 */
/* kind: CLEFQ_PREP_PLAIN or CLEFQ_PREP_SWIGLU; rowmax f32 [rows]: max |Hadamard| of the row,
 * non-finite rows +inf */
CLEFQ_API int clefq_prepare_rowmax(void *stream, int kind, const void *x, int64_t x_ld, const void *aux,
                                   int64_t aux_ld, int64_t rows, int64_t width, float *rowmax);
/* as clefq_prepare (no norm output), with the row scale taken from rowmax[row] */
CLEFQ_API int clefq_prepare_scaled(void *stream, int kind, int bits, const void *x, int64_t x_ld, const void *aux,
                                   int64_t aux_ld, int64_t rows, int64_t width, int64_t stride, const float *rowmax,
                                   void *out, void *operand, int64_t operand_ld);
/* codes u32 [world][rows][shard_width/8] -> s8 operand [rows][operand_ld] (world*shard_width used) */
CLEFQ_API int clefq_tp_gather_unpack(void *stream, const void *codes, int world, int64_t rows, int64_t shard_width,
                                     void *operand, int64_t operand_ld);
/* src [world][rows][shard_bytes] -> dst [rows][dst_ld_bytes]: rank shards side by side */
CLEFQ_API int clefq_tp_interleave(void *stream, const void *src, int world, int64_t rows, int64_t shard_bytes,
                                  void *dst, int64_t dst_ld_bytes);

/*
 * Symmetric device regions for the ranks of one node (no counterpart in the reference, which
 * runs on one GPU).  Each rank creates a region of the same size; peers map it through CUDA
 * IPC handles exchanged by the host (clefq_comm_open), or, when one process drives several
 * GPUs with peer access enabled, through clefq_comm_attach.  Kernels then store into peers'
 * regions over NVLink; clefq_comm_barrier orders such phases on the device.  A barrier wait
 * gives up after the timeout (default 5 s) and clefq_status then reports CLEFQ_ERR_TIMEOUT;
 * the communicator is out of step after that and must be recreated.
 */
typedef struct clefq_comm clefq_comm;
/* bytes of one IPC handle (the host gathers world of them, in rank order) */
CLEFQ_API int64_t clefq_comm_handle_bytes(void);
/* allocates this rank's region of `bytes` (on the current device); handle may be NULL */
CLEFQ_API int clefq_comm_create(int rank, int world, int64_t bytes, clefq_comm **comm, void *handle);
/* maps every peer's region from handles[world] (this rank's entry is ignored) */
CLEFQ_API int clefq_comm_open(clefq_comm *comm, const void *handles);
/* uses `peer` (rank `rank` of the same group, created in this process) as that rank's region */
CLEFQ_API int clefq_comm_attach(clefq_comm *comm, int rank, clefq_comm *peer);
/* 1 when every rank's region is mapped */
CLEFQ_API int clefq_comm_ready(const clefq_comm *comm);
CLEFQ_API void *clefq_comm_region(clefq_comm *comm);
CLEFQ_API int64_t clefq_comm_region_bytes(const clefq_comm *comm);
CLEFQ_API int clefq_comm_set_timeout_ms(clefq_comm *comm, int64_t ms);
/* device barrier over the group, ordered on `stream` */
CLEFQ_API int clefq_comm_barrier(clefq_comm *comm, void *stream);
CLEFQ_API int clefq_comm_destroy(clefq_comm *comm);

/*
 * Tensor-parallel MLP block with its collectives inside the kernels (the reference's MLP block,
 * src/backbone.rs:880-894 and src/quantized.rs:406-439, sharded over the communicator's
 * ranks).  Rank r passes its shards: gate/up tiled rows [r*I/G, (r+1)*I/G) with their scales,
 * down tiled rows [r*H/G, (r+1)*H/G); every rank passes the same x [m][hidden] and residual
 * (nullable) and receives the whole output [m][hidden], bit-identical to clefq_mlp.
 *   1. pack x; gate|up GEMM of the shard
 *   2. SwiGLU shard row maxima -> the barrier stores them into every peer and reduces (max)
 *   3. the shard packed with the full-row maxima; the packing kernel stores its int4 code
 *      words into every rank's region; barrier; the full code rows unpacked to the s8 operand
 *   4. down GEMM of the rank's output columns over the full operand; the epilogue stores them
 *      into every rank's region; barrier; copy to out (skipped when out is
 *      clefq_tp_mlp_output(), which stays valid until this rank's next call)
 * Needs I % (256*G) == 0 and H % (256*G) == 0, a region of clefq_tp_mlp_region_bytes and a
 * workspace of clefq_tp_mlp_workspace_size (both -1 for an unsupported shape).
 */
CLEFQ_API int64_t clefq_tp_mlp_region_bytes(int64_t m, int64_t hidden, int64_t inter, int world);
CLEFQ_API int64_t clefq_tp_mlp_workspace_size(int64_t m, int64_t hidden, int64_t inter, int world);
CLEFQ_API int clefq_tp_mlp(clefq_comm *comm, void *stream, const void *x, int64_t m, int64_t hidden, int64_t inter,
                           const void *gate_tiled, const float *gate_scales, const void *up_tiled,
                           const float *up_scales, const void *down_tiled, const float *down_scales,
                           const void *residual, void *out, void *workspace, int64_t workspace_bytes);
CLEFQ_API void *clefq_tp_mlp_output(clefq_comm *comm, int64_t m, int64_t hidden, int64_t inter);

/*
 * Expert-parallel Omni MoE layer with its exchanges inside the kernels (the reference's MoE
 * block, src/omni.rs:761-857, with the experts split over the communicator's ranks: rank r
 * owns experts [r*E/G, (r+1)*E/G) and passes their tiled weights, in clefq_moe's layout for
 * E/G experts).  Every rank passes its own tokens; out [tokens][hidden] is bit-identical to
 * clefq_moe over those tokens on one GPU.  No host synchronisation:
 *   1. route and pack the tokens; group the routes by destination rank
 *   2. barrier that also stores this rank's per-destination counts into every peer
 *   3. dispatch: one record per route stored straight into the destination's receive buffer
 *      (int4 code row, scale, expert id, probability, home route index); barrier
 *   4. the received routes grouped by local expert; grouped gate|up GEMM, SwiGLU packing and
 *      down GEMM, whose epilogue stores bf16(value * probability) into the home rank's
 *      product buffer at the route's index; barrier
 *   5. the reference's ascending-expert BF16 chain over the returned products
 * recv_cap bounds the records one rank receives (the same on every rank; world*tokens*topk
 * always suffices); exceeding it records status site 9 (clefq_status -> CLEFQ_ERR_TIMEOUT
 * class error) and drops the excess.  Region and workspace sizes from the two queries (-1
 * for an unsupported shape).
 */
CLEFQ_API int64_t clefq_moe_ep_layer_region_bytes(int64_t tokens, int64_t hidden, int topk, int world,
                                                  int64_t recv_cap);
CLEFQ_API int64_t clefq_moe_ep_layer_workspace_size(int64_t tokens, int64_t hidden, int64_t inter, int experts,
                                                    int topk, int world, int64_t recv_cap);
CLEFQ_API int clefq_moe_ep_layer(clefq_comm *comm, void *stream, const void *x, const void *logits,
                                 int logits_dtype, int64_t tokens, int64_t hidden, int64_t inter, int experts,
                                 int topk, int64_t recv_cap, const void *gate_tiled, const float *gate_scales,
                                 const void *up_tiled, const float *up_scales, const void *down_tiled,
                                 const float *down_scales, void *out, float *routes_out, void *workspace,
                                 int64_t workspace_bytes);

#ifdef __cplusplus
}
#endif
#endif /* CLEFQ_H */
