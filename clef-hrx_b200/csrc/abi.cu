// clefq: the C ABI (include/clefq.h).  Argument checks mirror the reference's ensure!
// conditions; every entry point is stream-ordered and allocates nothing.
#include <mutex>
#include <stdarg.h>
#include <stdio.h>

#include "clefq_internal.h"
#include "cq_common.cuh"

namespace cq {
int launch_route(const void *logits, int is_f32, int64_t tokens, int experts, int topk, float *routes,
                 cudaStream_t stream);
int launch_group(const float *routes, int64_t tokens, int topk, int experts, int tile_rows, int *counts, int *offsets,
                 int *tile_list, int *perm, float *groups, float *order, float *tasks, cudaStream_t stream,
                 int num_sms);
int launch_tasks(const float *groups, int64_t tokens, int experts, float *tasks, cudaStream_t stream);
int launch_route_linear(const void *x, const void *w, int64_t tokens, int hidden, int experts, int topk, float *routes,
                        uint16_t *logits_out, int *err, cudaStream_t stream);
int launch_groups_to_sorted(const float *groups, int64_t tokens, int topk, int experts, int tile_rows, int *offsets,
                            int *perm, int *tile_list, cudaStream_t stream);
int launch_gather(const uint8_t *src, int64_t src_ld, const int *perm, int div, int64_t rows, int64_t row_bytes,
                  uint8_t *dst, int64_t dst_ld, cudaStream_t stream, int num_sms);
int launch_gather_unpack_i4(const uint32_t *a, int64_t a_ld, const int *perm, int div, int64_t rows, int k,
                            uint8_t *dst, int64_t dst_ld, cudaStream_t stream, int num_sms,
                            const int64_t *rows_dev = nullptr);
int launch_combine(const uint16_t *values, const float *routes, const float *order, int64_t tokens, int topk,
                   int64_t width, uint16_t *out, cudaStream_t stream, int num_sms, bool weighted = false);
int launch_tp_gather_unpack(const uint32_t *codes, int world, int64_t rows, int shard_words, uint8_t *op,
                            int64_t op_ld, cudaStream_t stream, int num_sms);
int launch_tp_interleave(const uint8_t *src, int world, int64_t rows, int64_t shard_bytes, uint8_t *dst,
                         int64_t dst_ld, cudaStream_t stream, int num_sms);
int launch_ep_plan(const float *routes, int64_t tokens, int topk, int experts, int world, long long *counts,
                   int *slots, int *scratch, cudaStream_t stream);
int launch_ep_pack(const uint32_t *xq, int64_t words_ld, const float *scales, const float *routes, const int *slots,
                   int64_t tokens, int topk, int code_words, int64_t rec_words, uint32_t *send, cudaStream_t stream,
                   int num_sms);
int launch_ep_unpack_meta(const uint32_t *recv, int64_t n, int code_words, int64_t rec_words, int expert_base,
                          int local_experts, float *scales, float *routes, cudaStream_t stream, int num_sms);
int launch_ep_weigh(const uint16_t *values, const float *routes, int64_t n, int64_t width, uint16_t *products,
                    cudaStream_t stream, int num_sms);
int launch_ep_combine(const uint16_t *products, const int *slots, const float *routes, int64_t tokens, int topk,
                      int64_t width, uint16_t *out, cudaStream_t stream, int num_sms);

// Status word set by bounded device-side waits (static: nothing is allocated for it).
static __device__ int g_status_word;

namespace {
thread_local char g_err[512] = "";
thread_local cudaError_t g_launch_err = cudaSuccess;
std::mutex g_mu;
int g_sms[64];
int *g_status_ptr[64];

int set_err(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
  return code;
}
int cuda_err(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = g_launch_err;  // a launch helper already took it
  return set_err(CLEFQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}
int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d < 0 || d >= 64 ? 0 : d;
}

bool al16(const void *p) { return ((uintptr_t)p & 15) == 0; }
}  // namespace

// Records a failure message for clefq_last_error() from another translation unit.
int report_error(int code, const char *msg) { return set_err(code, "%s", msg); }

int launch_check() {
  const cudaError_t e = cudaGetLastError();
  g_launch_err = e;
  return e == cudaSuccess ? 0 : CLEFQ_ERR_CUDA;
}

cudaError_t last_launch_error() { return g_launch_err; }

int device_sms() {
  const int d = current_device();
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_sms[d]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, d);
    g_sms[d] = v > 0 ? v : 148;
  }
  return g_sms[d];
}

int *device_status_word() {
  const int d = current_device();
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_status_ptr[d]) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_status_word) != cudaSuccess) return nullptr;
    g_status_ptr[d] = static_cast<int *>(p);
  }
  return g_status_ptr[d];
}

// ---- validation shared by the packing entry points (src/quantized.rs:621-640) --------
static int check_prepare(int kind, int bits, int64_t rows, int64_t width, int64_t stride) {
  if (!(bits == 4 || bits == 8)) return set_err(CLEFQ_ERR_SHAPE, "unsupported rotated integer operand: bits=%d", bits);
  if (kind < 0 || kind > 4) return set_err(CLEFQ_ERR_SHAPE, "unknown packing kind %d", kind);
  if (width < 256 || width > 32768 || width % 256)
    return set_err(CLEFQ_ERR_SHAPE, "unsupported rotated integer operand: width=%lld", (long long)width);
  if (rows < 1 || rows > 1048576)
    return set_err(CLEFQ_ERR_SHAPE, "unsupported rotated integer operand: rows=%lld", (long long)rows);
  if (stride < width || stride > 65536 || stride % (512 / bits))
    return set_err(CLEFQ_ERR_SHAPE, "unsupported rotated integer operand: stride=%lld", (long long)stride);
  return 0;
}

static int run_prepare(cudaStream_t s, int kind, int bits, const void *x, int64_t x_ld, const void *aux,
                       int64_t aux_ld, int64_t rows, int64_t width, int64_t stride, void *out, void *operand,
                       int64_t operand_ld, void *norm_out, int64_t norm_ld, float *rowmax_out = nullptr,
                       const float *rowmax_in = nullptr, uint32_t *const *code_dst = nullptr,
                       int n_code_dst = 0, int64_t code_ld = 0, const int64_t *rows_dev = nullptr,
                       const int *dup_rows = nullptr, int dup = 0) {
  int rc = check_prepare(kind, bits, rows, width, stride);
  if (rc) return rc;
  if (!x || (!out && !rowmax_out) || (kind != CLEFQ_PREP_PLAIN && !aux) ||
      (kind == CLEFQ_PREP_NORM_STORE && !norm_out))
    return set_err(CLEFQ_ERR_SHAPE, "packing input count");
  if (x_ld < width || !al16(x) || (x_ld * 2) % 16) return set_err(CLEFQ_ERR_ALIGN, "x must be 16-byte aligned rows");
  if (kind == CLEFQ_PREP_SWIGLU && (aux_ld < width || !al16(aux) || (aux_ld * 2) % 16))
    return set_err(CLEFQ_ERR_SHAPE, "packing input shape/dtype mismatch");
  if (kind == CLEFQ_PREP_ATTN_GATE && (aux_ld < 2 * width || !al16(aux) || (aux_ld * 2) % 16))
    return set_err(CLEFQ_ERR_SHAPE, "attention packing input count");
  if ((kind == CLEFQ_PREP_NORM || kind == CLEFQ_PREP_NORM_STORE) && !al16(aux))
    return set_err(CLEFQ_ERR_ALIGN, "norm weight must be 16-byte aligned");
  if (kind == CLEFQ_PREP_NORM_STORE && (norm_ld < width || !al16(norm_out) || (norm_ld * 2) % 16))
    return set_err(CLEFQ_ERR_ALIGN, "norm output must be 16-byte aligned rows");
  if (operand) {
    if (bits != 4) return set_err(CLEFQ_ERR_SHAPE, "the s8 operand output is for 4-bit codes");
    if (operand_ld < width || !al16(operand) || operand_ld % 16)
      return set_err(CLEFQ_ERR_ALIGN, "operand must be 16-byte aligned rows of >= width bytes");
  }
  if ((uintptr_t)out % 8) return set_err(CLEFQ_ERR_ALIGN, "packed output must be 8-byte aligned");
  PrepareArgs a{};
  a.x = static_cast<const uint16_t *>(x);
  a.x_ld = x_ld;
  a.aux = static_cast<const uint16_t *>(aux);
  a.aux_ld = aux_ld;
  a.rows = rows;
  a.width = (int)width;
  a.stride = (int)stride;
  a.bits = bits;
  a.mode = kind;
  a.out = static_cast<uint32_t *>(out);
  a.op8 = static_cast<uint8_t *>(operand);
  a.op_ld = operand_ld;
  a.norm_out = static_cast<uint16_t *>(norm_out);
  a.norm_ld = norm_ld;
  a.rowmax_out = rowmax_out;
  a.rowmax_in = rowmax_in;
  for (int d = 0; d < n_code_dst; ++d) a.code_dst[d] = code_dst[d];
  a.n_code_dst = n_code_dst;
  a.code_ld = code_ld;
  a.rows_dev = rows_dev;
  a.dup_rows = dup_rows;
  a.dup = dup;
  return launch_prepare(a, s);  // sets clefq_last_error() itself on failure
}

static int run_gemm(cudaStream_t s, int bits, const uint8_t *op, int64_t op_ld, int64_t op_rows, const float *a_scales,
                    int64_t m, const void *w0, const float *ws0, const void *w1, const float *ws1, int n_split, int64_t n,
                    int64_t k, const void *residual, int64_t residual_ld, int out_dtype, void *out, int64_t out_ld,
                    uint16_t *const *out_peer = nullptr, int n_out_peer = 0, bool swiglu = false) {
  int *status = device_status_word();
  if (!status) return cuda_err("status word");
  GemmParams p{};
  p.a_op = op;
  p.a_rows = op_rows;
  p.a_ld = op_ld;
  p.a_scales = a_scales;
  p.w[0] = static_cast<const uint32_t *>(w0);
  p.w[1] = static_cast<const uint32_t *>(w1);
  p.w_scales[0] = ws0;
  p.w_scales[1] = ws1;
  p.n_split = n_split;
  p.m = m;
  p.n = (int)n;
  p.k = (int)k;
  p.bits = bits;
  p.out = out_dtype == CLEFQ_BF16 ? static_cast<uint16_t *>(out) : nullptr;
  p.out_f32 = out_dtype == CLEFQ_F32 ? static_cast<float *>(out) : nullptr;
  p.ldo = out_ld;
  p.residual = static_cast<const uint16_t *>(residual);
  p.ldr = residual_ld;
  p.err = status;
  for (int d = 0; d < n_out_peer; ++d) p.out_peer[d] = out_peer[d];
  p.n_out_peer = n_out_peer;
  if (swiglu) {
    p.swiglu = 1;
    p.silu_tab = silu_table_device();
  }
  int rc = launch_gemm(p, s);
  if (rc == CLEFQ_ERR_CUDA) return cuda_err("gemm launch");
  if (rc) return set_err(rc, "unsupported integer GEMM shape or alignment (n %% 128, k %% 256, 16-byte operand rows)");
  return 0;
}

static int check_gemm(int bits, int64_t m, int64_t n, int64_t k, int64_t a_cols, const void *residual,
                      int64_t residual_ld, int out_dtype, int64_t out_ld) {
  if (!(bits == 4 || bits == 8)) return set_err(CLEFQ_ERR_SHAPE, "integer projections need 4 or 8 bits");
  if (m < 0 || m > 16777216) return set_err(CLEFQ_ERR_SHAPE, "row count out of range");
  if (n < 128 || n > 65536 || n % 128) return set_err(CLEFQ_ERR_SHAPE, "n must be a multiple of 128 in [128, 65536]");
  if (k < 256 || k > 65536 || k % 256) return set_err(CLEFQ_ERR_SHAPE, "k must be a multiple of 256 in [256, 65536]");
  if (a_cols < k) return set_err(CLEFQ_ERR_SHAPE, "quantized projection shape/dtype mismatch");
  if (out_dtype != CLEFQ_BF16 && out_dtype != CLEFQ_F32) return set_err(CLEFQ_ERR_SHAPE, "unknown output dtype");
  if (out_ld < n) return set_err(CLEFQ_ERR_SHAPE, "output pitch below n");
  if (residual && (out_dtype != CLEFQ_BF16 || residual_ld < n))
    return set_err(CLEFQ_ERR_SHAPE, "projection residual shape/dtype mismatch");
  return 0;
}

}  // namespace cq

using namespace cq;

extern "C" {

const char *clefq_last_error(void) { return g_err; }
int clefq_version(void) { return 100; }

int clefq_status(void *stream) {
  int *w = device_status_word();
  if (!w) return cuda_err("status word");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(s) != cudaSuccess) return cuda_err("stream");
  int v = 0;
  if (cudaMemcpy(&v, w, sizeof v, cudaMemcpyDeviceToHost) != cudaSuccess) return cuda_err("status read");
  if (v) {
    int zero = 0;
    cudaMemcpy(w, &zero, sizeof zero, cudaMemcpyHostToDevice);
    return set_err(CLEFQ_ERR_TIMEOUT, "a device-side wait gave up (site %d)", v);
  }
  return 0;
}

int clefq_prepare(void *stream, int kind, int bits, const void *x, int64_t x_ld, const void *aux, int64_t aux_ld,
                  int64_t rows, int64_t width, int64_t stride, void *out, void *operand, int64_t operand_ld,
                  void *norm_out, int64_t norm_ld) {
  return run_prepare(static_cast<cudaStream_t>(stream), kind, bits, x, x_ld, aux, aux_ld, rows, width, stride, out,
                     operand, operand_ld, norm_out, norm_ld);
}

// Split packing of rows sharded by columns over several GPUs (no reference counterpart):
// each shard publishes its row maxima, the host reduces them with MAX, and every shard then
// quantises with the full row's maximum, so the codes and scales equal one-GPU packing.
int clefq_prepare_rowmax(void *stream, int kind, const void *x, int64_t x_ld, const void *aux, int64_t aux_ld,
                         int64_t rows, int64_t width, float *rowmax) {
  if (kind != CLEFQ_PREP_PLAIN && kind != CLEFQ_PREP_SWIGLU)
    return set_err(CLEFQ_ERR_SHAPE, "split packing supports plain and SwiGLU rows");
  if (!rowmax) return set_err(CLEFQ_ERR_SHAPE, "null row maxima");
  return run_prepare(static_cast<cudaStream_t>(stream), kind, 4, x, x_ld, aux, aux_ld, rows, width, width, nullptr,
                     nullptr, 0, nullptr, 0, rowmax, nullptr);
}

int clefq_prepare_scaled(void *stream, int kind, int bits, const void *x, int64_t x_ld, const void *aux,
                         int64_t aux_ld, int64_t rows, int64_t width, int64_t stride, const float *rowmax, void *out,
                         void *operand, int64_t operand_ld) {
  if (kind != CLEFQ_PREP_PLAIN && kind != CLEFQ_PREP_SWIGLU)
    return set_err(CLEFQ_ERR_SHAPE, "split packing supports plain and SwiGLU rows");
  if (!rowmax) return set_err(CLEFQ_ERR_SHAPE, "null row maxima");
  return run_prepare(static_cast<cudaStream_t>(stream), kind, bits, x, x_ld, aux, aux_ld, rows, width, stride, out,
                     operand, operand_ld, nullptr, 0, nullptr, rowmax);
}

int clefq_retile(void *stream, const void *codes, int64_t rows, int64_t cols, int bits, int64_t in_words, void *out) {
  if (!(bits == 4 || bits == 8)) return set_err(CLEFQ_ERR_SHAPE, "unsupported packed weight shape for tiling");
  const int64_t words = cols / (32 / bits);
  if (rows <= 0 || rows % 128 || cols % (32 / bits) || words % 32 || in_words < words)
    return set_err(CLEFQ_ERR_SHAPE, "unsupported packed weight shape for tiling");
  if (!al16(codes) || !al16(out)) return set_err(CLEFQ_ERR_ALIGN, "codes/out must be 16-byte aligned");
  int rc = launch_retile(static_cast<const uint32_t *>(codes), rows, in_words, words, static_cast<uint32_t *>(out),
                         static_cast<cudaStream_t>(stream), device_sms());
  return rc ? cuda_err("retile launch") : 0;
}

int64_t clefq_gemm_workspace_size(int64_t m, int64_t k, int bits) { return bits == 4 ? ((m * k + 255) & ~255LL) : 0; }

int clefq_gemm(void *stream, int bits, const void *a_codes, int64_t a_ld_words, const float *a_scales, int64_t m,
               const void *w_tiled, const float *w_scales, int64_t n, int64_t k, const void *residual,
               int64_t residual_ld, int out_dtype, void *out, int64_t out_ld, void *workspace,
               int64_t workspace_bytes) {
  int rc = check_gemm(bits, m, n, k, a_ld_words * (32 / bits), residual, residual_ld, out_dtype, out_ld);
  if (rc) return rc;
  if (m == 0) return 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (bits == 8) {
    if ((a_ld_words * 4) % 16 || !al16(a_codes))
      return set_err(CLEFQ_ERR_ALIGN, "8-bit codes are read in place: 16-byte aligned rows needed");
    return run_gemm(s, 8, static_cast<const uint8_t *>(a_codes), a_ld_words * 4, m, a_scales, m, w_tiled, w_scales,
                    nullptr, nullptr, (int)(n / 128), n, k, residual, residual_ld, out_dtype, out, out_ld);
  }
  if (!workspace || workspace_bytes < clefq_gemm_workspace_size(m, k, 4))
    return set_err(CLEFQ_ERR_WORKSPACE, "gemm workspace must hold m*k bytes");
  if (!al16(workspace)) return set_err(CLEFQ_ERR_ALIGN, "workspace must be 16-byte aligned");
  uint8_t *op = static_cast<uint8_t *>(workspace);
  rc = launch_unpack_i4(static_cast<const uint32_t *>(a_codes), a_ld_words, m, (int)k, op, k, s, device_sms());
  if (rc) return cuda_err("unpack launch");
  return run_gemm(s, 4, op, k, m, a_scales, m, w_tiled, w_scales, nullptr, nullptr, (int)(n / 128), n, k, residual,
                  residual_ld, out_dtype, out, out_ld);
}

int clefq_gemm_s8(void *stream, int bits, const void *operand, int64_t operand_ld, const float *a_scales, int64_t m,
                  const void *w_tiled, const float *w_scales, int64_t n, int64_t k, const void *residual,
                  int64_t residual_ld, int out_dtype, void *out, int64_t out_ld) {
  int rc = check_gemm(bits, m, n, k, operand_ld, residual, residual_ld, out_dtype, out_ld);
  if (rc) return rc;
  if (m == 0) return 0;
  return run_gemm(static_cast<cudaStream_t>(stream), bits, static_cast<const uint8_t *>(operand), operand_ld, m,
                  a_scales, m, w_tiled, w_scales, nullptr, nullptr, (int)(n / 128), n, k, residual, residual_ld,
                  out_dtype, out, out_ld);
}

int clefq_gemm_pair_s8(void *stream, const void *operand, int64_t operand_ld, const float *a_scales, int64_t m,
                       const void *w0_tiled, const float *w0_scales, const void *w1_tiled, const float *w1_scales,
                       int64_t n, int64_t k, void *out, int64_t out_ld) {
  int rc = check_gemm(4, m, 2 * n, k, operand_ld, nullptr, 0, CLEFQ_BF16, out_ld);
  if (rc) return rc;
  if (!w0_tiled || !w1_tiled) return set_err(CLEFQ_ERR_SHAPE, "two weight matrices needed");
  if (m == 0) return 0;
  return run_gemm(static_cast<cudaStream_t>(stream), 4, static_cast<const uint8_t *>(operand), operand_ld, m, a_scales,
                  m, w0_tiled, w0_scales, w1_tiled, w1_scales, (int)(n / 128), 2 * n, k, nullptr, 0, CLEFQ_BF16, out,
                  out_ld);
}

int clefq_gemm_swiglu_s8(void *stream, const void *operand, int64_t operand_ld, const float *a_scales, int64_t m,
                         const void *gate_tiled, const float *gate_scales, const void *up_tiled,
                         const float *up_scales, int64_t n, int64_t k, void *out, int64_t out_ld) {
  // the GEMM is 2n wide (gate | up); its SwiGLU output is n wide, checked on its own below
  int rc = check_gemm(4, m, 2 * n, k, operand_ld, nullptr, 0, CLEFQ_BF16, 2 * n);
  if (rc) return rc;
  if (!gate_tiled || !up_tiled) return set_err(CLEFQ_ERR_SHAPE, "two weight matrices needed");
  if (!gemm_swiglu_ok(n, k) || out_ld < n || out_ld % 2)
    return set_err(CLEFQ_ERR_SHAPE, "SwiGLU epilogue needs n % 256 == 0, k >= 2048 and an even out_ld >= n");
  if (m == 0) return 0;
  return run_gemm(static_cast<cudaStream_t>(stream), 4, static_cast<const uint8_t *>(operand), operand_ld, m, a_scales,
                  m, gate_tiled, gate_scales, up_tiled, up_scales, (int)(n / 128), 2 * n, k, nullptr, 0, CLEFQ_BF16,
                  out, out_ld, nullptr, 0, true);
}

int clefq_swiglu(void *stream, const void *gate, const void *up, int64_t n, void *out) {
  if (n < 0) return set_err(CLEFQ_ERR_SHAPE, "SwiGLU shape/dtype mismatch");
  if (n == 0) return 0;
  int rc = launch_swiglu(static_cast<const uint16_t *>(gate), static_cast<const uint16_t *>(up),
                         static_cast<uint16_t *>(out), n, static_cast<cudaStream_t>(stream), device_sms());
  return rc ? cuda_err("swiglu launch") : 0;
}

int clefq_silu(void *stream, const void *x, int64_t n, void *out) {
  if (n < 0) return set_err(CLEFQ_ERR_SHAPE, "SiLU element count");
  if (n == 0) return 0;
  int rc = launch_silu(static_cast<const uint16_t *>(x), static_cast<uint16_t *>(out), n,
                       static_cast<cudaStream_t>(stream), device_sms());
  return rc ? cuda_err("silu launch") : 0;
}

int clefq_route(void *stream, const void *logits, int logits_dtype, int64_t tokens, int experts, int topk,
                float *routes) {
  if (!(topk > 0 && topk <= experts && experts <= 128 && topk <= 32))
    return set_err(CLEFQ_ERR_SHAPE, "invalid expert router shape");
  if (logits_dtype != CLEFQ_BF16 && logits_dtype != CLEFQ_F32) return set_err(CLEFQ_ERR_SHAPE, "logits dtype");
  if (tokens < 0) return set_err(CLEFQ_ERR_SHAPE, "invalid expert router shape");
  int rc = launch_route(logits, logits_dtype == CLEFQ_F32, tokens, experts, topk, routes,
                        static_cast<cudaStream_t>(stream));
  return rc ? cuda_err("route launch") : 0;
}

static Arena group_tables(Arena a, int64_t tokens, int topk, int experts, int **counts, int **offsets, int **tiles,
                          int **perm) {
  const int64_t routes = tokens * topk;
  *counts = a.take<int>(experts + sort_scratch_ints(experts));  // counts, then sort scratch
  *offsets = a.take<int>(experts + 1);
  *tiles = a.take<int>(1 + 2 * ((routes + 127) / 128 + experts));
  *perm = a.take<int>(routes > 0 ? routes : 1);
  return a;
}

int64_t clefq_group_workspace_size(int64_t tokens, int topk, int experts) {
  int *c, *o, *t, *p;
  Arena a{nullptr, INT64_MAX};
  a = group_tables(a, tokens, topk, experts, &c, &o, &t, &p);
  return aligned_total(a);
}

// The MoE blocks' router step: logits given (BF16 or F32), or CLEFQ_ROUTER_WEIGHT_BF16: `logits`
// is the router weight [experts][hidden] and the fused router linear computes them from x.
static int route_step(const void *x, const void *logits, int logits_dtype, int64_t tokens, int64_t hidden,
                      int experts, int topk, float *routes, cudaStream_t s) {
  if (logits_dtype == CLEFQ_ROUTER_WEIGHT_BF16) {
    if (hidden % 64 || experts < 32 || experts % 32 || topk > 8 || !al16(x) || !al16(logits))
      return set_err(CLEFQ_ERR_SHAPE, "the fused router needs hidden %% 64 == 0, experts a multiple of 32 and "
                                      "topk <= 8");
    int *status = device_status_word();
    if (!status) return cuda_err("status word");
    return launch_route_linear(x, logits, tokens, (int)hidden, experts, topk, routes, nullptr, status, s)
               ? cuda_err("fused router launch")
               : 0;
  }
  if (logits_dtype != CLEFQ_BF16 && logits_dtype != CLEFQ_F32) return set_err(CLEFQ_ERR_SHAPE, "logits dtype");
  return launch_route(logits, logits_dtype == CLEFQ_F32, tokens, experts, topk, routes, s) ? cuda_err("routing launch")
                                                                                          : 0;
}

int clefq_route_linear(void *stream, const void *x, const void *router_weight, int64_t tokens, int64_t hidden,
                       int experts, int topk, float *routes, void *logits_out) {
  if (tokens < 0 || tokens > 16777216 || hidden < 64 || hidden > 65536 || hidden % 64 || experts < 32 ||
      experts > 128 || experts % 32 || topk < 1 || topk > 8)
    return set_err(CLEFQ_ERR_SHAPE, "invalid fused router shape (hidden %% 64, experts 32..128 in steps of 32, "
                                    "topk 1..8)");
  if (tokens == 0) return 0;
  if (!al16(x) || !al16(router_weight) || (logits_out && !al16(logits_out)))
    return set_err(CLEFQ_ERR_ALIGN, "router inputs and logits must be 16-byte aligned");
  int *status = device_status_word();
  if (!status) return cuda_err("status word");
  const int rc = launch_route_linear(x, router_weight, tokens, (int)hidden, experts, topk, routes,
                                     static_cast<uint16_t *>(logits_out), status, static_cast<cudaStream_t>(stream));
  return rc ? cuda_err("fused router launch") : 0;
}

int clefq_group_routes(void *stream, const float *routes, int64_t tokens, int topk, int experts, float *groups,
                       float *order, void *workspace, int64_t workspace_bytes) {
  if (tokens < 1 || tokens > 1048576 || topk < 1 || topk > 32 || experts < 1 || experts > 1024)
    return set_err(CLEFQ_ERR_SHAPE, "unsupported Omni route grouping shape");
  int *counts, *offsets, *tiles, *perm;
  Arena a = group_tables(Arena{static_cast<uint8_t *>(workspace), workspace_bytes}, tokens, topk, experts, &counts,
                         &offsets, &tiles, &perm);
  if (!a.ok || !workspace) return set_err(CLEFQ_ERR_WORKSPACE, "group workspace too small");
  int rc = launch_group(routes, tokens, topk, experts, 128, counts, offsets, tiles, perm, groups, order, nullptr,
                        static_cast<cudaStream_t>(stream), device_sms());
  return rc ? cuda_err("group launch") : 0;
}

int clefq_expert_tasks(void *stream, const float *groups, int64_t tokens, int experts, float *tasks) {
  if (tokens < 1 || experts < 1 || experts > 1024) return set_err(CLEFQ_ERR_SHAPE, "unsupported compact Omni routes");
  int rc = launch_tasks(groups, tokens, experts, tasks, static_cast<cudaStream_t>(stream));
  return rc ? cuda_err("tasks launch") : 0;
}

static Arena expert_tables(Arena a, int64_t tokens, int topk, int experts, int64_t k, int **offsets, int **tiles,
                           int **perm, uint8_t **op) {
  const int64_t routes = tokens * topk;
  *offsets = a.take<int>(experts + 1);
  *tiles = a.take<int>(1 + 2 * ((routes + 127) / 128 + experts));
  *perm = a.take<int>(routes > 0 ? routes : 1);
  *op = a.take<uint8_t>(routes * k);
  return a;
}

int64_t clefq_expert_workspace_size(int64_t tokens, int topk, int experts, int64_t k) {
  int *o, *t, *p;
  uint8_t *op;
  Arena a{nullptr, INT64_MAX};
  a = expert_tables(a, tokens, topk, experts, k, &o, &t, &p, &op);
  return aligned_total(a);
}

int clefq_expert(void *stream, const void *a_codes, int64_t a_ld_words, const float *a_scales, const void *w_tiled,
                 const float *w_scales, const float *groups, int64_t tokens, int topk, int experts, int64_t k,
                 int64_t n, int input_routed, void *out, void *workspace, int64_t workspace_bytes) {
  if (tokens < 1 || tokens > 1048576 || topk < 1 || topk > 32 || experts < 1 || experts > 1024)
    return set_err(CLEFQ_ERR_SHAPE, "invalid grouped expert routes");
  if (n < 128 || n % 128 || k < 256 || k % 256 || a_ld_words * 8 < k)
    return set_err(CLEFQ_ERR_SHAPE, "unsupported Omni expert tile shape");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int *offsets, *tiles, *perm;
  uint8_t *op;
  Arena a = expert_tables(Arena{static_cast<uint8_t *>(workspace), workspace_bytes}, tokens, topk, experts, k,
                          &offsets, &tiles, &perm, &op);
  if (!a.ok || !workspace) return set_err(CLEFQ_ERR_WORKSPACE, "expert workspace too small");
  const int64_t routes = tokens * topk;
  const int tile_rows = gemm_tile_rows((int)n, (int)(n / 128));
  int rc = launch_groups_to_sorted(groups, tokens, topk, experts, tile_rows, offsets, perm, tiles, s);
  if (!rc)
    rc = launch_gather_unpack_i4(static_cast<const uint32_t *>(a_codes), a_ld_words, perm, input_routed ? 1 : topk,
                                 routes, (int)k, op, k, s, device_sms());
  if (rc) return cuda_err("expert table launch");
  int *status = device_status_word();
  if (!status) return cuda_err("status word");
  GemmParams p{};
  p.a_op = op;
  p.a_rows = routes;
  p.a_ld = k;
  p.a_scales = a_scales;
  p.w[0] = static_cast<const uint32_t *>(w_tiled);
  p.w_scales[0] = w_scales;
  p.n_split = (int)(n / 128);
  p.n = (int)n;
  p.k = (int)k;
  p.bits = 4;
  p.out = static_cast<uint16_t *>(out);
  p.ldo = n;
  p.grouped = 1;
  p.tile_list = tiles;
  p.expert_offsets = offsets;
  p.perm = perm;
  p.max_tiles = (int)((routes + tile_rows - 1) / tile_rows + experts);
  p.experts = experts;
  p.tile_rows = tile_rows;
  p.topk = topk;
  p.scale_mode = input_routed ? 2 : 1;
  p.scatter = 1;
  p.err = status;
  rc = launch_gemm(p, s);
  if (rc == CLEFQ_ERR_CUDA) return cuda_err("expert gemm launch");
  return rc ? set_err(rc, "unsupported Omni expert tile shape") : 0;
}

int clefq_expert_gate_up(void *stream, const void *a_codes, int64_t a_ld_words, const float *a_scales,
                         const void *gate_tiled, const float *gate_scales, const void *up_tiled, const float *up_scales,
                         const float *groups, int64_t tokens, int topk, int experts, int64_t k, int64_t n, void *out,
                         void *workspace, int64_t workspace_bytes) {
  if (tokens < 1 || tokens > 1048576 || topk < 1 || topk > 32 || experts < 1 || experts > 1024)
    return set_err(CLEFQ_ERR_SHAPE, "invalid grouped expert routes");
  if (n < 256 || n % 256 || k % 256 || a_ld_words * 8 < k || !gemm_swiglu_ok(n, k))
    return set_err(CLEFQ_ERR_SHAPE, "fused gate/up experts need n %% 256 == 0 and k a multiple of 256, >= 2048");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int *offsets, *tiles, *perm;
  uint8_t *op;
  Arena a = expert_tables(Arena{static_cast<uint8_t *>(workspace), workspace_bytes}, tokens, topk, experts, k,
                          &offsets, &tiles, &perm, &op);
  if (!a.ok || !workspace) return set_err(CLEFQ_ERR_WORKSPACE, "expert workspace too small");
  const int64_t routes = tokens * topk;
  const int tile_rows = gemm_tile_rows((int)(2 * n), (int)(n / 128));
  int rc = launch_groups_to_sorted(groups, tokens, topk, experts, tile_rows, offsets, perm, tiles, s);
  if (!rc)
    rc = launch_gather_unpack_i4(static_cast<const uint32_t *>(a_codes), a_ld_words, perm, topk, routes, (int)k, op, k,
                                 s, device_sms());
  if (rc) return cuda_err("expert table launch");
  int *status = device_status_word();
  if (!status) return cuda_err("status word");
  GemmParams p{};
  p.a_op = op;
  p.a_rows = routes;
  p.a_ld = k;
  p.a_scales = a_scales;
  p.w[0] = static_cast<const uint32_t *>(gate_tiled);
  p.w[1] = static_cast<const uint32_t *>(up_tiled);
  p.w_scales[0] = gate_scales;
  p.w_scales[1] = up_scales;
  p.n_split = (int)(n / 128);
  p.n = (int)(2 * n);
  p.k = (int)k;
  p.bits = 4;
  p.out = static_cast<uint16_t *>(out);
  p.ldo = n;
  p.grouped = 1;
  p.tile_list = tiles;
  p.expert_offsets = offsets;
  p.perm = perm;
  p.max_tiles = (int)((routes + tile_rows - 1) / tile_rows + experts);
  p.experts = experts;
  p.tile_rows = tile_rows;
  p.topk = topk;
  p.scale_mode = 1;  // activation scale of the token
  p.scatter = 1;     // hidden row of route r at out row r
  p.swiglu = 1;
  p.silu_tab = silu_table_device();
  p.err = status;
  rc = launch_gemm(p, s);
  if (rc == CLEFQ_ERR_CUDA) return cuda_err("expert gate/up launch");
  return rc ? set_err(rc, "unsupported fused gate/up expert shape") : 0;
}

int clefq_combine(void *stream, const void *values, const float *routes, const float *order, int64_t tokens, int topk,
                  int64_t width, void *out) {
  if (width % 8 || width <= 0 || topk < 1 || topk > 32 || tokens < 0)
    return set_err(CLEFQ_ERR_SHAPE, "unsupported ordered Omni accumulation");
  int rc = launch_combine(static_cast<const uint16_t *>(values), routes, order, tokens, topk, width,
                          static_cast<uint16_t *>(out), static_cast<cudaStream_t>(stream), device_sms());
  if (rc == CLEFQ_ERR_ALIGN) return set_err(rc, "values/out must be 16-byte aligned");
  return rc ? cuda_err("combine launch") : 0;
}

// ---- fused dense MLP -------------------------------------------------------------------
static int64_t stride_for(int64_t k) { return k + (k % 1024 == 0 ? 128 : 0); }

static Arena mlp_tables(Arena a, int64_t m, int64_t hidden, int64_t inter, uint32_t **xq, uint8_t **x8, uint16_t **gu,
                        uint32_t **hq, uint8_t **h8) {
  *xq = a.take<uint32_t>(m * (stride_for(hidden) / 8 + 1));
  *x8 = a.take<uint8_t>(m * hidden);
  *gu = a.take<uint16_t>(m * 2 * inter);
  *hq = a.take<uint32_t>(m * (stride_for(inter) / 8 + 1));
  *h8 = a.take<uint8_t>(m * inter);
  return a;
}

int64_t clefq_mlp_workspace_size(int64_t m, int64_t hidden, int64_t inter) {
  uint32_t *xq, *hq;
  uint8_t *x8, *h8;
  uint16_t *gu;
  Arena a{nullptr, INT64_MAX};
  a = mlp_tables(a, m, hidden, inter, &xq, &x8, &gu, &hq, &h8);
  return aligned_total(a);
}

// The MLP block behind clefq_mlp and clefq_normalized_mlp: norm_weight == NULL packs x as it
// is; otherwise x is RMS-normalised with that weight inside its packing (the reference's
// prepare_norm_with_source) and the un-normalised x is the down projection's residual.
static int run_mlp(cudaStream_t s, const void *x, int64_t m, int64_t hidden, int64_t inter, const void *norm_weight,
                   const void *gate_tiled, const float *gate_scales, const void *up_tiled, const float *up_scales,
                   const void *down_tiled, const float *down_scales, const void *residual, void *out, void *workspace,
                   int64_t workspace_bytes) {
  if (m < 1 || hidden % 256 || inter % 256 || hidden < 256 || inter < 256 || hidden > 32768 || inter > 32768)
    return set_err(CLEFQ_ERR_SHAPE, "unsupported MLP shape");
  uint32_t *xq, *hq;
  uint8_t *x8, *h8;
  uint16_t *gu;
  Arena a = mlp_tables(Arena{static_cast<uint8_t *>(workspace), workspace_bytes}, m, hidden, inter, &xq, &x8, &gu, &hq,
                       &h8);
  if (!a.ok || !workspace) return set_err(CLEFQ_ERR_WORKSPACE, "mlp workspace too small");
  const int64_t sh = stride_for(hidden), si = stride_for(inter);
  int rc = norm_weight ? run_prepare(s, CLEFQ_PREP_NORM, 4, x, hidden, norm_weight, 0, m, hidden, sh, xq, x8, hidden,
                                     nullptr, 0)
                       : run_prepare(s, CLEFQ_PREP_PLAIN, 4, x, hidden, nullptr, 0, m, hidden, sh, xq, x8, hidden,
                                     nullptr, 0);
  if (rc) return rc;
  const float *xs = reinterpret_cast<const float *>(xq + m * (sh / 8));
  // SwiGLU in the gate|up epilogue pays where each tile has enough K stages to hide its extra
  // epilogue work: measured on one box, the C2 block (K = 4096) 0.484 against 0.498 ms, the C3
  // MLP (2048 x 2560 -> 9728, K = 2560) 0.241 against 0.228 ms; identical outputs either way.
  if (gemm_swiglu_ok(inter, hidden) && hidden >= 4096) {
    // gate and up in one launch whose epilogue applies SwiGLU: hidden [m][inter] BF16 (in the
    // gate|up buffer), then plain packing of the hidden rows -- the same values, so the same
    // codes, as SwiGLU fused into the packing of the two projections
    rc = run_gemm(s, 4, x8, hidden, m, xs, m, gate_tiled, gate_scales, up_tiled, up_scales, (int)(inter / 128),
                  2 * inter, hidden, nullptr, 0, CLEFQ_BF16, gu, inter, nullptr, 0, true);
    if (rc) return rc;
    rc = run_prepare(s, CLEFQ_PREP_PLAIN, 4, gu, inter, nullptr, 0, m, inter, si, hq, h8, inter, nullptr, 0);
    if (rc) return rc;
  } else {
    // gate and up in one launch: output columns [0, inter) gate, [inter, 2*inter) up
    rc = run_gemm(s, 4, x8, hidden, m, xs, m, gate_tiled, gate_scales, up_tiled, up_scales, (int)(inter / 128),
                  2 * inter, hidden, nullptr, 0, CLEFQ_BF16, gu, 2 * inter);
    if (rc) return rc;
    rc = run_prepare(s, CLEFQ_PREP_SWIGLU, 4, gu, 2 * inter, gu + inter, 2 * inter, m, inter, si, hq, h8, inter,
                     nullptr, 0);
    if (rc) return rc;
  }
  return run_gemm(s, 4, h8, inter, m, reinterpret_cast<const float *>(hq + m * (si / 8)), m, down_tiled, down_scales,
                  nullptr, nullptr, (int)(hidden / 128), hidden, inter, residual, hidden, CLEFQ_BF16, out, hidden);
}

int clefq_mlp(void *stream, const void *x, int64_t m, int64_t hidden, int64_t inter, const void *gate_tiled,
              const float *gate_scales, const void *up_tiled, const float *up_scales, const void *down_tiled,
              const float *down_scales, const void *residual, void *out, void *workspace, int64_t workspace_bytes) {
  return run_mlp(static_cast<cudaStream_t>(stream), x, m, hidden, inter, nullptr, gate_tiled, gate_scales, up_tiled,
                 up_scales, down_tiled, down_scales, residual, out, workspace, workspace_bytes);
}

int clefq_normalized_mlp(void *stream, const void *x, int64_t m, int64_t hidden, int64_t inter,
                         const void *norm_weight, const void *gate_tiled, const float *gate_scales,
                         const void *up_tiled, const float *up_scales, const void *down_tiled,
                         const float *down_scales, void *out, void *workspace, int64_t workspace_bytes) {
  if (!norm_weight) return set_err(CLEFQ_ERR_SHAPE, "normalized MLP needs the RMSNorm weight");
  return run_mlp(static_cast<cudaStream_t>(stream), x, m, hidden, inter, norm_weight, gate_tiled, gate_scales,
                 up_tiled, up_scales, down_tiled, down_scales, x, out, workspace, workspace_bytes);
}

// ---- tensor-parallel MLP block, collectives fused into its kernels --------------------
// Symmetric region (same offsets on every rank): maxes f32 [world][m] (slot g written by
// rank g), the int4 hidden codes [m][inter/8] (words [g*I/8G, (g+1)*I/8G) of each row written
// by rank g's packing kernel) and the output [m][hidden] (columns [g*H/G, (g+1)*H/G) written
// by rank g's GEMM epilogue).  Codes cross NVLink packed (half the bytes of the s8 operand,
// in whole 32-byte sectors); each rank unpacks the full operand locally.
static Arena tp_region(Arena a, int64_t m, int64_t hidden, int64_t inter, int world, float **maxes, uint32_t **codes,
                       uint16_t **out) {
  *maxes = a.take<float>(world * m);
  *codes = a.take<uint32_t>(m * (inter / 8));
  *out = a.take<uint16_t>(m * hidden);
  return a;
}

static Arena tp_tables(Arena a, int64_t m, int64_t hidden, int64_t inter, int64_t shard, uint32_t **xq, uint8_t **x8,
                       uint16_t **gu, uint32_t **hq, float **mx, uint8_t **h8) {
  *xq = a.take<uint32_t>(m * (stride_for(hidden) / 8 + 1));
  *x8 = a.take<uint8_t>(m * hidden);
  *gu = a.take<uint16_t>(m * 2 * shard);
  *hq = a.take<uint32_t>(m * (shard / 8 + 1));
  *mx = a.take<float>(m);
  *h8 = a.take<uint8_t>(m * inter);
  return a;
}

static int check_tp_mlp(int world, int64_t m, int64_t hidden, int64_t inter) {
  if (world < 1 || world > kMaxRanks || m < 1 || hidden < 256 || inter < 256 || hidden > 32768 || inter > 32768 ||
      inter % (256 * world) || hidden % (256 * world))
    return set_err(CLEFQ_ERR_SHAPE,
                   "unsupported tensor-parallel MLP shape: each rank needs whole 256-groups of the intermediate "
                   "and a multiple of 256 output columns");
  return 0;
}

int64_t clefq_tp_mlp_region_bytes(int64_t m, int64_t hidden, int64_t inter, int world) {
  if (check_tp_mlp(world, m, hidden, inter)) return -1;
  float *mx;
  uint32_t *codes;
  uint16_t *out;
  return aligned_total(tp_region(Arena{nullptr, INT64_MAX}, m, hidden, inter, world, &mx, &codes, &out));
}

int64_t clefq_tp_mlp_workspace_size(int64_t m, int64_t hidden, int64_t inter, int world) {
  if (check_tp_mlp(world, m, hidden, inter)) return -1;
  uint32_t *xq, *hq;
  uint8_t *x8, *h8;
  uint16_t *gu;
  float *mx;
  return aligned_total(
      tp_tables(Arena{nullptr, INT64_MAX}, m, hidden, inter, inter / world, &xq, &x8, &gu, &hq, &mx, &h8));
}

int clefq_tp_mlp(clefq_comm *c, void *stream, const void *x, int64_t m, int64_t hidden, int64_t inter,
                 const void *gate_tiled, const float *gate_scales, const void *up_tiled, const float *up_scales,
                 const void *down_tiled, const float *down_scales, const void *residual, void *out, void *workspace,
                 int64_t workspace_bytes) {
  if (!clefq_comm_ready(c)) return set_err(CLEFQ_ERR_SHAPE, "tensor-parallel MLP: communicator peers not opened");
  int rc = check_tp_mlp(c->world, m, hidden, inter);
  if (rc) return rc;
  if (!x || !out) return set_err(CLEFQ_ERR_SHAPE, "tensor-parallel MLP: null input or output");
  if (!al16(x) || (residual && !al16(residual))) return set_err(CLEFQ_ERR_ALIGN, "x and residual must be 16-byte aligned");
  const int world = c->world, rank = c->rank;
  const int64_t shard = inter / world, cols = hidden / world;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float *maxes;
  uint32_t *codes;
  uint16_t *rout;
  Arena region = tp_region(Arena{c->base + kCommHeader, c->bytes}, m, hidden, inter, world, &maxes, &codes, &rout);
  if (!region.ok) return set_err(CLEFQ_ERR_WORKSPACE, "communicator region too small for this MLP block");
  uint32_t *xq, *hq;
  uint8_t *x8, *h8;
  uint16_t *gu;
  float *mx;
  Arena a = tp_tables(Arena{static_cast<uint8_t *>(workspace), workspace_bytes}, m, hidden, inter, shard, &xq, &x8,
                      &gu, &hq, &mx, &h8);
  if (!a.ok || !workspace) return set_err(CLEFQ_ERR_WORKSPACE, "tensor-parallel MLP workspace too small");
  int *status = device_status_word();
  if (!status) return cuda_err("status word");
  // the same object in rank g's region
  auto at = [&](int g, const void *p) { return c->peer[g] + (static_cast<const uint8_t *>(p) - c->base); };
  const int64_t sh = stride_for(hidden);
  // 1. x packed on every rank; gate|up of this rank's intermediate rows
  rc = run_prepare(s, CLEFQ_PREP_PLAIN, 4, x, hidden, nullptr, 0, m, hidden, sh, xq, x8, hidden, nullptr, 0);
  if (rc) return rc;
  rc = run_gemm(s, 4, x8, hidden, m, reinterpret_cast<const float *>(xq + m * (sh / 8)), m, gate_tiled, gate_scales,
                up_tiled, up_scales, (int)(shard / 128), 2 * shard, hidden, nullptr, 0, CLEFQ_BF16, gu, 2 * shard);
  if (rc) return rc;
  // 2. |Hadamard| row maxima of the SwiGLU shard into this rank's slot; the barrier stores the
  //    slot into every peer and reduces the slots to the full-row maxima
  float *slot = maxes + rank * m;
  rc = run_prepare(s, CLEFQ_PREP_SWIGLU, 4, gu, 2 * shard, gu + shard, 2 * shard, m, shard, shard, nullptr, nullptr,
                   0, nullptr, 0, slot, nullptr);
  if (rc) return rc;
  CommBarrierArgs b = comm_barrier_args(c, status);
  b.src = reinterpret_cast<const uint32_t *>(slot);
  for (int g = 0; g < world; ++g) b.dst[g] = reinterpret_cast<uint32_t *>(at(g, slot));
  b.words = m;
  b.maxes = maxes;
  b.mx = mx;
  b.m = m;
  if ((rc = launch_comm_barrier(b, s))) return rc;
  // 3. the shard quantised with the full-row maxima; its code words go into every rank's
  //    code buffer (this rank's included); after the barrier the full rows are unpacked
  uint32_t *code_cols = codes + rank * (shard / 8);
  uint32_t *code_dst[kMaxRanks];
  uint16_t *out_peer[kMaxPeers];
  uint16_t *out_cols = rout + rank * cols;
  int np = 0;
  for (int g = 0; g < world; ++g) {
    code_dst[g] = reinterpret_cast<uint32_t *>(at(g, code_cols));
    if (g != rank) out_peer[np++] = reinterpret_cast<uint16_t *>(at(g, out_cols));
  }
  rc = run_prepare(s, CLEFQ_PREP_SWIGLU, 4, gu, 2 * shard, gu + shard, 2 * shard, m, shard, shard, hq, nullptr, 0,
                   nullptr, 0, nullptr, mx, code_dst, world, inter / 8);
  if (rc) return rc;
  if ((rc = launch_comm_barrier(comm_barrier_args(c, status), s))) return rc;
  if (launch_unpack_i4(codes, inter / 8, m, (int)inter, h8, inter, s, device_sms()))
    return cuda_err("tensor-parallel MLP operand unpack");
  // 4. down GEMM of this rank's output columns over the full operand, stored into every
  //    rank's output buffer
  const uint16_t *res_cols = residual ? static_cast<const uint16_t *>(residual) + rank * cols : nullptr;
  rc = run_gemm(s, 4, h8, inter, m, reinterpret_cast<const float *>(hq + m * (shard / 8)), m, down_tiled, down_scales,
                nullptr, nullptr, (int)(cols / 128), cols, inter, res_cols, hidden, CLEFQ_BF16, out_cols, hidden,
                out_peer, np);
  if (rc) return rc;
  if ((rc = launch_comm_barrier(comm_barrier_args(c, status), s))) return rc;
  if (out != rout && cudaMemcpyAsync(out, rout, m * hidden * 2, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return cuda_err("tensor-parallel MLP output copy");
  return 0;
}

void *clefq_tp_mlp_output(clefq_comm *c, int64_t m, int64_t hidden, int64_t inter) {
  if (!c || check_tp_mlp(c->world, m, hidden, inter)) return nullptr;
  float *maxes;
  uint32_t *codes;
  uint16_t *rout;
  Arena region = tp_region(Arena{c->base + kCommHeader, c->bytes}, m, hidden, inter, c->world, &maxes, &codes, &rout);
  return region.ok ? rout : nullptr;
}

// ---- grouped expert FFN shared by the fused MoE block and the expert-parallel path ----
// xs: expert-sorted s8 operand rows (route order given by perm); a_scales: the token
// scale of route r at a_scales[r / topk].  Writes values[route] = down(SwiGLU(gate|up)).
// Expert-parallel variant: nroutes is the capacity and rows_dev the routes present (a
// count on the device).
static int run_expert_ffn(cudaStream_t s, const uint8_t *xs, int64_t nroutes, const float *a_scales, int topk,
                          const int *tiles, const int *offsets, const int *perm, int experts, int tile_rows,
                          int64_t hidden, int64_t inter, const void *gate_tiled, const float *gate_scales,
                          const void *up_tiled, const float *up_scales, const void *down_tiled,
                          const float *down_scales, uint16_t *gu, uint32_t *hq, uint8_t *h8, uint16_t *values,
                          const int64_t *rows_dev = nullptr) {
  int *status = device_status_word();
  if (!status) return cuda_err("status word");
  GemmParams p{};
  p.a_op = xs;
  p.a_rows = nroutes;
  p.a_ld = hidden;
  p.a_scales = a_scales;
  p.w[0] = static_cast<const uint32_t *>(gate_tiled);
  p.w[1] = static_cast<const uint32_t *>(up_tiled);
  p.w_scales[0] = gate_scales;
  p.w_scales[1] = up_scales;
  p.n_split = (int)(inter / 128);
  p.n = (int)(2 * inter);
  p.k = (int)hidden;
  p.bits = 4;
  p.out = gu;
  p.ldo = 2 * inter;
  p.grouped = 1;
  p.tile_list = tiles;
  p.expert_offsets = offsets;
  p.perm = perm;
  p.max_tiles = (int)((nroutes + tile_rows - 1) / tile_rows + experts);
  p.experts = experts;
  p.tile_rows = tile_rows;
  p.topk = topk;
  p.scale_mode = 1;  // activation scale of the token
  p.scatter = 0;     // rows stay in expert-sorted order
  p.err = status;
  int rc = launch_gemm(p, s);
  if (rc) return rc == CLEFQ_ERR_CUDA ? cuda_err("expert gate/up launch") : set_err(rc, "expert gate/up shape");
  // SwiGLU fused into the packing of the hidden rows (still expert-sorted).  The gate|up
  // launch with SwiGLU in its epilogue (clefq_expert_gate_up) measured 0.656 against 0.571 ms
  // for the C4 layer (0.641 against 0.564 with table lookups for SiLU).  The likely cause is
  // its two 8 KB weight boxes per 192-token stage, one per weight map, where the plain launch
  // moves one 16 KB box: the TMA unit's rate is per box.
  rc = run_prepare(s, CLEFQ_PREP_SWIGLU, 4, gu, 2 * inter, gu + inter, 2 * inter, nroutes, inter, inter, hq, h8, inter,
                   nullptr, 0, nullptr, nullptr, nullptr, 0, 0, rows_dev);
  if (rc) return rc;
  p.a_op = h8;
  p.a_ld = inter;
  p.a_scales = reinterpret_cast<const float *>(hq + nroutes * (inter / 8));
  p.w[0] = static_cast<const uint32_t *>(down_tiled);
  p.w[1] = nullptr;
  p.w_scales[0] = down_scales;
  p.w_scales[1] = nullptr;
  p.n_split = (int)(hidden / 128);
  p.n = (int)hidden;
  p.k = (int)inter;
  p.out = values;
  p.ldo = hidden;
  p.scale_mode = 0;  // hidden rows were packed in sorted order
  p.scatter = 1;     // values land at their route id
  rc = launch_gemm(p, s);
  if (rc) return rc == CLEFQ_ERR_CUDA ? cuda_err("expert down launch") : set_err(rc, "expert down shape");
  return 0;
}

// ---- fused Omni MoE block --------------------------------------------------------------
struct MoeTables {
  float *routes, *order;
  int *counts, *offsets, *tiles, *perm, *slots;
  uint32_t *xq, *hq;
  uint8_t *x8, *xs, *h8;
  uint16_t *gu, *values;
};
static Arena moe_tables(Arena a, int64_t tokens, int64_t hidden, int64_t inter, int experts, int topk, MoeTables &t) {
  const int64_t routes = tokens * topk;
  t.routes = a.take<float>(tokens * 2 * topk);
  t.order = a.take<float>(tokens * topk);
  t.counts = a.take<int>(experts + sort_scratch_ints(experts));  // counts, then sort scratch
  t.offsets = a.take<int>(experts + 1);
  t.tiles = a.take<int>(1 + 2 * ((routes + 127) / 128 + experts));
  t.perm = a.take<int>(routes);
  t.slots = a.take<int>(routes);
  t.xq = a.take<uint32_t>(tokens * (stride_for(hidden) / 8 + 1));
  t.x8 = a.take<uint8_t>(tokens * hidden);
  t.xs = a.take<uint8_t>(routes * hidden);
  t.gu = a.take<uint16_t>(routes * 2 * inter);
  t.hq = a.take<uint32_t>(routes * (inter / 8 + 1));
  t.h8 = a.take<uint8_t>(routes * inter);
  t.values = a.take<uint16_t>(routes * hidden);
  return a;
}

int64_t clefq_moe_workspace_size(int64_t tokens, int64_t hidden, int64_t inter, int experts, int topk) {
  MoeTables t;
  Arena a{nullptr, INT64_MAX};
  a = moe_tables(a, tokens, hidden, inter, experts, topk, t);
  return aligned_total(a);
}

int clefq_moe(void *stream, const void *x, const void *logits, int logits_dtype, int64_t tokens, int64_t hidden,
              int64_t inter, int experts, int topk, const void *gate_tiled, const float *gate_scales,
              const void *up_tiled, const float *up_scales, const void *down_tiled, const float *down_scales,
              void *out, float *routes_out, void *workspace, int64_t workspace_bytes) {
  if (tokens < 1 || tokens > 1048576 || hidden % 256 || inter % 256 || hidden < 256 || inter < 256 ||
      hidden > 32768 || inter > 32768 || !(topk > 0 && topk <= experts && experts <= 128 && topk <= 32))
    return set_err(CLEFQ_ERR_SHAPE, "unsupported Omni MoE shape");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  MoeTables t;
  Arena a = moe_tables(Arena{static_cast<uint8_t *>(workspace), workspace_bytes}, tokens, hidden, inter, experts, topk,
                       t);
  if (!a.ok || !workspace) return set_err(CLEFQ_ERR_WORKSPACE, "moe workspace too small");
  float *routes = routes_out ? routes_out : t.routes;
  const int64_t nroutes = tokens * topk;
  const int sms = device_sms();
  // One tile list serves both expert GEMMs: both must run the same kernel family.
  const int tile_rows = gemm_tile_rows((int)(2 * inter), (int)(inter / 128));
  if (gemm_tile_rows((int)hidden, (int)(hidden / 128)) != tile_rows) {
    return set_err(CLEFQ_ERR_SHAPE, "hidden and intermediate must both be multiples of 256, or neither");
  }
  int rc = route_step(x, logits, logits_dtype, tokens, hidden, experts, topk, routes, s);
  if (rc) return rc;
  // the stable grouping also gives every route its expert-sorted row (slots; -1 for a route
  // left out), so packing x can write each token's operand straight to its routes' rows
  if (cudaMemsetAsync(t.slots, 0xff, sizeof(int) * nroutes, s) != cudaSuccess) return cuda_err("slot reset");
  {
    SortArgs g{};
    g.routes = routes;
    g.route_ld = 2 * topk;
    g.tokens = tokens;
    g.topk = topk;
    g.items = nroutes;
    g.key_div = 1;
    g.keys = experts;
    g.dedupe = true;
    g.hist = t.counts + experts;
    g.counts = t.counts;
    g.offsets = t.offsets;
    g.tile_list = t.tiles;
    g.tile_rows = tile_rows;
    g.perm = t.perm;
    g.slots = t.slots;
    g.order = t.order;
    if (launch_sort(g, s)) return cuda_err("routing launch");
  }
  const int64_t sh = stride_for(hidden);
  if (topk <= kMaxDup && hidden <= 16384) {
    rc = run_prepare(s, CLEFQ_PREP_PLAIN, 4, x, hidden, nullptr, 0, tokens, hidden, sh, t.xq, t.xs, hidden, nullptr, 0,
                     nullptr, nullptr, nullptr, 0, 0, nullptr, t.slots, topk);
    if (rc) return rc;
  } else {
    rc = run_prepare(s, CLEFQ_PREP_PLAIN, 4, x, hidden, nullptr, 0, tokens, hidden, sh, t.xq, t.x8, hidden, nullptr,
                     0);
    if (rc) return rc;
    rc = launch_gather(t.x8, hidden, t.perm, topk, nroutes, hidden, t.xs, hidden, s, sms);
    if (rc) return cuda_err("gather launch");
  }
  rc = run_expert_ffn(s, t.xs, nroutes, reinterpret_cast<const float *>(t.xq + tokens * (sh / 8)), topk, t.tiles,
                      t.offsets, t.perm, experts, tile_rows, hidden, inter, gate_tiled, gate_scales, up_tiled,
                      up_scales, down_tiled, down_scales, t.gu, t.hq, t.h8, t.values);
  if (rc) return rc;
  rc = launch_combine(t.values, routes, t.order, tokens, topk, hidden, static_cast<uint16_t *>(out), s, sms);
  return rc ? cuda_err("combine launch") : 0;
}


// ---- expert-parallel Omni MoE ----------------------------------------------------------
// No reference counterpart (the reference runs the layer on one GPU); the pieces around
// the two all-to-all exchanges a host makes.  Record of one dispatched route: the token's
// hidden/8 code words, its f32 scale, the global expert id, the probability, padding to
// 16 bytes.
int64_t clefq_moe_ep_record_bytes(int64_t hidden) { return ((hidden / 8 + 3) * 4 + 15) / 16 * 16; }

static int check_ep_shape(int64_t tokens, int64_t hidden, int experts, int topk, int world) {
  if (tokens < 0 || tokens > 1048576 || hidden % 256 || hidden < 256 || hidden > 32768 ||
      !(topk > 0 && topk <= experts && experts <= 128 && topk <= 32) || world < 1 || world > 64 || experts % world)
    return set_err(CLEFQ_ERR_SHAPE, "unsupported expert-parallel MoE shape");
  return 0;
}

int64_t clefq_moe_ep_plan_workspace_size(int world) {
  return world < 1 || world > 64 ? -1 : (sort_scratch_ints(world) * 4 + 255) & ~int64_t(255);
}

int clefq_moe_ep_plan(void *stream, const float *routes, int64_t tokens, int topk, int experts, int world,
                      int64_t *send_counts, int32_t *send_slots, void *workspace, int64_t workspace_bytes) {
  int rc = check_ep_shape(tokens, 256, experts, topk, world);
  if (rc) return rc;
  if (tokens > 0 && (!routes || !send_slots)) return set_err(CLEFQ_ERR_SHAPE, "null routes or slots");
  if (!send_counts) return set_err(CLEFQ_ERR_SHAPE, "null send counts");
  if (!workspace || workspace_bytes < clefq_moe_ep_plan_workspace_size(world))
    return set_err(CLEFQ_ERR_WORKSPACE, "expert-parallel plan workspace too small");
  rc = launch_ep_plan(routes, tokens, topk, experts, world, reinterpret_cast<long long *>(send_counts), send_slots,
                      static_cast<int *>(workspace), static_cast<cudaStream_t>(stream));
  return rc ? cuda_err("expert-parallel plan launch") : 0;
}

int clefq_moe_ep_pack(void *stream, const void *a_codes, int64_t a_ld_words, const float *a_scales, int64_t tokens,
                      int64_t hidden, const float *routes, int topk, const int32_t *send_slots, void *send_records) {
  int rc = check_ep_shape(tokens, hidden, topk, topk, 1);
  if (rc) return rc;
  if (a_ld_words < hidden / 8 || (a_ld_words & 3) || !al16(a_codes) || !al16(send_records))
    return set_err(CLEFQ_ERR_ALIGN, "codes and records must be 16-byte aligned rows");
  rc = launch_ep_pack(static_cast<const uint32_t *>(a_codes), a_ld_words, a_scales, routes, send_slots, tokens, topk,
                      (int)(hidden / 8), clefq_moe_ep_record_bytes(hidden) / 4, static_cast<uint32_t *>(send_records),
                      static_cast<cudaStream_t>(stream), device_sms());
  return rc ? cuda_err("expert-parallel pack launch") : 0;
}

struct EpTables {
  float *routes, *scales;
  int *counts, *offsets, *tiles, *perm;
  uint8_t *xs, *h8;
  uint16_t *gu, *values;
  uint32_t *hq;
};
static Arena ep_tables(Arena a, int64_t n, int64_t hidden, int64_t inter, int local_experts, EpTables &t) {
  const int64_t rows = n > 0 ? n : 1;
  t.routes = a.take<float>(2 * rows);
  t.scales = a.take<float>(rows);
  t.counts = a.take<int>(local_experts + sort_scratch_ints(local_experts));  // counts, then sort scratch
  t.offsets = a.take<int>(local_experts + 1);
  t.tiles = a.take<int>(1 + 2 * ((rows + 127) / 128 + local_experts));
  t.perm = a.take<int>(rows);
  t.xs = a.take<uint8_t>(rows * hidden);
  t.gu = a.take<uint16_t>(rows * 2 * inter);
  t.hq = a.take<uint32_t>(rows * (inter / 8 + 1));
  t.h8 = a.take<uint8_t>(rows * inter);
  t.values = a.take<uint16_t>(rows * hidden);
  return a;
}

int64_t clefq_moe_ep_experts_workspace_size(int64_t records, int64_t hidden, int64_t inter, int local_experts) {
  EpTables t;
  Arena a{nullptr, INT64_MAX};
  a = ep_tables(a, records, hidden, inter, local_experts, t);
  return aligned_total(a);
}

int clefq_moe_ep_experts(void *stream, const void *records, int64_t n, int64_t hidden, int64_t inter, int expert_base,
                         int local_experts, const void *gate_tiled, const float *gate_scales, const void *up_tiled,
                         const float *up_scales, const void *down_tiled, const float *down_scales, void *products,
                         void *workspace, int64_t workspace_bytes) {
  if (n < 0 || n > 32 * 1048576 || hidden % 256 || inter % 256 || hidden < 256 || inter < 256 || hidden > 32768 ||
      inter > 32768 || local_experts < 1 || local_experts > 128 || expert_base < 0)
    return set_err(CLEFQ_ERR_SHAPE, "unsupported expert-parallel expert shape");
  if (n == 0) return 0;
  if (!al16(records) || !al16(products)) return set_err(CLEFQ_ERR_ALIGN, "records and products must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  EpTables t;
  Arena a = ep_tables(Arena{static_cast<uint8_t *>(workspace), workspace_bytes}, n, hidden, inter, local_experts, t);
  if (!a.ok || !workspace) return set_err(CLEFQ_ERR_WORKSPACE, "expert-parallel workspace too small");
  const int sms = device_sms();
  const int tile_rows = gemm_tile_rows((int)(2 * inter), (int)(inter / 128));
  if (gemm_tile_rows((int)hidden, (int)(hidden / 128)) != tile_rows)
    return set_err(CLEFQ_ERR_SHAPE, "hidden and intermediate must both be multiples of 256, or neither");
  const int code_words = (int)(hidden / 8);
  const int64_t rec_words = clefq_moe_ep_record_bytes(hidden) / 4;
  const uint32_t *recv = static_cast<const uint32_t *>(records);
  int rc = launch_ep_unpack_meta(recv, n, code_words, rec_words, expert_base, local_experts, t.scales, t.routes, s, sms);
  if (!rc)
    rc = launch_group(t.routes, n, 1, local_experts, tile_rows, t.counts, t.offsets, t.tiles, t.perm, nullptr, nullptr,
                      nullptr, s, sms);
  if (!rc) rc = launch_gather_unpack_i4(recv, rec_words, t.perm, 1, n, (int)hidden, t.xs, hidden, s, sms);
  if (rc) return cuda_err("expert-parallel grouping launch");
  rc = run_expert_ffn(s, t.xs, n, t.scales, 1, t.tiles, t.offsets, t.perm, local_experts, tile_rows, hidden, inter,
                      gate_tiled, gate_scales, up_tiled, up_scales, down_tiled, down_scales, t.gu, t.hq, t.h8, t.values);
  if (rc) return rc;
  rc = launch_ep_weigh(t.values, t.routes, n, hidden, static_cast<uint16_t *>(products), s, sms);
  return rc ? cuda_err("expert-parallel weigh launch") : 0;
}

int clefq_moe_ep_combine(void *stream, const void *products, const int32_t *send_slots, const float *routes,
                         int64_t tokens, int topk, int64_t hidden, void *out) {
  int rc = check_ep_shape(tokens, hidden, topk, topk, 1);
  if (rc) return rc;
  if (!al16(products) || !al16(out)) return set_err(CLEFQ_ERR_ALIGN, "products and output must be 16-byte aligned");
  rc = launch_ep_combine(static_cast<const uint16_t *>(products), send_slots, routes, tokens, topk, hidden,
                         static_cast<uint16_t *>(out), static_cast<cudaStream_t>(stream), device_sms());
  return rc ? cuda_err("expert-parallel combine launch") : 0;
}

// ---- expert-parallel Omni MoE layer, exchanges fused into its kernels --------------------
// Symmetric region (same offsets on every rank): the counts matrix int [world][world], the
// receive buffer [recv_cap][record], then this rank's products [tokens * topk][hidden] BF16
// (written by the expert ranks' down-GEMM epilogues at the home route index).
static Arena ep_region(Arena a, int64_t tokens, int64_t hidden, int topk, int world, int64_t recv_cap, int **counts,
                       uint32_t **recv, uint16_t **products) {
  *counts = a.take<int>((int64_t)world * world);
  *recv = a.take<uint32_t>(recv_cap * (clefq_moe_ep_record_bytes(hidden) / 4));
  *products = a.take<uint16_t>((tokens > 0 ? tokens : 1) * topk * hidden);
  return a;
}

struct EpLayerTables {
  float *routes, *xs_scales, *rmeta, *ret_prob;
  uint32_t *xq, *hq;
  int *slots, *scratch, *offsets, *tiles, *perm, *ret_rank, *ret_row;
  int64_t *n_dev;
  uint8_t *xs, *h8;
  uint16_t *gu;
  uint16_t *vals;  // down-projection values [cap][hidden], over xs and gu (dead by then)
};

static Arena ep_layer_tables(Arena a, int64_t tokens, int64_t hidden, int64_t inter, int experts, int topk, int world,
                             int64_t cap, EpLayerTables &t) {
  const int local = experts / world;
  const int64_t rows = cap > 0 ? cap : 1;
  const int keys = local > world ? local : world;
  t.routes = a.take<float>((tokens > 0 ? tokens : 1) * 2 * topk);
  t.xq = a.take<uint32_t>((tokens > 0 ? tokens : 1) * (stride_for(hidden) / 8 + 1));
  t.slots = a.take<int>((tokens > 0 ? tokens : 1) * topk);
  t.scratch = a.take<int>(sort_scratch_ints(keys));
  t.n_dev = a.take<int64_t>(1);
  t.xs_scales = a.take<float>(rows);
  t.rmeta = a.take<float>(2 * rows);
  t.ret_prob = a.take<float>(rows);
  t.ret_rank = a.take<int>(rows);
  t.ret_row = a.take<int>(rows);
  t.offsets = a.take<int>(local + 1);
  t.tiles = a.take<int>(1 + 2 * ((rows + 127) / 128 + local));
  t.perm = a.take<int>(rows);
  t.xs = a.take<uint8_t>(rows * hidden);
  t.gu = a.take<uint16_t>(rows * 2 * inter);
  // xs and gu are contiguous (both sizes are multiples of 256 bytes); the values need
  // rows * hidden * 2 bytes from xs on, so extend the span when 4 * inter < hidden
  if (hidden > 4 * inter) a.take<uint8_t>(rows * (hidden - 4 * inter));
  t.vals = reinterpret_cast<uint16_t *>(t.xs);
  t.hq = a.take<uint32_t>(rows * (inter / 8 + 1));
  t.h8 = a.take<uint8_t>(rows * inter);
  return a;
}

static int check_ep_layer(int64_t tokens, int64_t hidden, int64_t inter, int experts, int topk, int world,
                          int64_t recv_cap) {
  if (tokens < 0 || tokens > 1048576 || hidden % 256 || inter % 256 || hidden < 256 || inter < 256 ||
      hidden > 32768 || inter > 32768 || !(topk > 0 && topk <= experts && experts <= 128 && topk <= 32) ||
      world < 1 || world > kMaxRanks || experts % world || recv_cap < 0 || recv_cap > 32 * 1048576)
    return set_err(CLEFQ_ERR_SHAPE, "unsupported expert-parallel MoE layer shape");
  return 0;
}

int64_t clefq_moe_ep_layer_region_bytes(int64_t tokens, int64_t hidden, int topk, int world, int64_t recv_cap) {
  if (check_ep_layer(tokens, hidden, 256, topk, topk, world, recv_cap)) return -1;
  int *c;
  uint32_t *r;
  uint16_t *p;
  return aligned_total(ep_region(Arena{nullptr, INT64_MAX}, tokens, hidden, topk, world, recv_cap, &c, &r, &p));
}

int64_t clefq_moe_ep_layer_workspace_size(int64_t tokens, int64_t hidden, int64_t inter, int experts, int topk,
                                          int world, int64_t recv_cap) {
  if (check_ep_layer(tokens, hidden, inter, experts, topk, world, recv_cap)) return -1;
  EpLayerTables t;
  return aligned_total(
      ep_layer_tables(Arena{nullptr, INT64_MAX}, tokens, hidden, inter, experts, topk, world, recv_cap, t));
}

int clefq_moe_ep_layer(clefq_comm *c, void *stream, const void *x, const void *logits, int logits_dtype,
                       int64_t tokens, int64_t hidden, int64_t inter, int experts, int topk, int64_t recv_cap,
                       const void *gate_tiled, const float *gate_scales, const void *up_tiled,
                       const float *up_scales, const void *down_tiled, const float *down_scales, void *out,
                       float *routes_out, void *workspace, int64_t workspace_bytes) {
  if (!clefq_comm_ready(c)) return set_err(CLEFQ_ERR_SHAPE, "expert-parallel layer: communicator peers not opened");
  const int world = c->world, rank = c->rank;
  int rc = check_ep_layer(tokens, hidden, inter, experts, topk, world, recv_cap);
  if (rc) return rc;
  if (logits_dtype != CLEFQ_BF16 && logits_dtype != CLEFQ_F32 && logits_dtype != CLEFQ_ROUTER_WEIGHT_BF16) return set_err(CLEFQ_ERR_SHAPE, "logits dtype");
  if ((tokens > 0 && (!x || !logits || !out)) || (tokens > 0 && (!al16(x) || !al16(out))))
    return set_err(CLEFQ_ERR_ALIGN, "x and out must be 16-byte aligned");
  const int local = experts / world;
  const int tile_rows = gemm_tile_rows((int)(2 * inter), (int)(inter / 128));
  // hidden and intermediate are multiples of 256, so both expert GEMMs run the 2-SM kernel,
  // whose epilogue holds the return path
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int *counts;
  uint32_t *recv;
  uint16_t *products;
  Arena region = ep_region(Arena{c->base + kCommHeader, c->bytes}, tokens, hidden, topk, world, recv_cap, &counts,
                           &recv, &products);
  if (!region.ok) return set_err(CLEFQ_ERR_WORKSPACE, "communicator region too small for this MoE layer");
  EpLayerTables t;
  Arena a = ep_layer_tables(Arena{static_cast<uint8_t *>(workspace), workspace_bytes}, tokens, hidden, inter, experts,
                            topk, world, recv_cap, t);
  if (!a.ok || !workspace) return set_err(CLEFQ_ERR_WORKSPACE, "expert-parallel layer workspace too small");
  int *status = device_status_word();
  if (!status) return cuda_err("status word");
  auto at = [&](int g, const void *p) { return c->peer[g] + (static_cast<const uint8_t *>(p) - c->base); };
  const int sms = device_sms();
  const int code_words = (int)(hidden / 8);
  const int64_t rec_words = clefq_moe_ep_record_bytes(hidden) / 4;
  const int64_t sh = stride_for(hidden);
  float *routes = routes_out ? routes_out : t.routes;
  int *my_counts = counts + rank * world;
  // 1. route and pack this rank's tokens; plan: routes grouped by destination rank
  if (tokens > 0) {
    rc = route_step(x, logits, logits_dtype, tokens, hidden, experts, topk, routes, s);
    if (rc) return rc;
    rc = run_prepare(s, CLEFQ_PREP_PLAIN, 4, x, hidden, nullptr, 0, tokens, hidden, sh, t.xq, nullptr, 0, nullptr, 0);
    if (rc) return rc;
  }
  SortArgs plan{};
  plan.routes = routes;
  plan.route_ld = 2 * topk;
  plan.tokens = tokens;
  plan.topk = topk;
  plan.items = tokens * topk;
  plan.key_div = local;
  plan.keys = world;
  plan.dedupe = false;
  plan.hist = t.scratch;
  plan.counts = my_counts;  // this rank's row of the matrix
  plan.slots = t.slots;
  if ((rc = launch_sort(plan, s))) return cuda_err("expert-parallel plan launch");
  // 2. barrier: every rank's row of the counts matrix into every peer
  CommBarrierArgs b = comm_barrier_args(c, status);
  b.src = reinterpret_cast<const uint32_t *>(my_counts);
  for (int g = 0; g < world; ++g) b.dst[g] = reinterpret_cast<uint32_t *>(at(g, my_counts));
  b.words = world;
  if ((rc = launch_comm_barrier(b, s))) return rc;
  // 3. dispatch: records stored straight into the destination ranks' receive buffers
  EpDispatchArgs d{};
  d.xq = t.xq;
  d.words_ld = sh / 8;
  d.scales = reinterpret_cast<const float *>(t.xq + tokens * (sh / 8));
  d.routes = routes;
  d.slots = t.slots;
  d.tokens = tokens;
  d.topk = topk;
  d.per_rank = local;
  d.counts = counts;
  d.rank = rank;
  d.world = world;
  d.code_words = code_words;
  d.rec_words = rec_words;
  for (int g = 0; g < world; ++g) d.recv[g] = reinterpret_cast<uint32_t *>(at(g, recv));
  d.recv_cap = recv_cap;
  d.err = status;
  if ((rc = launch_ep_dispatch(d, s, sms))) return cuda_err("expert-parallel dispatch launch");
  if ((rc = launch_comm_barrier(comm_barrier_args(c, status), s))) return rc;
  // 4. the received routes: metadata, grouping by local expert, expert-sorted operand
  EpReceiveArgs r{};
  r.recv = recv;
  r.counts = counts;
  r.rank = rank;
  r.world = world;
  r.code_words = code_words;
  r.rec_words = rec_words;
  r.recv_cap = recv_cap;
  r.expert_base = rank * local;
  r.local_experts = local;
  r.scales = t.xs_scales;
  r.routes = t.rmeta;
  r.ret_rank = t.ret_rank;
  r.ret_row = t.ret_row;
  r.ret_prob = t.ret_prob;
  r.n_dev = t.n_dev;
  r.err = status;
  if ((rc = launch_ep_receive(r, s, sms))) return cuda_err("expert-parallel receive launch");
  SortArgs grp{};
  grp.routes = t.rmeta;
  grp.route_ld = 2;
  grp.tokens = recv_cap;
  grp.topk = 1;
  grp.items = recv_cap;
  grp.items_dev = t.n_dev;
  grp.key_div = 1;
  grp.keys = local;
  grp.dedupe = false;
  grp.hist = t.scratch;
  grp.offsets = t.offsets;
  grp.tile_list = t.tiles;
  grp.tile_rows = tile_rows;
  grp.perm = t.perm;
  if ((rc = launch_sort(grp, s))) return cuda_err("expert-parallel grouping launch");
  if (recv_cap > 0 && launch_gather_unpack_i4(recv, rec_words, t.perm, 1, recv_cap, (int)hidden, t.xs, hidden, s, sms,
                                              t.n_dev))
    return cuda_err("expert-parallel gather launch");
  // 5. expert FFN with the values in received-route order, then each product goes home:
  //    bf16(value * probability) into the home rank's product row, by its own kernel.  (A
  //    return stored from the down GEMM's epilogue produced wrong tiles at full size -- C4,
  //    8192 tokens -- also on one rank with local stores only; it was taken out.)
  if (recv_cap > 0) {
    rc = run_expert_ffn(s, t.xs, recv_cap, t.xs_scales, 1, t.tiles, t.offsets, t.perm, local, tile_rows, hidden,
                        inter, gate_tiled, gate_scales, up_tiled, up_scales, down_tiled, down_scales, t.gu, t.hq,
                        t.h8, t.vals, t.n_dev);
    if (rc) return rc;
    EpReturnArgs ra{};
    ra.values = t.vals;
    ra.n_dev = t.n_dev;
    ra.cap = recv_cap;
    ra.hidden = (int)hidden;
    ra.rank = t.ret_rank;
    ra.row = t.ret_row;
    ra.prob = t.ret_prob;
    for (int g = 0; g < world; ++g) ra.base[g] = reinterpret_cast<uint16_t *>(at(g, products));
    if (launch_ep_return(ra, s, sms)) return cuda_err("expert-parallel return launch");
  }
  // 6. barrier: every product is home; the reference's ascending-expert chain
  if ((rc = launch_comm_barrier(comm_barrier_args(c, status), s))) return rc;
  if (tokens > 0 && launch_combine(products, routes, nullptr, tokens, topk, hidden, static_cast<uint16_t *>(out), s,
                                   sms, true))
    return cuda_err("combine launch");
  return 0;
}

// ---- tensor-parallel dense MLP --------------------------------------------------------
// No reference counterpart (the reference runs the MLP block on one GPU): the data movement
// after the all-gathers of a host that shards the intermediate dimension over `world` ranks.
int clefq_tp_gather_unpack(void *stream, const void *codes, int world, int64_t rows, int64_t shard_width,
                           void *operand, int64_t operand_ld) {
  if (world < 1 || world > 64 || rows < 0 || shard_width < 256 || shard_width % 256)
    return set_err(CLEFQ_ERR_SHAPE, "shards must be whole 256-code groups");
  if (operand_ld < world * shard_width || operand_ld % 16 || !al16(codes) || !al16(operand))
    return set_err(CLEFQ_ERR_ALIGN, "codes and operand must be 16-byte aligned rows");
  const int rc = launch_tp_gather_unpack(static_cast<const uint32_t *>(codes), world, rows, (int)(shard_width / 8),
                                         static_cast<uint8_t *>(operand), operand_ld,
                                         static_cast<cudaStream_t>(stream), device_sms());
  return rc ? cuda_err("tensor-parallel unpack launch") : 0;
}

int clefq_tp_interleave(void *stream, const void *src, int world, int64_t rows, int64_t shard_bytes, void *dst,
                        int64_t dst_ld_bytes) {
  if (world < 1 || world > 64 || rows < 0 || shard_bytes <= 0 || shard_bytes % 16)
    return set_err(CLEFQ_ERR_SHAPE, "shard rows must be a multiple of 16 bytes");
  if (dst_ld_bytes < world * shard_bytes || dst_ld_bytes % 16 || !al16(src) || !al16(dst))
    return set_err(CLEFQ_ERR_ALIGN, "source and destination must be 16-byte aligned rows");
  const int rc = launch_tp_interleave(static_cast<const uint8_t *>(src), world, rows, shard_bytes,
                                      static_cast<uint8_t *>(dst), dst_ld_bytes, static_cast<cudaStream_t>(stream),
                                      device_sms());
  return rc ? cuda_err("tensor-parallel interleave launch") : 0;
}

}  // extern "C"
