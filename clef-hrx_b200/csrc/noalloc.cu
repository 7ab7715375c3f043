// clefq: the quantized projection for callers that cannot allocate device memory.
//
// clefq_gemm needs an s8 copy of the packed int4 activation codes (m * k bytes) and takes
// it from a caller-provided workspace.  Some callers have no way to provide one: a host
// runtime that reserves every byte of device memory for its own allocator at start-up and
// hands plugins only the input and output buffers of each call, or an FFI binding whose
// ABI has no workspace argument.  clefq_gemm_noalloc serves them from a fixed scratch
// array that is part of this library's device image instead.
//
// Costs and limits of the fixed scratch:
//   * the array lives in this library's device module.  With the CUDA runtime's default
//     lazy module loading (CUDA 12.2 and later) the module, and with it the 64 MiB, is
//     loaded on a device the first time this entry point runs there, and stays until the
//     process exits.  With CUDA_MODULE_LOADING=EAGER every device on which the library
//     creates a context holds the 64 MiB, whether or not it ever calls this;
//   * one array per device is shared by all calls: calls whose kernels overlap on the GPU
//     (other streams, other host threads) race on it and must be serialised by the caller;
//   * m * k must not exceed NOALLOC_SCRATCH_BYTES; larger problems get CLEFQ_ERR_WORKSPACE.
// The first call on each device looks up the array's device address with the device
// current; that lookup is what loads the module.  A call with m == 0 does the lookup and
// nothing else, so a host whose allocator will take all of device memory makes one such
// call on each device before reserving it.  Nothing here calls cudaMalloc, cudaFree or any
// allocating routine.
#include <stdio.h>

#include <mutex>

#include "clefq_internal.h"

namespace cq {

constexpr int64_t NOALLOC_SCRATCH_BYTES = CLEFQ_GEMM_NOALLOC_MAX_BYTES;  // m * k of e.g. 4096 x 16384
static_assert(NOALLOC_SCRATCH_BYTES == 64ll << 20, "the header states 64 MiB");

// The s8 operand scratch.  In host code this name is only a stand-in for the symbol: the
// device address must come from cudaGetSymbolAddress on the current device.
static __device__ __align__(256) uint8_t g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

namespace {
std::mutex g_noalloc_mu;

// Records "clefq_gemm_noalloc: <what>: <CUDA's message>" for clefq_last_error().
int cuda_failure(const char *what, cudaError_t e) {
  char msg[256];
  snprintf(msg, sizeof msg, "clefq_gemm_noalloc: %s: %s", what, cudaGetErrorString(e));
  return report_error(CLEFQ_ERR_CUDA, msg);
}

uint8_t *g_noalloc_ptr[64];

// Device address of this device's scratch array (looked up once per device).
int scratch_for_current_device(uint8_t **out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return report_error(CLEFQ_ERR_CUDA, "clefq_gemm_noalloc: no current CUDA device");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      cudaGetLastError();
      return cuda_failure("cannot resolve the scratch array on this device", e);
    }
    g_noalloc_ptr[dev] = static_cast<uint8_t *>(p);
  }
  *out = g_noalloc_ptr[dev];
  return 0;
}
}  // namespace

}  // namespace cq

using namespace cq;

extern "C" __attribute__((visibility("default"))) int clefq_gemm_noalloc(
    void *stream, const void *a_codes, int64_t a_ld_words, const float *a_scales, int64_t m, const void *w_tiled,
    const float *w_scales, int64_t n, int64_t k, const void *residual, int64_t residual_ld, int out_dtype, void *out,
    int64_t out_ld) {
  if (m < 0 || m > 16777216 || n < 128 || n > 65536 || n % 128 || k < 256 || k > 65536 || k % 256 ||
      a_ld_words * 8 < k || out_ld < n || (out_dtype != CLEFQ_BF16 && out_dtype != CLEFQ_F32) ||
      (residual && (out_dtype != CLEFQ_BF16 || residual_ld < n)))
    return report_error(CLEFQ_ERR_SHAPE, "clefq_gemm_noalloc: unsupported shape (n % 128, k % 256, 4-bit codes)");
  if (m * k > NOALLOC_SCRATCH_BYTES)
    return report_error(CLEFQ_ERR_WORKSPACE,
                        "clefq_gemm_noalloc: m * k exceeds the 64 MiB built-in scratch; use clefq_gemm with a workspace");
  // Resolve the scratch first, also for m == 0: that call is the documented way to load
  // the array on a device before the host's allocator takes the rest of its memory.
  uint8_t *op = nullptr;
  int rc = scratch_for_current_device(&op);
  if (rc) return rc;
  if (m == 0) return 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The unpack kernel rewrites every byte of [m][k] that the GEMM reads; nothing needs
  // clearing between calls.
  rc = launch_unpack_i4(static_cast<const uint32_t *>(a_codes), a_ld_words, m, (int)k, op, k, s, device_sms());
  if (rc) return cuda_failure("unpack launch failed", last_launch_error());
  int *status = device_status_word();
  if (!status) return report_error(CLEFQ_ERR_CUDA, "clefq_gemm_noalloc: status word");
  GemmParams p{};
  p.a_op = op;
  p.a_rows = m;
  p.a_ld = k;
  p.a_scales = a_scales;
  p.w[0] = static_cast<const uint32_t *>(w_tiled);
  p.w_scales[0] = w_scales;
  p.n_split = (int)(n / 128);
  p.m = m;
  p.n = (int)n;
  p.k = (int)k;
  p.bits = 4;
  p.out = out_dtype == CLEFQ_BF16 ? static_cast<uint16_t *>(out) : nullptr;
  p.out_f32 = out_dtype == CLEFQ_F32 ? static_cast<float *>(out) : nullptr;
  p.ldo = out_ld;
  p.residual = static_cast<const uint16_t *>(residual);
  p.ldr = residual_ld;
  p.err = status;
  rc = launch_gemm(p, s);
  if (rc == CLEFQ_ERR_CUDA) return cuda_failure("gemm launch failed", last_launch_error());
  if (rc) return report_error(rc, "clefq_gemm_noalloc: unsupported shape or alignment");
  return 0;
}
