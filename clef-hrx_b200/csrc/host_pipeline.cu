// clefq: the dense MLP block from host memory to host memory, with the PCIe copies of one
// row chunk overlapping the kernels of its neighbours.
//
// Every row of the MLP block is independent (per-row quantisation, per-row GEMM outputs), so
// the block over m rows equals the block over any split of the rows into chunks; the
// reference states the same for its chunked call sites (src/backbone.rs:866-907, at most
// 2048 tokens per chunk).  Each chunk uses device staging buffer (chunk sequence number) % 2:
//
//   copy-in stream   H2D x chunk (and residual)          after the buffer's previous kernels
//   caller's stream  clefq_mlp on the chunk              after its H2D and the buffer's
//                                                        previous D2H
//   copy-out stream  D2H output chunk                    after the chunk's kernels
//
// The sequence number and the buffer events live in the library (one set per device) and
// carry over from call to call, so with CLEFQ_HOST_STREAMING the next call's first input
// copy overlaps this call's kernels: a stream of calls runs at the pace of its slowest
// engine (PCIe in, kernels, PCIe out) instead of their sum.  Without that flag a call first
// waits for all earlier work on the caller's stream.  The call's end: done_event (when given)
// is recorded after its last output copy; otherwise the caller's stream waits for that copy.
// Enqueueing is serialised by a per-device lock; a stream-wait captures an event when it is
// enqueued, so later re-recording is harmless.
#include <mutex>

#include "clefq_internal.h"

namespace cq {
namespace {

struct HostPipe {
  bool ready = false;
  cudaStream_t in = nullptr, out = nullptr;
  cudaEvent_t entry = nullptr, done = nullptr, loaded[2] = {}, computed[2] = {}, stored[2] = {};
  uint64_t seq = 0;          // chunks enqueued so far on this device
  bool used[2] = {};         // the buffer's events have been recorded
};
HostPipe g_pipe[64];
std::mutex g_pipe_mu[64];

bool pipe_init(HostPipe &p) {
  if (p.ready) return true;
  if (cudaStreamCreateWithFlags(&p.in, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&p.out, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&p.entry, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&p.done, cudaEventDisableTiming) != cudaSuccess)
    return false;
  for (int b = 0; b < 2; ++b)
    if (cudaEventCreateWithFlags(&p.loaded[b], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&p.computed[b], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&p.stored[b], cudaEventDisableTiming) != cudaSuccess)
      return false;
  p.ready = true;
  return true;
}

struct HostTables {
  uint8_t *mlp_ws;
  int64_t mlp_bytes;
  uint16_t *x[2], *res[2], *out[2];
};

Arena host_tables(Arena a, int64_t chunk, int64_t hidden, int64_t inter, bool residual, HostTables &t) {
  t.mlp_bytes = clefq_mlp_workspace_size(chunk, hidden, inter);
  t.mlp_ws = a.take<uint8_t>(t.mlp_bytes);
  for (int b = 0; b < 2; ++b) {
    t.x[b] = a.take<uint16_t>(chunk * hidden);
    t.res[b] = residual ? a.take<uint16_t>(chunk * hidden) : nullptr;
    t.out[b] = a.take<uint16_t>(chunk * hidden);
  }
  return a;
}

}  // namespace
}  // namespace cq

using namespace cq;

extern "C" {

int64_t clefq_mlp_host_workspace_size(int64_t chunk_rows, int64_t hidden, int64_t inter, int with_residual) {
  if (chunk_rows < 1 || hidden < 256 || inter < 256) return -1;
  HostTables t;
  return aligned_total(host_tables(Arena{nullptr, INT64_MAX}, chunk_rows, hidden, inter, with_residual != 0, t));
}

int clefq_mlp_host(void *stream, const void *x_host, int64_t m, int64_t hidden, int64_t inter, const void *gate_tiled,
                   const float *gate_scales, const void *up_tiled, const float *up_scales, const void *down_tiled,
                   const float *down_scales, const void *residual_host, void *out_host, int64_t chunk_rows,
                   int flags, void *done_event, void *workspace, int64_t workspace_bytes) {
  if (m < 1 || chunk_rows < 1 || !x_host || !out_host)
    return report_error(CLEFQ_ERR_SHAPE, "host MLP: rows, chunk rows and buffers must be given");
  if (flags & ~CLEFQ_HOST_STREAMING) return report_error(CLEFQ_ERR_SHAPE, "host MLP: unknown flags");
  HostTables t;
  Arena a = host_tables(Arena{static_cast<uint8_t *>(workspace), workspace_bytes}, chunk_rows, hidden, inter,
                        residual_host != nullptr, t);
  if (t.mlp_bytes < 0) return report_error(CLEFQ_ERR_SHAPE, "unsupported MLP shape");
  if (!a.ok || !workspace) return report_error(CLEFQ_ERR_WORKSPACE, "host MLP workspace too small");
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return report_error(CLEFQ_ERR_CUDA, "device index");
  std::lock_guard<std::mutex> lk(g_pipe_mu[dev]);
  HostPipe &p = g_pipe[dev];
  if (!pipe_init(p)) return report_error(CLEFQ_ERR_CUDA, "host MLP: stream or event creation failed");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t row_bytes = hidden * 2;
  auto fail = [](const char *what) { return report_error(CLEFQ_ERR_CUDA, what); };
  if (!(flags & CLEFQ_HOST_STREAMING)) {
    // the staging buffers may still be in use by earlier work on the caller's stream
    if (cudaEventRecord(p.entry, s) != cudaSuccess || cudaStreamWaitEvent(p.in, p.entry, 0) != cudaSuccess ||
        cudaStreamWaitEvent(p.out, p.entry, 0) != cudaSuccess)
      return fail("host MLP: stream ordering");
  }
  const int64_t chunks = (m + chunk_rows - 1) / chunk_rows;
  for (int64_t i = 0; i < chunks; ++i, ++p.seq) {
    const int b = (int)(p.seq & 1);
    const bool reuse = p.used[b];
    const int64_t r0 = i * chunk_rows;
    const int64_t rows = m - r0 < chunk_rows ? m - r0 : chunk_rows;
    const uint8_t *xh = static_cast<const uint8_t *>(x_host) + r0 * row_bytes;
    if (reuse && cudaStreamWaitEvent(p.in, p.computed[b], 0) != cudaSuccess) return fail("host MLP: stream ordering");
    if (cudaMemcpyAsync(t.x[b], xh, rows * row_bytes, cudaMemcpyHostToDevice, p.in) != cudaSuccess ||
        (residual_host &&
         cudaMemcpyAsync(t.res[b], static_cast<const uint8_t *>(residual_host) + r0 * row_bytes, rows * row_bytes,
                         cudaMemcpyHostToDevice, p.in) != cudaSuccess) ||
        cudaEventRecord(p.loaded[b], p.in) != cudaSuccess)
      return fail("host MLP: input copy");
    if (cudaStreamWaitEvent(s, p.loaded[b], 0) != cudaSuccess ||
        (reuse && cudaStreamWaitEvent(s, p.stored[b], 0) != cudaSuccess))
      return fail("host MLP: stream ordering");
    int rc = clefq_mlp(stream, t.x[b], rows, hidden, inter, gate_tiled, gate_scales, up_tiled, up_scales, down_tiled,
                       down_scales, residual_host ? t.res[b] : nullptr, t.out[b], t.mlp_ws, t.mlp_bytes);
    if (rc) return rc;
    if (cudaEventRecord(p.computed[b], s) != cudaSuccess || cudaStreamWaitEvent(p.out, p.computed[b], 0) != cudaSuccess)
      return fail("host MLP: stream ordering");
    if (cudaMemcpyAsync(static_cast<uint8_t *>(out_host) + r0 * row_bytes, t.out[b], rows * row_bytes,
                        cudaMemcpyDeviceToHost, p.out) != cudaSuccess ||
        cudaEventRecord(p.stored[b], p.out) != cudaSuccess)
      return fail("host MLP: output copy");
    p.used[b] = true;
  }
  // the end of the call: after its last output copy
  if (done_event) {
    if (cudaEventRecord(static_cast<cudaEvent_t>(done_event), p.out) != cudaSuccess) return fail("host MLP: event");
  } else if (cudaEventRecord(p.done, p.out) != cudaSuccess || cudaStreamWaitEvent(s, p.done, 0) != cudaSuccess) {
    return fail("host MLP: stream ordering");
  }
  return 0;
}

}  // extern "C"
