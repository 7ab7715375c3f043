// clefq: symmetric device buffers shared by the ranks of one node, and a device barrier.
//
// Every rank allocates one region of the same size; the regions are mapped into each other's
// address space (CUDA IPC between processes, or plain device pointers when one process drives
// several GPUs with peer access), so a kernel on rank r can store straight into rank g's
// region over NVLink.  The fused tensor-parallel MLP (clefq_tp_mlp) uses this for its
// collectives: the packing kernel and the GEMM epilogue write their shards into every rank's
// buffer, and a one-block barrier kernel orders the phases.
//
// Region layout: a 4 KB header, then the caller's bytes.
//   header[0, 32)   u32 flags[8]: flags[g] = the last barrier epoch rank g has signalled here
//   header[64]      u32 counter: this rank's barrier epochs (never written by peers)
// A barrier bumps the counter to e, stores e into flags[rank] of every peer (release, system
// scope) and waits until its own flags[g] >= e for every peer g (acquire, system scope).  The
// ranks run the same sequence of barriers, so their epochs agree; a flag that is already past
// e (a peer one barrier ahead) also satisfies the wait.  Each wait is bounded: on expiry the
// kernel records site 8 in the device status word (clefq_status -> CLEFQ_ERR_TIMEOUT) and
// returns; the communicator is then out of step and must be recreated.
#include <string.h>

#include "cq_common.cuh"
#include "clefq_internal.h"

namespace cq {

constexpr int kSiteCommBarrier = 8;

CQ_DEV void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
CQ_DEV uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(1024) comm_barrier_kernel(CommBarrierArgs a) {
  __shared__ uint32_t epoch;
  __shared__ int failed;
  // optional payload: this rank's slot of a small exchanged array, stored into every peer
  if (a.words) {
    for (int64_t i = threadIdx.x; i < a.words; i += blockDim.x) {
      const uint32_t v = a.src[i];
#pragma unroll
      for (int g = 0; g < kMaxRanks; ++g)
        if (g < a.world && g != a.rank) a.dst[g][i] = v;
    }
    __threadfence_system();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    failed = 0;
    __threadfence_system();  // every store this rank made before the barrier, then the flags
    const uint32_t e = *a.counter + 1u;
    *a.counter = e;
    epoch = e;
    for (int g = 0; g < a.world; ++g)
      if (g != a.rank) st_release_sys(a.peer_flags[g] + a.rank, e);
  }
  __syncthreads();
  const uint32_t e = epoch;
  if ((int)threadIdx.x < a.world && (int)threadIdx.x != a.rank) {
    const uint32_t *f = a.flags + threadIdx.x;
    const uint64_t t0 = globaltimer_ns();
    while ((int32_t)(ld_acquire_sys(f) - e) < 0) {
      if (globaltimer_ns() - t0 > a.timeout_ns) {
        atomicExch(&failed, 1);
        atomicCAS(a.err, 0, kSiteCommBarrier);
        break;
      }
      __nanosleep(100);
    }
  }
  __syncthreads();
  if (failed) return;
  // optional reduction of the exchanged per-rank arrays: mx[i] = max over ranks
  for (int64_t i = threadIdx.x; i < a.m; i += blockDim.x) {
    float v = a.maxes[i];
    for (int g = 1; g < a.world; ++g) v = fmaxf(v, a.maxes[g * a.m + i]);
    a.mx[i] = v;
  }
}

int launch_comm_barrier(const CommBarrierArgs &a, cudaStream_t stream) {
  comm_barrier_kernel<<<1, 1024, 0, stream>>>(a);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : report_error(CLEFQ_ERR_CUDA, cudaGetErrorString(e));
}

CommBarrierArgs comm_barrier_args(clefq_comm *c, int *err) {
  CommBarrierArgs a{};
  a.flags = reinterpret_cast<uint32_t *>(c->base);
  for (int g = 0; g < c->world; ++g)
    a.peer_flags[g] = g == c->rank ? nullptr : reinterpret_cast<uint32_t *>(c->peer[g]);
  a.counter = reinterpret_cast<uint32_t *>(c->base + 64);
  a.rank = c->rank;
  a.world = c->world;
  a.timeout_ns = c->timeout_ns;
  a.err = err;
  return a;
}

}  // namespace cq

using namespace cq;

extern "C" {

int64_t clefq_comm_handle_bytes(void) { return (int64_t)sizeof(cudaIpcMemHandle_t); }

int clefq_comm_create(int rank, int world, int64_t bytes, clefq_comm **comm, void *handle) {
  if (!comm) return report_error(CLEFQ_ERR_SHAPE, "comm: null output");
  *comm = nullptr;
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world || bytes < 0)
    return report_error(CLEFQ_ERR_SHAPE, "comm: world must be 1..8 and 0 <= rank < world");
  clefq_comm *c = new clefq_comm{};
  c->rank = rank;
  c->world = world;
  c->bytes = (bytes + 4095) & ~int64_t(4095);
  c->timeout_ns = 5000000000ll;
  cudaGetDevice(&c->device);
  void *p = nullptr;
  if (cudaMalloc(&p, kCommHeader + c->bytes) != cudaSuccess) {
    delete c;
    return report_error(CLEFQ_ERR_CUDA, "comm: region allocation failed");
  }
  c->base = static_cast<uint8_t *>(p);
  c->peer[rank] = c->base;
  if (cudaMemset(c->base, 0, kCommHeader) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
      (handle && cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t *>(handle), c->base) != cudaSuccess)) {
    cudaFree(c->base);
    delete c;
    return report_error(CLEFQ_ERR_CUDA, "comm: region setup failed");
  }
  *comm = c;
  return 0;
}

int clefq_comm_open(clefq_comm *c, const void *handles) {
  if (!c || !handles) return report_error(CLEFQ_ERR_SHAPE, "comm: null argument");
  const cudaIpcMemHandle_t *h = static_cast<const cudaIpcMemHandle_t *>(handles);
  for (int g = 0; g < c->world; ++g) {
    if (g == c->rank || c->peer[g]) continue;
    void *p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h[g], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
      return report_error(CLEFQ_ERR_CUDA, "comm: opening a peer region failed");
    c->peer[g] = static_cast<uint8_t *>(p);
    c->opened[g] = true;
  }
  return 0;
}

int clefq_comm_attach(clefq_comm *c, int rank, clefq_comm *peer) {
  if (!c || !peer || rank < 0 || rank >= c->world || rank == c->rank || peer->rank != rank ||
      peer->world != c->world || peer->bytes != c->bytes)
    return report_error(CLEFQ_ERR_SHAPE, "comm: attach needs the peer of that rank in the same group");
  c->peer[rank] = peer->base;
  c->opened[rank] = false;
  return 0;
}

int clefq_comm_ready(const clefq_comm *c) {
  if (!c) return 0;
  for (int g = 0; g < c->world; ++g)
    if (!c->peer[g]) return 0;
  return 1;
}

void *clefq_comm_region(clefq_comm *c) { return c ? c->base + kCommHeader : nullptr; }
int64_t clefq_comm_region_bytes(const clefq_comm *c) { return c ? c->bytes : 0; }

int clefq_comm_set_timeout_ms(clefq_comm *c, int64_t ms) {
  if (!c || ms <= 0) return report_error(CLEFQ_ERR_SHAPE, "comm: timeout must be positive");
  c->timeout_ns = ms * 1000000ll;
  return 0;
}

int clefq_comm_barrier(clefq_comm *c, void *stream) {
  if (!clefq_comm_ready(c)) return report_error(CLEFQ_ERR_SHAPE, "comm: peers not opened");
  int *status = device_status_word();
  if (!status) return report_error(CLEFQ_ERR_CUDA, "status word");
  return launch_comm_barrier(comm_barrier_args(c, status), static_cast<cudaStream_t>(stream));
}

int clefq_comm_destroy(clefq_comm *c) {
  if (!c) return 0;
  int rc = 0;
  for (int g = 0; g < c->world; ++g)
    if (c->opened[g] && cudaIpcCloseMemHandle(c->peer[g]) != cudaSuccess) rc = CLEFQ_ERR_CUDA;
  if (cudaFree(c->base) != cudaSuccess) rc = CLEFQ_ERR_CUDA;
  delete c;
  return rc ? report_error(rc, "comm: release failed") : 0;
}

}  // extern "C"
