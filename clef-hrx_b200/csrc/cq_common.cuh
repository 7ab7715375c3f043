// clefq: shared device helpers for the sm_100a kernels.
//
// Numerics: IEEE binary32 with round-to-nearest-even; every multiply and add whose
// rounding is part of the reference contract is written with __fmul_rn / __fadd_rn /
// __fsub_rn / __fmaf_rn so the compiler cannot contract or reassociate it.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include "cq_math.h"

#define CQ_DEV __device__ __forceinline__

namespace cq {

// IEEE maxNum / minNum (return the non-NaN operand).
CQ_DEV float maxnum(float a, float b) { return fmaxf(a, b); }
CQ_DEV float minnum(float a, float b) { return fminf(a, b); }

// The s8 GEMM operand of a packed int4 word: 16 * code, K-permuted within each 32-code
// group (low nibbles of the 4 words first, then high nibbles).  Both GEMM operands use
// the same permutation, so dot products are unchanged; the x16 on each side makes every
// accumulator exactly 256 * the reference's int32 dot.
CQ_DEV uint32_t nib_lo16(uint32_t w) { return (w << 4) & 0xF0F0F0F0u; }
CQ_DEV uint32_t nib_hi16(uint32_t w) { return w & 0xF0F0F0F0u; }

// SiLU of one BF16 input rounded to BF16, bit-identical to silu_bf16() (cq_math.h) and to the
// table generated from it (tab, 65,536 entries), without reading the table in the common case.
// Ziv's rounding test (A. Ziv, "Fast evaluation of elementary mathematical functions with
// correctly rounded last bit", ACM TOMS 17(3), 1991): for -16 < g < 8 the quotient
// q = g * rcp(1 + 2^(-g log2(e))) from the hardware's approximate exp2 and reciprocal lies
// within about 40 units of 2^-24 (relative) of the reference quotient g / (1 + exp_cw(-g)):
// the product g log2(e) carries at most |g log2(e)| 2^-24 of absolute error (about 24 units
// through 2^x), exp2 and the reciprocal a few units each, the reference a few more.  When q's
// bits lie more than kSiluMargin f32 steps from a BF16 rounding midpoint, both quotients round
// to the same BF16 value.  g >= 8 (and +Inf) gives g exactly; the rest (g <= -16, -Inf, NaN)
// and the near-midpoint cases (about 0.4% of inputs) read the table.  The exhaustive GPU test
// of clefq_silu checks every BF16 input against the table.
constexpr uint32_t kSiluMargin = 128;
CQ_DEV uint32_t silu_bf16_ziv(uint32_t g16, const uint16_t *__restrict__ tab) {
  const float g = __uint_as_float(g16 << 16);
  float t, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(t) : "f"(__fmul_rn(g, -1.44269502162933349609375f)));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(__fadd_rn(1.0f, t)));
  const uint32_t b = __float_as_uint(__fmul_rn(g, r));
  uint32_t out = (b + 0x7fffu + ((b >> 16) & 1u)) >> 16;  // nearest even; q is finite here
  const bool fast = g > -16.0f && g < 8.0f && ((b + (kSiluMargin - 0x8000u)) & 0xffffu) > 2 * kSiluMargin;
  if (!fast) out = g >= 8.0f ? g16 : (uint32_t)__ldg(tab + g16);
  return out;
}

// ---------------------------------------------------------------------------------------
// Shared-memory addresses, mbarriers, TMA, tcgen05 (inline PTX for sm_100a)
// ---------------------------------------------------------------------------------------
CQ_DEV uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

CQ_DEV void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
CQ_DEV void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
CQ_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

CQ_DEV void mbar_arrive(uint64_t *bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar)) : "memory");
}
CQ_DEV void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
CQ_DEV bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

CQ_DEV uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait: polls for at most ~2 s of wall time, then records `code` in *err and
// returns false.  The caller then skips the rest of its role; the kernel still frees its
// TMEM and exits, so a lost arrival shows up as an error status, never as a hang.
// A wait also gives up early once another role of the same CTA has reported an error.
CQ_DEV bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, int *err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*(volatile int *)err) return false;
    if (globaltimer_ns() - t0 > 2000000000ull) {
      atomicCAS(err, 0, code);
      return false;
    }
  }
}

struct alignas(64) TmaDesc {
  uint8_t bytes[128];
};

CQ_DEV void tma_prefetch_desc(const void *desc) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(desc) : "memory");
}

// 2D tiled TMA load (no multicast) into CTA shared memory, completing on `bar`.
CQ_DEV void tma_load_2d(void *dst, const void *desc, uint64_t *bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(desc), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// 3D tiled TMA load (no multicast).
CQ_DEV void tma_load_3d(void *dst, const void *desc, uint64_t *bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(desc), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Barrier among `count` threads (a subset of the CTA), id 1..15.
CQ_DEV void named_barrier_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Barrier among `count` threads that also returns the AND of `pred` over them, so that
// the participating warps take the same branch afterwards.
CQ_DEV bool named_barrier_and(int id, int count, bool pred) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(out)
      : "r"((uint32_t)pred), "r"(id), "r"(count)
      : "memory");
  return out != 0;
}

CQ_DEV uint4 lds_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

// --- tcgen05 ---------------------------------------------------------------------------
CQ_DEV void tmem_alloc(uint32_t *slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot_smem)),
               "r"(ncols)
               : "memory");
}
CQ_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
CQ_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
CQ_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
CQ_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[tmem] x B[smem desc], kind::i8 (s8 x s8 -> s32), one CTA.
CQ_DEV void mma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once every previously issued tcgen05.mma of this thread has completed.
CQ_DEV void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Instruction descriptor: kind::i8, D s32, A s8, B s8, both K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// Shared-memory matrix descriptor, K-major, 128-byte swizzle, 8-row core groups 1024 B
// apart (SBO), version 1 (sm_100).  `addr` is the byte address in shared memory.
CQ_DEV uint64_t smem_desc_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;              // LBO (unused for swizzled K-major)
  d |= (uint64_t)(1024u >> 4) << 32;    // SBO
  d |= (uint64_t)1u << 46;              // version
  d |= (uint64_t)2u << 61;              // SWIZZLE_128B
  return d;
}

// 32 lanes x 32-bit, 64 consecutive columns per thread.
CQ_DEV void tmem_st_x64(uint32_t taddr, const uint32_t (&v)[64]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x64.b32 [%0], {"
      "%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,"
      "%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,"
      "%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63,%64};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31]), "r"(v[32]), "r"(v[33]), "r"(v[34]), "r"(v[35]), "r"(v[36]),
      "r"(v[37]), "r"(v[38]), "r"(v[39]), "r"(v[40]), "r"(v[41]), "r"(v[42]), "r"(v[43]), "r"(v[44]), "r"(v[45]),
      "r"(v[46]), "r"(v[47]), "r"(v[48]), "r"(v[49]), "r"(v[50]), "r"(v[51]), "r"(v[52]), "r"(v[53]), "r"(v[54]),
      "r"(v[55]), "r"(v[56]), "r"(v[57]), "r"(v[58]), "r"(v[59]), "r"(v[60]), "r"(v[61]), "r"(v[62]), "r"(v[63])
      : "memory");
}
CQ_DEV void tmem_st_x32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {"
      "%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
// tcgen05.st and tcgen05.ld move registers asynchronously: a store's source registers must
// keep their values until tcgen05.wait::st, and a load's destination registers hold the data
// only after tcgen05.wait::ld.  A wait written as a bare statement orders memory, not
// registers, so the compiler could reuse a source register or schedule a use of a loaded
// one across it.  These waits take the registers as operands: store sources stay live and
// unchanged until the wait, and every use of loaded values depends on the wait.
CQ_DEV void tmem_st_wait(const uint32_t (&v)[32]) {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
      "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
      "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
               : "memory");
}
// A second source array of the same wait: keeps its registers live up to this point, which
// follows the wait (volatile statements keep their order).
CQ_DEV void tmem_st_keep(const uint32_t (&v)[32]) {
  asm volatile("" ::
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
      "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
      "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
               : "memory");
}

CQ_DEV void tmem_ld_x32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {"
      "%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr)
      : "memory");
}
CQ_DEV void tmem_ld_wait(uint32_t (&v)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
      "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15]),
      "+r"(v[16]), "+r"(v[17]), "+r"(v[18]), "+r"(v[19]), "+r"(v[20]), "+r"(v[21]), "+r"(v[22]), "+r"(v[23]),
      "+r"(v[24]), "+r"(v[25]), "+r"(v[26]), "+r"(v[27]), "+r"(v[28]), "+r"(v[29]), "+r"(v[30]), "+r"(v[31])
               :
               : "memory");
}
// A second destination array of the same wait: uses of its registers depend on this
// statement, which follows the wait.
CQ_DEV void tmem_ld_tie(uint32_t (&v)[32]) {
  asm volatile(""
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
      "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15]),
      "+r"(v[16]), "+r"(v[17]), "+r"(v[18]), "+r"(v[19]), "+r"(v[20]), "+r"(v[21]), "+r"(v[22]), "+r"(v[23]),
      "+r"(v[24]), "+r"(v[25]), "+r"(v[26]), "+r"(v[27]), "+r"(v[28]), "+r"(v[29]), "+r"(v[30]), "+r"(v[31])
               :
               : "memory");
}

// Programmatic dependent launch.  A kernel launched with programmatic stream serialization
// may start while the previous kernel of its stream still runs: pdl_wait() returns once that
// kernel has completed and its memory is visible, so nothing that kernel writes (or reads and
// this kernel overwrites) may be touched before it.  pdl_trigger() lets the next such kernel
// of the stream be scheduled; it waits in its own pdl_wait() all the same.
CQ_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
CQ_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

CQ_DEV uint4 ldg_nc_v4(const void *p) { return __ldg(reinterpret_cast<const uint4 *>(p)); }

// --- clusters and 2-SM (cta_group::2) forms --------------------------------------------
CQ_DEV uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
CQ_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Shared::cluster address of the same shared variable in CTA `rank` of this cluster.
CQ_DEV uint32_t mapa_shared(uint32_t local_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
  return r;
}
// Arrive on a barrier of another CTA of the cluster (default .release.cta semantics; a
// .cluster-scope release here costs ~1.5k cycles per call and serialised the pair
// pipeline).  Ordering of tensor-memory writes is given by tcgen05.wait::st and
// tcgen05.fence::before_thread_sync ahead of the arrive.
CQ_DEV void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Asynchronous cross-CTA signal: stores 4 bytes into shared word `word` of another CTA
// and counts them as completed transaction bytes on that CTA's barrier `bar` (both are
// cluster addresses).  The issuing thread does not wait for the round trip, unlike a
// remote mbarrier.arrive.
CQ_DEV void st_async_signal(uint32_t word, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.u32 [%0], %1, [%2];" ::"r"(word), "r"(1u),
               "r"(bar)
               : "memory");
}
CQ_DEV void mbar_arrive_expect_tx_u32(uint32_t bar_addr, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar_addr), "r"(bytes) : "memory");
}
// 2D tiled TMA load into this CTA's shared memory whose completion is counted on the
// barrier at cluster address `bar` (the pair leader's), as the 2-SM MMA requires.
CQ_DEV void tma_load_2d_cg2(void *dst, const void *desc, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(desc), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
CQ_DEV void tma_load_3d_cg2(void *dst, const void *desc, uint32_t bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(desc), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}
CQ_DEV void tmem_alloc2(uint32_t *slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot_smem)),
               "r"(ncols)
               : "memory");
}
CQ_DEV void tmem_relinquish2() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory"); }
CQ_DEV void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[tmem] (+)= A[tmem] x B[smem desc] across the CTA pair (M = 256 rows, 128 per CTA;
// B's N rows split in halves between the two CTAs' shared memory at the same offset).
CQ_DEV void mma_i8_ts2(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the barrier at this shared offset in every CTA of `mask` when the pair's
// previously issued MMAs complete.
CQ_DEV void mma_commit2_mc(uint64_t *bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}

}  // namespace cq
