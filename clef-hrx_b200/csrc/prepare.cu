// clefq: activation/weight packing kernels for sm_100a.
//
//   prepare   per row: optional fused pre-op (SwiGLU, attention sigmoid gate, RMSNorm),
//             Hadamard-256 rotation, row absmax, one FP32 scale, int4/int8 codes packed
//             in the reference layout (codes[rows][stride/P] then f32 scales[rows]), and
//             optionally the s8 GEMM operand of the same codes.
//             Follows kernels/prepare_integer.loom:55-291 and
//             kernels/prepare_integer_register.loom:58-311; storage layout
//             src/quantized.rs:626-686.
//   swiglu    kernels/swiglu.loom:41-50
//   retile    kernels/retile_codes.loom:1-56
//   unpack    packed int4 activation codes -> s8 GEMM operand (no reference counterpart:
//             the operand format of the tcgen05 GEMM)
//
// Layout of one row in registers: a warp owns Hadamard groups of 256 elements, each lane
// eight consecutive elements of a group.  Radix-4 stride 1 runs inside a lane; strides 4,
// 16 and 64 exchange partial sums/differences with xor-shuffles.  The reference's
// operation order is kept (s01 = a+b, s23 = c+d, d01 = a-b, d23 = c-d; o = s01+d23,
// s01-d23, d01+s23, s23-d01), bit-identical under IEEE round-to-nearest-even.
#include <atomic>

#include "cq_common.cuh"
#include "clefq_internal.h"

// 1: the packing kernels are launched with programmatic stream serialization (each waits
// in-kernel for the previous kernel, griddepcontrol).
#ifndef CLEFQ_PDL_PREPARE
#define CLEFQ_PDL_PREPARE 1
#endif

namespace cq {

enum { MODE_PLAIN = 0, MODE_SWIGLU = 1, MODE_ATTN_GATE = 2, MODE_NORM = 3, MODE_NORM_STORE = 4 };

// One radix-4 stage across lanes.  Lane bits (xbit, ybit) select the element's role in
// the quad (a: 0,0  b: 1,0  c: 0,1  d: 1,1).  Every lane computes s = own + peer_x and
// t = own - peer_x, then adds the t of its y-partner:
//   a: (a+b) + (c-d) = s01 + d23        b: (a+b) + (d-c) = s01 - d23
//   c: (c+d) + (a-b) = d01 + s23        d: (c+d) + (b-a) = s23 - d01
// which are the reference's rounded results because x - y = -(y - x) and s + (-t) = s - t
// exactly under round-to-nearest-even.  Only the sign of an exact zero can differ, and no
// code or row scale depends on it.
template <int N>
CQ_DEV void radix4_lanes(float (&v)[N], int xmask, int ymask) {
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const float own = v[i];
    const float peer = __shfl_xor_sync(0xffffffffu, own, xmask);
    const float s = __fadd_rn(own, peer);
    const float t = __fsub_rn(own, peer);
    v[i] = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, t, ymask));
  }
}

CQ_DEV void hadamard256_lane(float (&v)[8]) {
  // stride 1: two quads inside the lane
#pragma unroll
  for (int q = 0; q < 8; q += 4) {
    const float a = v[q], b = v[q + 1], c = v[q + 2], d = v[q + 3];
    const float s01 = __fadd_rn(a, b), s23 = __fadd_rn(c, d), d01 = __fsub_rn(a, b), d23 = __fsub_rn(c, d);
    v[q] = __fadd_rn(s01, d23);
    v[q + 1] = __fsub_rn(s01, d23);
    v[q + 2] = __fadd_rn(d01, s23);
    v[q + 3] = __fsub_rn(s23, d01);
  }
  // stride 4: (a, b) = (v[i], v[i+4]) of the even lane, (c, d) of the odd lane
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float x = v[i], y = v[i + 4];
    const float s = __fadd_rn(x, y), d = __fsub_rn(x, y);
    const float p2 = __shfl_xor_sync(0xffffffffu, d, 1);
    v[i] = __fadd_rn(s, p2);
    v[i + 4] = __fsub_rn(s, p2);
  }
  radix4_lanes(v, 2, 4);    // stride 16
  radix4_lanes(v, 8, 16);   // stride 64
}

// Two products rounded to BF16 by one cvt.rn.bf16x2 and widened back to F32.  Finite and
// infinite values round exactly like f32_to_bf16; a NaN may lose its payload, which the
// packing never observes (a non-finite row packs to zero codes with an infinite scale).
CQ_DEV void bf16r_pair(float &lo, float &hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  lo = __uint_as_float(r << 16);
  hi = __uint_as_float(r & 0xffff0000u);
}

// max(m, |a|, |b|) propagating NaN (PTX max.NaN), so one non-finite element poisons the row.
CQ_DEV float absmax3_nan(float m, float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(m), "f"(fabsf(a)), "f"(fabsf(b)));
  return r;
}
CQ_DEV float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Round to the nearest integer, ties to even (cvt.rni), as the reference's rint().
CQ_DEV int rint_s32(float x) {
  int r;
  asm("cvt.rni.s32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

// Packs a pair of codes below the low bits of c: (c << 2w) | (hi << w) | lo, each code
// saturated to the signed w-bit range (cvt.pack.sat).  For a finite row every code lies in
// [-qmax, qmax]: scale = R/16/qmax and inv = 0.0625/scale are each rounded once, so
// |x * inv| <= qmax (1 + 3 * 2^-24) < qmax + 0.5 for |x| <= R, and the saturation never
// acts -- it equals the reference's clamp to +-qmax.
CQ_DEV uint32_t pack_s4(int hi, int lo, uint32_t c) {
  uint32_t r;
  asm("cvt.pack.sat.s4.s32.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(hi), "r"(lo), "r"(c));
  return r;
}
CQ_DEV uint32_t pack_s8(int hi, int lo, uint32_t c) {
  uint32_t r;
  asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(hi), "r"(lo), "r"(c));
  return r;
}

// bf16(silu(g)) for every BF16 bit pattern g, generated at build time by gen_tables.cpp
// with the arithmetic of cq_math.h (identical to silu_bf16() evaluated on the device).
constexpr int kSiluEntries = 65536;
__device__ const uint16_t g_silu_bf16[kSiluEntries] __align__(16) = {
#include "silu_bf16.inc"
};

// Device address of the table on the current device (looked up once per device), for the
// GEMM epilogue that applies SwiGLU; null if the lookup fails.
const uint16_t *silu_table_device() {
  static std::atomic<const uint16_t *> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  const uint16_t *p = cache[dev].load(std::memory_order_acquire);
  if (!p) {
    void *addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_silu_bf16) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    p = static_cast<const uint16_t *>(addr);
    cache[dev].store(p, std::memory_order_release);
  }
  return p;
}

// KIND_PLAIN and KIND_SILU_TABLE are the GEMM-input paths: int4 codes plus the s8 operand,
// with no pre-op or with SwiGLU through the table.  KIND_GENERAL reads mode, bits and the
// operand pointer at run time (SwiGLU evaluated directly, attention gate, RMSNorm).
enum { KIND_PLAIN = 0, KIND_SILU_TABLE = 1, KIND_GENERAL = 2 };

// Row-independent loads of one row's CH groups into registers (x, and the SwiGLU up /
// attention q-gate / norm weight operand), zero where the group or row does not exist.
template <int CH, bool AUX>
CQ_DEV void fetch_groups(const PrepareArgs &p, int64_t row, bool ok, int wt, int lane, int ngroups,
                         uint4 (&rx)[CH], uint4 (&ra)[CH]) {
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    const int g = wt + j * p.team_warps;
    rx[j] = make_uint4(0, 0, 0, 0);
    ra[j] = make_uint4(0, 0, 0, 0);
    if (ok && g < ngroups) {
      const int col0 = g * 256 + lane * 8;
      rx[j] = *reinterpret_cast<const uint4 *>(p.x + row * p.x_ld + col0);
      if (!AUX) {
      } else if (p.mode == MODE_SWIGLU)
        ra[j] = *reinterpret_cast<const uint4 *>(p.aux + row * p.aux_ld + col0);
      else if (p.mode == MODE_ATTN_GATE)
        ra[j] = *reinterpret_cast<const uint4 *>(p.aux + row * p.aux_ld + g * 512 + 256 + lane * 8);
      else if (p.mode != MODE_PLAIN)
        ra[j] = *reinterpret_cast<const uint4 *>(p.aux + col0);
    }
  }
}

// 16-byte global -> shared copy that holds no register while in flight (cp.async, L2 only);
// a zero source size writes zeros without reading global memory.
CQ_DEV void cp_async16(uint32_t dst, const void *src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
CQ_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
CQ_DEV void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Load pipeline of a kernel instance: 0 = loads at the top of each iteration, 1 = one
// iteration prefetched in registers, >= 2 = that many cp.async stages per thread (each
// thread stages and later reads only its own 16-byte chunks, so the stages need no
// barrier).  A stage is refilled as soon as its data is in registers, so all STG stages
// are in flight while a row is rotated: about 96-128 KB per SM.
constexpr int stages_for(int ch, int kind) {
  return kind == KIND_PLAIN ? (ch <= 4 ? 4 : 2)
         : kind == KIND_SILU_TABLE ? (ch == 1 ? 4 : ch == 2 ? 3 : ch == 3 ? 2 : ch == 4 ? 1 : 0)
                                   : (ch <= 4 ? 1 : 0);
}
constexpr int operands_for(int kind) { return kind == KIND_PLAIN ? 1 : 2; }
constexpr int min_blocks_for(int ch, int kind) { return kind == KIND_PLAIN && ch <= 2 ? 2 : 1; }

// Issues the cp.async copies of one row's CH groups (x and, for SwiGLU, up) into a stage.
template <int CH, int KIND>
CQ_DEV void stage_groups(const PrepareArgs &p, uint32_t stage_base, int64_t row, bool ok, int wt, int lane,
                         int ngroups) {
  constexpr int NOP = operands_for(KIND);
  const uint16_t *xr = p.x + row * p.x_ld + lane * 8;
  const uint16_t *ar = p.aux + row * p.aux_ld + lane * 8;
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    const int g = wt + j * p.team_warps;
    const bool valid = ok && g < ngroups;
    const uint32_t slot = stage_base + (uint32_t)(j * NOP) * blockDim.x * 16 + threadIdx.x * 16;
    cp_async16(slot, valid ? (const void *)(xr + g * 256) : (const void *)p.x, valid);
    if (NOP == 2) cp_async16(slot + blockDim.x * 16, valid ? (const void *)(ar + g * 256) : (const void *)p.x, valid);
  }
}

// Persistent packing kernel.  A team of team_warps warps owns one row, each warp CH
// Hadamard groups of it; rows_per_block teams per CTA; the CTA strides over row blocks.
//
// Per iteration: [RMSNorm partials -> barrier] -> pre-op -> Hadamard -> warp absmax ->
// barrier -> row scale -> codes.  The per-warp maxima and norm partials are double
// buffered by iteration parity, so one barrier per phase is enough.
template <int CH, int KIND>
__global__ void __launch_bounds__(512, min_blocks_for(CH, KIND)) prepare_kernel(PrepareArgs p) {
  // launched with programmatic stream serialization: the input is the previous kernel's output
  pdl_wait();
  pdl_trigger();
  constexpr bool FAST = KIND != KIND_GENERAL;
  constexpr bool TAB = KIND == KIND_SILU_TABLE;
  constexpr int STG = stages_for(CH, KIND);
  constexpr bool PF = STG == 1;
  constexpr int NOP = operands_for(KIND);
  extern __shared__ __align__(16) uint8_t smem[];
  const uint16_t *tab = reinterpret_cast<const uint16_t *>(smem);
  float *red = reinterpret_cast<float *>(smem + (TAB ? kSiluEntries * 2 : 0));  // [2][slots] maxima
  const int tw = p.team_warps, rpb = p.rows_per_block;
  const int slots = rpb * tw;
  float *wsum = red + 2 * slots;                                                 // [2][slots] norm partials
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int team = warp / tw, wt = warp % tw;
  const int tid_team = wt * 32 + lane;
  const int ngroups = p.width >> 8;
  const int bits = FAST ? 4 : p.bits;
  const bool has_op = FAST || p.op8 != nullptr;
  const int words = FAST ? p.stride >> 3 : p.stride / (32 / bits);
  const int code_words = FAST ? p.width >> 3 : p.width / (32 / bits);
  const bool norm = KIND == KIND_GENERAL && (p.mode == MODE_NORM || p.mode == MODE_NORM_STORE);
  const int64_t nblk = (p.rows + rpb - 1) / rpb;
  const float qmax = bits == 8 ? 127.0f : 7.0f;
  // this lane's word inside its 32-code operand block (low-nibble half; high half +16 B)
  const int lane_op = (lane >> 2) * 32 + (lane & 3) * 4;
  // cp.async stages follow the maxima and norm partials: [STG][CH][NOP][threads] x 16 B
  const uint32_t stage0 = smem_u32(wsum + 2 * slots);
  const uint32_t stage_bytes = (uint32_t)(CH * NOP) * blockDim.x * 16;

  uint4 rx[CH], ra[CH];
  int64_t blk = blockIdx.x;
  if (PF) fetch_groups<CH, KIND != KIND_PLAIN>(p, blk * rpb + team, blk * rpb + team < p.rows, wt, lane, ngroups, rx, ra);
  if (STG >= 2) {
#pragma unroll
    for (int st = 0; st < STG; ++st) {
      const int64_t b = blk + (int64_t)st * gridDim.x;
      stage_groups<CH, KIND>(p, stage0 + st * stage_bytes, b * rpb + team, b < nblk && b * rpb + team < p.rows, wt,
                             lane, ngroups);
      cp_async_commit();
    }
  }
  if (TAB) {
    const uint4 *src = reinterpret_cast<const uint4 *>(g_silu_bf16);
    uint4 *dst = reinterpret_cast<uint4 *>(smem);
    for (int i = threadIdx.x; i < kSiluEntries * 2 / 16; i += blockDim.x) dst[i] = src[i];
    __syncthreads();
  }
  int par = 0, st = 0;
  for (; blk < nblk; blk += gridDim.x, par ^= 1) {
    const int64_t row = blk * rpb + team;
    const bool row_ok = row < p.rows;
    if (STG == 0) fetch_groups<CH, KIND != KIND_PLAIN>(p, row, row_ok, wt, lane, ngroups, rx, ra);
    if (STG >= 2) {
      cp_async_wait<STG - 1>();  // this block's copies (all but the STG-1 newest groups)
      const uint32_t base = stage0 + st * stage_bytes + threadIdx.x * 16;
#pragma unroll
      for (int j = 0; j < CH; ++j) {
        rx[j] = lds_v4(base + (uint32_t)(j * NOP) * blockDim.x * 16);
        if (NOP == 2) ra[j] = lds_v4(base + (uint32_t)(j * NOP + 1) * blockDim.x * 16);
      }
    }

    // RMSNorm: 256 strided partial sums -> warp butterflies -> the 8 warp totals in order.
    float norm_inv = 1.0f;
    if (norm) {
      const uint16_t *xr = p.x + (row_ok ? row : 0) * p.x_ld;
      float s = 0.0f;
      for (int j = tid_team; j < p.width; j += 256) {
        float v = bf16_to_f32(xr[j]);
        s = __fmaf_rn(v, v, s);
      }
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
      float *ws = wsum + par * slots + team * tw;
      if (lane == 0) ws[wt] = s;
      __syncthreads();
      float total = ws[0];
      for (int w = 1; w < 8; ++w) total = __fadd_rn(total, ws[w]);
      float var = __fdiv_rn(total, (float)p.width);
      norm_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-6f)));
    }

    float v[CH][8];
#pragma unroll
    for (int j = 0; j < CH; ++j) {
      const uint16_t *h = reinterpret_cast<const uint16_t *>(&rx[j]);
      const uint16_t *a = reinterpret_cast<const uint16_t *>(&ra[j]);
      if (TAB) {
        const uint32_t *gw = reinterpret_cast<const uint32_t *>(&rx[j]);
        const uint32_t *uw = reinterpret_cast<const uint32_t *>(&ra[j]);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float lo = __fmul_rn(bf16_to_f32(tab[gw[k] & 0xffffu]), __uint_as_float(uw[k] << 16));
          float hi = __fmul_rn(bf16_to_f32(tab[gw[k] >> 16]), __uint_as_float(uw[k] & 0xffff0000u));
          bf16r_pair(lo, hi);
          v[j][2 * k] = lo;
          v[j][2 * k + 1] = hi;
        }
        continue;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) v[j][i] = bf16_to_f32(h[i]);
      if (KIND == KIND_PLAIN) continue;
      const int g = wt + j * tw;
      const bool active = row_ok && g < ngroups;
      if (active && p.mode == MODE_SWIGLU) {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[j][i] = bf16r(__fmul_rn(bf16_to_f32(silu_bf16(h[i])), bf16_to_f32(a[i])));
      } else if (active && p.mode == MODE_ATTN_GATE) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float sg = bf16r(__fdiv_rn(1.0f, __fadd_rn(1.0f, exp_cw(-bf16_to_f32(a[i])))));
          v[j][i] = bf16r(__fmul_rn(v[j][i], sg));
        }
      } else if (active && norm) {
        uint4 nh4;
        uint16_t *nh = reinterpret_cast<uint16_t *>(&nh4);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float wf = __fadd_rn(bf16_to_f32(a[i]), 1.0f);
          float nn = __fmul_rn(__fsub_rn(v[j][i], 0.0f), norm_inv);
          nh[i] = f32_to_bf16(__fmaf_rn(nn, wf, 0.0f));
          v[j][i] = bf16_to_f32(nh[i]);
        }
        if (p.mode == MODE_NORM_STORE)
          *reinterpret_cast<uint4 *>(p.norm_out + row * p.norm_ld + g * 256 + lane * 8) = nh4;
      }
    }
    // the stage is in registers now: refill it with the block STG iterations ahead
    if (STG >= 2) {
      const int64_t b = blk + (int64_t)STG * gridDim.x;
      stage_groups<CH, KIND>(p, stage0 + st * stage_bytes, b * rpb + team, b < nblk && b * rpb + team < p.rows, wt,
                             lane, ngroups);
      cp_async_commit();
      st = st + 1 == STG ? 0 : st + 1;
    }
    if (PF) {
      const int64_t nrow = (blk + gridDim.x) * rpb + team;
      fetch_groups<CH, KIND != KIND_PLAIN>(p, nrow, blk + gridDim.x < nblk && nrow < p.rows, wt, lane, ngroups, rx, ra);
    }

    // Rotation and row absmax; absent groups and rows hold zeros.  NaN propagates and
    // becomes +inf, like the reference's clamp of non-finite magnitudes.
    float m = 0.0f;
#pragma unroll
    for (int j = 0; j < CH; ++j) {
      hadamard256_lane(v[j]);
#pragma unroll
      for (int i = 0; i < 8; i += 2) m = absmax3_nan(m, v[j][i], v[j][i + 1]);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) m = max_nan(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (m != m) m = __int_as_float(0x7f800000);
    float *rs = red + par * slots + team * tw;
    if (lane == 0) rs[wt] = m;
    __syncthreads();
    // the team's maxima, one per lane, reduced across the lanes (tw <= 16)
    float rmax = lane < tw ? rs[lane] : 0.0f;
#pragma unroll
    for (int off = 8; off >= 1; off >>= 1) rmax = maxnum(rmax, __shfl_xor_sync(0xffffffffu, rmax, off));
    rmax = __shfl_sync(0xffffffffu, rmax, 0);
    if (!row_ok) continue;
    // split packing of a row sharded over several GPUs: publish this shard's maximum, or
    // quantise with the maximum over all shards
    if (p.rowmax_out) {
      if (tid_team == 0) p.rowmax_out[row] = rmax;
      continue;
    }
    if (p.rowmax_in) rmax = p.rowmax_in[row];

    const float scale = __fdiv_rn(maxnum(__fmul_rn(rmax, 0.0625f), 1e-30f), qmax);
    const float inv = __fdiv_rn(0.0625f, scale);
    uint32_t *orow = p.out + row * words;
    uint8_t *oprow = has_op ? p.op8 + row * p.op_ld + lane_op : nullptr;
    if (scale < __int_as_float(0x7f800000)) {
#pragma unroll
      for (int j = 0; j < CH; ++j) {
        const int g = wt + j * tw;
        if (g >= ngroups) continue;
        int c[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) c[i] = rint_s32(__fmul_rn(v[j][i], inv));
        if (bits == 4) {
          const uint32_t w = pack_s4(c[1], c[0], pack_s4(c[3], c[2], pack_s4(c[5], c[4], pack_s4(c[7], c[6], 0u))));
          orow[g * 32 + lane] = w;
          if (has_op) {
            // word g*32 + lane is word (lane & 3) of its 32-code group: the s8 operand holds
            // 16 * code, low nibbles of the group's 4 words first, then high nibbles
            *reinterpret_cast<uint32_t *>(oprow + g * 256) = nib_lo16(w);
            *reinterpret_cast<uint32_t *>(oprow + g * 256 + 16) = nib_hi16(w);
          }
        } else {
          *reinterpret_cast<uint2 *>(orow + g * 64 + lane * 2) =
              make_uint2(pack_s8(c[1], c[0], pack_s8(c[3], c[2], 0u)), pack_s8(c[5], c[4], pack_s8(c[7], c[6], 0u)));
        }
      }
    } else {
      // a non-finite row: zero codes, infinite scale
#pragma unroll
      for (int j = 0; j < CH; ++j) {
        const int g = wt + j * tw;
        if (g >= ngroups) continue;
        if (bits == 4) {
          orow[g * 32 + lane] = 0u;
          if (has_op) {
            *reinterpret_cast<uint32_t *>(oprow + g * 256) = 0u;
            *reinterpret_cast<uint32_t *>(oprow + g * 256 + 16) = 0u;
          }
        } else {
          *reinterpret_cast<uint2 *>(orow + g * 64 + lane * 2) = make_uint2(0u, 0u);
        }
      }
    }
    // Stride padding words are zeroed; the scale follows all code rows.
    for (int w = code_words + tid_team; w < words; w += tw * 32) orow[w] = 0u;
    if (tid_team == 0) reinterpret_cast<float *>(p.out + p.rows * words)[row] = scale;
  }
  if (STG >= 2) cp_async_wait<0>();
}

// ---------------------------------------------------------------------------------------
// GEMM-input packing (int4 codes + s8 operand, no pre-op or SwiGLU through the table).
// Eight lanes share a group and a lane holds 32 of its elements: element
// e = 64 k + 8 r + t (r = lane & 7, k = 0..3, t = 0..7) sits in v[8 k + t], so a warp
// covers four groups per slot and every 16-byte load of the eight lanes is one contiguous
// 128-byte line.  Hadamard strides 1 and 64 run inside the lane, stride 4 pairs lane r
// with r ^ 1 (one shuffle per two elements), stride 16 spans lanes r, r ^ 2, r ^ 4, r ^ 6:
// 9 adds and 2.5 shuffles per element.  For each k a lane's eight codes are one code word.
// ---------------------------------------------------------------------------------------
CQ_DEV void radix4_in_lane(float &a, float &b, float &c, float &d) {
  const float s01 = __fadd_rn(a, b), s23 = __fadd_rn(c, d), d01 = __fsub_rn(a, b), d23 = __fsub_rn(c, d);
  a = __fadd_rn(s01, d23);
  b = __fsub_rn(s01, d23);
  c = __fadd_rn(d01, s23);
  d = __fsub_rn(s23, d01);
}

CQ_DEV void hadamard256_x32(float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 32; q += 4) radix4_in_lane(v[q], v[q + 1], v[q + 2], v[q + 3]);  // stride 1
  // stride 4: (a, b) = (v[8k+u], v[8k+u+4]) of the even lane, (c, d) of the odd lane
#pragma unroll
  for (int k = 0; k < 4; ++k) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float x = v[8 * k + u], y = v[8 * k + u + 4];
      const float s = __fadd_rn(x, y), d = __fsub_rn(x, y);
      const float p2 = __shfl_xor_sync(0xffffffffu, d, 1);
      v[8 * k + u] = __fadd_rn(s, p2);
      v[8 * k + u + 4] = __fsub_rn(s, p2);
    }
  }
  radix4_lanes(v, 2, 4);  // stride 16
#pragma unroll
  for (int t = 0; t < 8; ++t) radix4_in_lane(v[t], v[8 + t], v[16 + t], v[24 + t]);  // stride 64
}

CQ_DEV void cp_async_wait_dyn(int n) {
  if (n <= 0) cp_async_wait<0>();
  else if (n == 1) cp_async_wait<1>();
  else if (n == 2) cp_async_wait<2>();
  else cp_async_wait<3>();
}

constexpr int kPackRedBytes = 2 * 64 * 4;  // [2][64] team maxima (16 warps x 4 teams)

// NS slots (of four groups) per warp, team_warps warps per row, rows_per_block rows per
// CTA; p.stages cp.async stages per thread of NS x NOP x 64 bytes each.
template <int NS, bool TAB>
__global__ void __launch_bounds__(512, 1) pack_kernel(PrepareArgs p) {
  // launched with programmatic stream serialization: the input is the previous kernel's output
  pdl_wait();
  pdl_trigger();
  constexpr int NOP = TAB ? 2 : 1;
  extern __shared__ __align__(16) uint8_t smem[];
  const uint16_t *tab = reinterpret_cast<const uint16_t *>(smem);
  float *red = reinterpret_cast<float *>(smem + (TAB ? kSiluEntries * 2 : 0));  // [2][slots]
  const int tw = p.team_warps, rpb = p.rows_per_block, slots = tw * rpb;
  const int nstg = p.stages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int team = warp / tw, wt = warp % tw;
  const int tid_team = wt * 32 + lane;
  const int ngroups = p.width >> 8;
  const int words = p.stride >> 3;
  const int code_words = p.width >> 3;
  const int q = lane >> 3, r = lane & 7;
  // Narrow rows (G = 1..3 groups, NS = 1): each 8-lane team packs one group of one row, so a
  // 16-warp block holds rpb = 64 / G rows and no team idles; the row maximum goes through
  // shared memory.  Otherwise tw warps share a row and each team packs groups 4 apart.
  const int G = NS == 1 ? p.narrow : 0;
  const int Gd = G ? G : 1;      // divisor that is never zero
  const int tau = warp * 4 + q;  // team of the block
  const int tgroup = tau % Gd;   // narrow: this team's group of its row
  const int team_row = G ? tau / Gd : team;
  const bool team_on = G ? tau < rpb * G : true;
  const bool row_leader = G ? (team_on && tgroup == 0 && r == 0) : tid_team == 0;
  // rows to pack: p.rows, or fewer when the count is only known on the device (the code
  // and scale layout always spans p.rows)
  int64_t nrows = p.rows;
  if (p.rows_dev) {
    const int64_t d = *p.rows_dev;
    nrows = d < 0 ? 0 : (d < p.rows ? d : p.rows);
  }
  const int64_t nblk = (nrows + rpb - 1) / rpb;
  const uint32_t stage0 = smem_u32(smem + (TAB ? kSiluEntries * 2 : 0) + kPackRedBytes);
  const uint32_t chunk = blockDim.x * 16;                    // one 16-byte chunk per thread
  const uint32_t stage_bytes = (uint32_t)(NS * NOP * 4) * chunk;
  int gidx[NS];                                              // this lane's group per slot
#pragma unroll
  for (int sl = 0; sl < NS; ++sl) gidx[sl] = G ? (team_on ? tgroup : ngroups) : (sl * tw + wt) * 4 + q;

  auto issue = [&](int64_t b, int stg) {
    const int64_t row = b * rpb + team_row;
    const bool ok = b < nblk && row < nrows;
    const uint32_t base = stage0 + stg * stage_bytes + threadIdx.x * 16;
#pragma unroll
    for (int sl = 0; sl < NS; ++sl) {
      const bool valid = ok && gidx[sl] < ngroups;
      const int64_t off = row * p.x_ld + gidx[sl] * 256 + r * 8;
      const int64_t aoff = row * p.aux_ld + gidx[sl] * 256 + r * 8;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        cp_async16(base + ((sl * NOP) * 4 + k) * chunk, valid ? (const void *)(p.x + off + k * 64) : (const void *)p.x,
                   valid);
        if (NOP == 2)
          cp_async16(base + ((sl * NOP + 1) * 4 + k) * chunk,
                     valid ? (const void *)(p.aux + aoff + k * 64) : (const void *)p.x, valid);
      }
    }
    cp_async_commit();
  };

  int64_t blk = blockIdx.x;
  for (int st = 0; st < nstg; ++st) issue(blk + (int64_t)st * gridDim.x, st);
  if (TAB) {
    const uint4 *src = reinterpret_cast<const uint4 *>(g_silu_bf16);
    uint4 *dst = reinterpret_cast<uint4 *>(smem);
    for (int i = threadIdx.x; i < kSiluEntries * 2 / 16; i += blockDim.x) dst[i] = src[i];
    __syncthreads();
  }
  int par = 0, st = 0;
  for (; blk < nblk; blk += gridDim.x, par ^= 1) {
    const int64_t row = blk * rpb + team_row;
    const bool row_ok = team_on && row < nrows;
    cp_async_wait_dyn(nstg - 1);  // this block's copies (all but the nstg-1 newest groups)
    const uint32_t base = stage0 + st * stage_bytes + threadIdx.x * 16;
    float v[NS][32];
#pragma unroll
    for (int sl = 0; sl < NS; ++sl) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint4 gx = lds_v4(base + ((sl * NOP) * 4 + k) * chunk);
        const uint32_t gw[4] = {gx.x, gx.y, gx.z, gx.w};
        if (TAB) {
          const uint4 ux = lds_v4(base + ((sl * NOP + 1) * 4 + k) * chunk);
          const uint32_t uw[4] = {ux.x, ux.y, ux.z, ux.w};
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            float lo = __fmul_rn(bf16_to_f32(tab[gw[t] & 0xffffu]), __uint_as_float(uw[t] << 16));
            float hi = __fmul_rn(bf16_to_f32(tab[gw[t] >> 16]), __uint_as_float(uw[t] & 0xffff0000u));
            bf16r_pair(lo, hi);
            v[sl][8 * k + 2 * t] = lo;
            v[sl][8 * k + 2 * t + 1] = hi;
          }
        } else {
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            v[sl][8 * k + 2 * t] = __uint_as_float(gw[t] << 16);
            v[sl][8 * k + 2 * t + 1] = __uint_as_float(gw[t] & 0xffff0000u);
          }
        }
      }
    }
    // the stage is in registers now: refill it with the block nstg iterations ahead
    issue(blk + (int64_t)nstg * gridDim.x, st);
    st = st + 1 == nstg ? 0 : st + 1;

    float m = 0.0f;
#pragma unroll
    for (int sl = 0; sl < NS; ++sl) {
      hadamard256_x32(v[sl]);
#pragma unroll
      for (int i = 0; i < 32; i += 2) m = absmax3_nan(m, v[sl][i], v[sl][i + 1]);
    }
    float rmax = 0.0f;
    if (G) {
      // the team's group maximum, then the maximum over the row's G teams
#pragma unroll
      for (int off = 4; off >= 1; off >>= 1) m = max_nan(m, __shfl_xor_sync(0xffffffffu, m, off));
      if (m != m) m = __int_as_float(0x7f800000);
      float *rs = red + par * 64;
      if (r == 0) rs[tau] = m;
      __syncthreads();
      if (team_on) {
        const int first = tau - tgroup;
        for (int j = 0; j < G; ++j) rmax = maxnum(rmax, rs[first + j]);
      }
    } else {
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) m = max_nan(m, __shfl_xor_sync(0xffffffffu, m, off));
      if (m != m) m = __int_as_float(0x7f800000);
      float *rs = red + par * slots + team * tw;
      if (lane == 0) rs[wt] = m;
      __syncthreads();
      rmax = lane < tw ? rs[lane] : 0.0f;
#pragma unroll
      for (int off = 8; off >= 1; off >>= 1) rmax = maxnum(rmax, __shfl_xor_sync(0xffffffffu, rmax, off));
      rmax = __shfl_sync(0xffffffffu, rmax, 0);
    }
    if (!row_ok) continue;
    if (p.rowmax_out) {
      if (row_leader) p.rowmax_out[row] = rmax;
      continue;
    }
    if (p.rowmax_in) rmax = p.rowmax_in[row];

    const float scale = __fdiv_rn(maxnum(__fmul_rn(rmax, 0.0625f), 1e-30f), 7.0f);
    const float inv = __fdiv_rn(0.0625f, scale);
    const bool finite = scale < __int_as_float(0x7f800000);
    uint32_t *orow = p.out + row * words;
    constexpr bool DUP = !TAB && NS == 1;  // instance that can write the operand to several rows
    int drow[kMaxDup];
    if (DUP && p.dup) {
#pragma unroll
      for (int d = 0; d < kMaxDup; ++d) drow[d] = d < p.dup ? p.dup_rows[row * p.dup + d] : -1;
    }
#pragma unroll
    for (int sl = 0; sl < NS; ++sl) {
      const int g = gidx[sl];
      if (g >= ngroups) continue;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint32_t w = 0u;
        if (finite) {
          int c[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) c[i] = rint_s32(__fmul_rn(v[sl][8 * k + i], inv));
          w = pack_s4(c[1], c[0], pack_s4(c[3], c[2], pack_s4(c[5], c[4], pack_s4(c[7], c[6], 0u))));
        }
        // code word g*32 + 8k + r is word (r & 3) of its 32-code operand block: the s8
        // operand holds 16 * code, low nibbles of the block's 4 words first, then high
        orow[g * 32 + 8 * k + r] = w;
        if (TAB && p.n_code_dst) {
          // eight lanes store 32 contiguous bytes: whole sectors, also over NVLink
          const int64_t cw = row * p.code_ld + g * 32 + 8 * k + r;
#pragma unroll
          for (int d = 0; d < kMaxRanks; ++d)
            if (d < p.n_code_dst) p.code_dst[d][cw] = w;
        }
        if (p.op8) {
          const int off = g * 256 + k * 64 + (r >> 2) * 32 + (r & 3) * 4;
          const uint32_t lo = nib_lo16(w), hi = nib_hi16(w);
          if (DUP && p.dup) {
            // the row's operand goes to each of its routes' expert-sorted rows
#pragma unroll
            for (int d = 0; d < kMaxDup; ++d) {
              if (drow[d] < 0) continue;
              uint8_t *op = p.op8 + (int64_t)drow[d] * p.op_ld + off;
              *reinterpret_cast<uint32_t *>(op) = lo;
              *reinterpret_cast<uint32_t *>(op + 16) = hi;
            }
          } else {
            uint8_t *op = p.op8 + row * p.op_ld + off;
            *reinterpret_cast<uint32_t *>(op) = lo;
            *reinterpret_cast<uint32_t *>(op + 16) = hi;
          }
        }
      }
    }
    // Stride padding words are zeroed; the scale follows all code rows.
    if (!G) {
      for (int w = code_words + tid_team; w < words; w += tw * 32) orow[w] = 0u;
    } else if (tgroup == 0) {
      for (int w = code_words + r; w < words; w += 8) orow[w] = 0u;
    }
    if (row_leader) reinterpret_cast<float *>(p.out + p.rows * words)[row] = scale;
  }
  cp_async_wait<0>();
  // Code words stored into other ranks' buffers are made visible at system scope by the
  // thread that stored them, before the kernel ends: the barrier kernel that follows raises
  // the peers' flags from one thread, and its fence orders only what that thread observed.
  if (TAB && p.n_code_dst) __threadfence_system();
}

namespace {
// Per-device launch facts of one kernel instance: resident CTAs per SM for a block size.
// The dynamic shared-memory limit is one attribute per kernel, so it is raised once per
// device to what the instance can need at its largest block (512 threads, 16 team slots).
constexpr int kMaxDevices = 64;
template <int CH, int KIND>
size_t max_smem_bytes() {
  constexpr int STG = stages_for(CH, KIND);
  return (KIND == KIND_SILU_TABLE ? kSiluEntries * 2 : 0) + sizeof(float) * 4 * 16 +
         (STG >= 2 ? (size_t)STG * CH * operands_for(KIND) * 512 * 16 : 0);
}

template <int CH, int KIND>
int resident_ctas(int threads, size_t smem) {
  // Filled on first use by whichever host thread gets there; concurrent fillers compute the
  // same values, and the release/acquire pair orders the attribute call before its flag.
  static std::atomic<int> cache[kMaxDevices][17];
  static std::atomic<bool> attr[kMaxDevices];
  int dev = 0;
  cudaGetDevice(&dev);
  const int warps = threads / 32 > 16 ? 16 : threads / 32;
  if (dev < 0 || dev >= kMaxDevices) return 1;
  if (!attr[dev].load(std::memory_order_acquire)) {
    const size_t most = max_smem_bytes<CH, KIND>();
    if (most > 48 * 1024)
      cudaFuncSetAttribute(prepare_kernel<CH, KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)most);
    attr[dev].store(true, std::memory_order_release);
  }
  int n = cache[dev][warps].load(std::memory_order_relaxed);
  if (!n) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, prepare_kernel<CH, KIND>, threads, smem) != cudaSuccess ||
        n <= 0)
      n = 1;
    cache[dev][warps].store(n, std::memory_order_relaxed);
  }
  return n;
}

// Launch with programmatic stream serialization (the kernels wait for the previous kernel
// in-kernel, pdl_wait), so their start overlaps the previous kernel's last blocks.
void launch_pdl(void (*kern)(PrepareArgs), unsigned grid, int threads, size_t smem, cudaStream_t stream,
                const PrepareArgs &a) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = CLEFQ_PDL_PREPARE;
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kern, a);
}

template <int CH, int KIND>
void launch_instance(const PrepareArgs &a, int threads, size_t smem0, int64_t nblk, cudaStream_t stream) {
  constexpr int STG = stages_for(CH, KIND);
  const size_t smem = smem0 + (STG >= 2 ? (size_t)STG * CH * operands_for(KIND) * threads * 16 : 0);
  const int per_sm = resident_ctas<CH, KIND>(threads, smem);
  int64_t grid = (int64_t)device_sms() * per_sm;
  if (grid > nblk) grid = nblk;
  launch_pdl(prepare_kernel<CH, KIND>, (unsigned)grid, threads, smem, stream, a);
}

template <int KIND>
bool launch_kind(int ch, const PrepareArgs &a, int threads, size_t smem, int64_t nblk, cudaStream_t stream) {
  switch (ch) {
    case 1: launch_instance<1, KIND>(a, threads, smem, nblk, stream); return true;
    case 2: launch_instance<2, KIND>(a, threads, smem, nblk, stream); return true;
    case 3: launch_instance<3, KIND>(a, threads, smem, nblk, stream); return true;
    case 4: launch_instance<4, KIND>(a, threads, smem, nblk, stream); return true;
    case 5: launch_instance<5, KIND>(a, threads, smem, nblk, stream); return true;
    case 6: launch_instance<6, KIND>(a, threads, smem, nblk, stream); return true;
    case 7: launch_instance<7, KIND>(a, threads, smem, nblk, stream); return true;
    case 8: launch_instance<8, KIND>(a, threads, smem, nblk, stream); return true;
  }
  return false;
}
}  // namespace

namespace {
template <int NS, bool TAB>
void launch_pack(const PrepareArgs &a, int threads, size_t smem, int64_t nblk, cudaStream_t stream) {
  static std::atomic<bool> attr[kMaxDevices];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices || !attr[dev].load(std::memory_order_acquire)) {
    // largest request of this instance: table + maxima + the stage budget
    const int most = (TAB ? kSiluEntries * 2 : 0) + kPackRedBytes + (TAB ? 96 : 128) * 1024;
    cudaFuncSetAttribute(pack_kernel<NS, TAB>, cudaFuncAttributeMaxDynamicSharedMemorySize, most);
    if (dev >= 0 && dev < kMaxDevices) attr[dev].store(true, std::memory_order_release);
  }
  int64_t grid = device_sms();
  if (grid > nblk) grid = nblk;
  launch_pdl(pack_kernel<NS, TAB>, (unsigned)grid, threads, smem, stream, a);
}

// GEMM-input packing: int4 codes with the s8 operand, 16-byte aligned rows, no pre-op or
// SwiGLU through the table.  Returns false when the shape needs the general kernel.
bool try_launch_pack(PrepareArgs a, bool tab, cudaStream_t stream) {
  const int ngroups = a.width >> 8;
  const int sg = (ngroups + 3) / 4;  // slots of four groups
  const int ns = (sg + 15) / 16;
  if (ns > (tab ? 1 : 2) || (a.dup && (tab || ns != 1))) return false;
  const int tw = (sg + ns - 1) / ns;
  // rows of fewer than four groups: one group per 8-lane team (narrow mode), 64 / G rows per
  // 16-warp block; wider rows: tw warps per row
  const bool narrow = ngroups < 4 && ns == 1;
  const int rpb = narrow ? 64 / ngroups : (16 / tw > 0 ? 16 / tw : 1);
  const int threads = narrow ? 512 : tw * 32 * rpb;
  a.narrow = narrow ? ngroups : 0;
  const size_t per_stage = (size_t)threads * ns * (tab ? 2 : 1) * 64;
  int stages = (int)(((tab ? 96 : 128) * 1024) / per_stage);
  if (stages > 4) stages = 4;
  if (stages < 1) return false;
  a.team_warps = tw;
  a.rows_per_block = rpb;
  a.stages = stages;
  const size_t smem = (tab ? kSiluEntries * 2 : 0) + kPackRedBytes + stages * per_stage;
  const int64_t nblk = (a.rows + rpb - 1) / rpb;
  if (ns == 1)
    tab ? launch_pack<1, true>(a, threads, smem, nblk, stream) : launch_pack<1, false>(a, threads, smem, nblk, stream);
  else
    launch_pack<2, false>(a, threads, smem, nblk, stream);
  return true;
}
}  // namespace

int launch_prepare(const PrepareArgs &a0, cudaStream_t stream) {
  PrepareArgs a = a0;
  const int ngroups = a.width >> 8;
  const bool norm = a.mode == MODE_NORM || a.mode == MODE_NORM_STORE;
  if (a.rows == 0) return 0;
  // int4 codes (plain, or with the operand / row maxima / extra code destinations) take the
  // persistent packing kernels; everything else the general one
  const bool gemm_input = a.bits == 4 &&
                          (a.op8 != nullptr || a.rowmax_out != nullptr || a.n_code_dst > 0 || a.mode == MODE_PLAIN) &&
                          ((uintptr_t)a.out & 15) == 0 &&
                          (a.x_ld & 7) == 0 && (a.mode != MODE_SWIGLU || (a.aux_ld & 7) == 0);
  // The table pays for its 128 KB shared-memory fill once a launch has about a full
  // wave of groups to process; small launches evaluate the activation directly.
  // Extra code destinations and device row counts exist only in the GEMM-input kernel, so
  // they take the table at any size.
  const bool tab = gemm_input && a.mode == MODE_SWIGLU &&
                   (a.rows * (int64_t)ngroups >= 2048 || a.n_code_dst || a.rows_dev);
  if (a.n_code_dst && !tab)
    return report_error(CLEFQ_ERR_SHAPE, "prepare: extra code destinations are for SwiGLU GEMM-input packing");
  if (a.rows_dev && !(gemm_input && (a.mode == MODE_PLAIN || tab)))
    return report_error(CLEFQ_ERR_SHAPE, "prepare: a device row count needs the GEMM-input kernel");
  if (a.dup && (a.dup > kMaxDup || !a.dup_rows || !a.op8 || !gemm_input || a.mode != MODE_PLAIN))
    return report_error(CLEFQ_ERR_SHAPE, "prepare: operand rows per input row need plain int4 GEMM-input packing");
  if (gemm_input && (a.mode == MODE_PLAIN || tab) && try_launch_pack(a, tab, stream)) {
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : report_error(CLEFQ_ERR_CUDA, cudaGetErrorString(e));
  }
  if (a.n_code_dst || a.rows_dev || a.dup)
    return report_error(CLEFQ_ERR_SHAPE, "prepare: this launch shape needs the GEMM-input kernel");
  int tw, ch;
  if (norm) {
    tw = 8;  // the reference's 256-thread reduction order
    ch = (ngroups + 7) / 8;
  } else {
    ch = ngroups >= 2 ? 2 : 1;
    if ((ngroups + ch - 1) / ch > 16) ch = (ngroups + 15) / 16;
    tw = (ngroups + ch - 1) / ch;
  }
  if (ch < 1 || ch > 8 || tw < 1) return report_error(CLEFQ_ERR_SHAPE, "prepare: row width above the supported maximum");
  const int rpb = 16 / tw > 0 ? 16 / tw : 1;
  a.team_warps = tw;
  a.rows_per_block = rpb;
  const int threads = tw * 32 * rpb;
  const int64_t nblk = (a.rows + rpb - 1) / rpb;
  const size_t smem = sizeof(float) * 4 * (size_t)(tw * rpb);
  if (!launch_kind<KIND_GENERAL>(ch, a, threads, smem, nblk, stream))
    return report_error(CLEFQ_ERR_SHAPE, "prepare: no kernel for this row width");
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : report_error(CLEFQ_ERR_CUDA, cudaGetErrorString(e));
}

// ---------------------------------------------------------------------------------------
// SwiGLU: bf16(bf16(g / (1 + exp(-g))) * u), eight elements per thread.
// ---------------------------------------------------------------------------------------
__global__ void swiglu_kernel(const uint16_t *__restrict__ g, const uint16_t *__restrict__ u, uint16_t *__restrict__ out,
                              int64_t n8) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    uint4 gr = reinterpret_cast<const uint4 *>(g)[i];
    uint4 ur = reinterpret_cast<const uint4 *>(u)[i];
    const uint16_t *gh = reinterpret_cast<const uint16_t *>(&gr);
    const uint16_t *uh = reinterpret_cast<const uint16_t *>(&ur);
    uint4 o;
    uint16_t *oh = reinterpret_cast<uint16_t *>(&o);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      oh[k] = f32_to_bf16(__fmul_rn(bf16_to_f32(silu_bf16(gh[k])), bf16_to_f32(uh[k])));
    }
    reinterpret_cast<uint4 *>(out)[i] = o;
  }
}
__global__ void swiglu_tail_kernel(const uint16_t *g, const uint16_t *u, uint16_t *out, int64_t start, int64_t n) {
  int64_t i = start + blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i < n) {
    out[i] = f32_to_bf16(__fmul_rn(bf16_to_f32(silu_bf16(g[i])), bf16_to_f32(u[i])));
  }
}

// SiLU of n BF16 values as the SwiGLU GEMM epilogue computes it (silu_bf16_ziv).
__global__ void silu_kernel(const uint16_t *__restrict__ x, uint16_t *__restrict__ out, int64_t n,
                            const uint16_t *__restrict__ tab) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = (uint16_t)silu_bf16_ziv(x[i], tab);
}

int launch_silu(const uint16_t *x, uint16_t *out, int64_t n, cudaStream_t stream, int num_sms) {
  const uint16_t *tab = silu_table_device();
  if (!tab) return (int)cudaErrorInvalidSymbol;
  const int64_t blocks = (n + 255) / 256, cap = (int64_t)num_sms * 8;
  silu_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, stream>>>(x, out, n, tab);
  return launch_check();
}

int launch_swiglu(const uint16_t *g, const uint16_t *u, uint16_t *out, int64_t n, cudaStream_t stream,
                  int num_sms) {
  const int64_t n8 = n / 8;
  bool aligned = ((uintptr_t)g % 16 == 0) && ((uintptr_t)u % 16 == 0) && ((uintptr_t)out % 16 == 0);
  int64_t done = 0;
  if (aligned && n8 > 0) {
    int64_t blocks = (n8 + 255) / 256;
    int64_t cap = (int64_t)num_sms * 8;
    swiglu_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, stream>>>(g, u, out, n8);
    done = n8 * 8;
  }
  if (done < n) {
    int64_t rest = n - done;
    swiglu_tail_kernel<<<(unsigned)((rest + 255) / 256), 256, 0, stream>>>(g, u, out, done, n);
  }
  return launch_check();
}

// ---------------------------------------------------------------------------------------
// retile: word (n, q) -> ((n/128)*blocks_k + q/32)*4096 + (n%128)*32 + q%32, four words
// (16 bytes) per thread on both sides.
// ---------------------------------------------------------------------------------------
__global__ void retile_kernel(const uint32_t *__restrict__ codes, int64_t in_words, int64_t words, int64_t rows,
                              uint32_t *__restrict__ out) {
  const int64_t total4 = rows * words / 4;
  const int64_t blocks_k = words / 32;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total4; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = i * 4;
    const int64_t block = o / 4096, within = o % 4096;
    const int64_t r = within / 32, c = within % 32;
    const int64_t n = (block / blocks_k) * 128 + r, q = (block % blocks_k) * 32 + c;
    const uint32_t *src = codes + n * in_words + q;
    uint4 val;
    if ((in_words & 3) == 0) {
      val = *reinterpret_cast<const uint4 *>(src);
    } else {
      val = make_uint4(src[0], src[1], src[2], src[3]);
    }
    *reinterpret_cast<uint4 *>(out + o) = val;
  }
}

int launch_retile(const uint32_t *codes, int64_t rows, int64_t in_words, int64_t words, uint32_t *out,
                  cudaStream_t stream, int num_sms) {
  const int64_t total4 = rows * words / 4;
  if (total4 == 0) return 0;
  int64_t blocks = (total4 + 255) / 256, cap = (int64_t)num_sms * 16;
  retile_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, stream>>>(codes, in_words, words, rows, out);
  return launch_check();
}

// ---------------------------------------------------------------------------------------
// unpack: packed int4 codes [rows][a_ld words] -> s8 operand [rows][op_ld bytes], k < K.
// One thread per 4 words (32 codes) -> 32 operand bytes.
// ---------------------------------------------------------------------------------------
__global__ void unpack_i4_kernel(const uint32_t *__restrict__ a, int64_t a_ld, int64_t rows, int k, uint8_t *__restrict__ op,
                                 int64_t op_ld) {
  const int groups = k / 32;
  const int64_t total = rows * groups;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / groups;
    const int gq = (int)(i % groups);
    const uint32_t *src = a + r * a_ld + gq * 4;
    uint32_t w0, w1, w2, w3;
    if ((a_ld & 3) == 0) {
      uint4 v = *reinterpret_cast<const uint4 *>(src);
      w0 = v.x; w1 = v.y; w2 = v.z; w3 = v.w;
    } else {
      w0 = src[0]; w1 = src[1]; w2 = src[2]; w3 = src[3];
    }
    uint4 lo = make_uint4(nib_lo16(w0), nib_lo16(w1), nib_lo16(w2), nib_lo16(w3));
    uint4 hi = make_uint4(nib_hi16(w0), nib_hi16(w1), nib_hi16(w2), nib_hi16(w3));
    uint4 *dst = reinterpret_cast<uint4 *>(op + r * op_ld + gq * 32);
    dst[0] = lo;
    dst[1] = hi;
  }
}

int launch_unpack_i4(const uint32_t *a, int64_t a_ld, int64_t rows, int k, uint8_t *op, int64_t op_ld,
                     cudaStream_t stream, int num_sms) {
  const int64_t total = rows * (k / 32);
  if (total == 0) return 0;
  int64_t blocks = (total + 255) / 256, cap = (int64_t)num_sms * 16;
  unpack_i4_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, stream>>>(a, a_ld, rows, k, op, op_ld);
  return launch_check();
}

}  // namespace cq
