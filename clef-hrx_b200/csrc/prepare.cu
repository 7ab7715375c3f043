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
// Layout of one row in registers: a warp owns a 256-element Hadamard group, each lane
// eight consecutive elements.  Radix-4 stride 1 runs inside a lane; strides 4, 16 and 64
// exchange partial sums/differences with xor-shuffles, keeping the reference's exact
// operation order (s01 = a+b, s23 = c+d, d01 = a-b, d23 = c-d; o = s01+d23, s01-d23,
// d01+s23, s23-d01), which is bit-identical under IEEE commutativity.
#include "cq_common.cuh"
#include "clefq_internal.h"

namespace cq {

enum { MODE_PLAIN = 0, MODE_SWIGLU = 1, MODE_ATTN_GATE = 2, MODE_NORM = 3, MODE_NORM_STORE = 4 };


// One radix-4 stage across lanes.  Lane bits (xbit, ybit) select the element's role in
// the quad (a: 0,0  b: 1,0  c: 0,1  d: 1,1).
CQ_DEV void radix4_lanes(float (&v)[8], int lane, int xmask, int ymask) {
  const bool bx = (lane & xmask) != 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float own = v[i];
    float peer = __shfl_xor_sync(0xffffffffu, own, xmask);
    float s = __fadd_rn(own, peer);                              // a+b or c+d
    float d = bx ? __fsub_rn(peer, own) : __fsub_rn(own, peer);  // a-b or c-d
    float p2 = __shfl_xor_sync(0xffffffffu, d, ymask);
    v[i] = bx ? __fsub_rn(s, p2) : __fadd_rn(s, p2);
  }
}

CQ_DEV void hadamard256_lane(float (&v)[8], int lane) {
  // stride 1: two quads inside the lane
#pragma unroll
  for (int q = 0; q < 8; q += 4) {
    float a = v[q], b = v[q + 1], c = v[q + 2], d = v[q + 3];
    float s01 = __fadd_rn(a, b), s23 = __fadd_rn(c, d), d01 = __fsub_rn(a, b), d23 = __fsub_rn(c, d);
    v[q] = __fadd_rn(s01, d23);
    v[q + 1] = __fsub_rn(s01, d23);
    v[q + 2] = __fadd_rn(d01, s23);
    v[q + 3] = __fsub_rn(s23, d01);
  }
  // stride 4: (a, b) = (v[i], v[i+4]) of the even lane, (c, d) of the odd lane
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float x = v[i], y = v[i + 4];
    float s = __fadd_rn(x, y), d = __fsub_rn(x, y);
    float p2 = __shfl_xor_sync(0xffffffffu, d, 1);
    v[i] = __fadd_rn(s, p2);
    v[i + 4] = __fsub_rn(s, p2);
  }
  radix4_lanes(v, lane, 2, 4);    // stride 16
  radix4_lanes(v, lane, 8, 16);   // stride 64
}

template <int CH>
__global__ void __launch_bounds__(512) prepare_kernel(PrepareArgs p) {
  extern __shared__ float red[];  // [rows_per_block][team_warps] maxima, then norm partials
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int team = warp / p.team_warps, wt = warp % p.team_warps;
  const int64_t row = (int64_t)blockIdx.x * p.rows_per_block + team;
  const bool row_ok = row < p.rows;
  const int ngroups = p.width >> 8;
  const int bits = p.bits;
  const int P = 32 / bits;
  const int words = p.stride / P;
  const uint16_t *xr = p.x + (row_ok ? row : 0) * p.x_ld;

  // RMSNorm: 256 strided partial sums -> warp butterflies -> warp totals in order.
  float norm_inv = 1.0f;
  if (p.mode == MODE_NORM || p.mode == MODE_NORM_STORE) {
    float s = 0.0f;
    for (int j = threadIdx.x; j < p.width; j += 256) {
      float v = bf16_to_f32(xr[j]);
      s = __fmaf_rn(v, v, s);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
    float *wsum = red + p.rows_per_block * p.team_warps;
    if (lane == 0) wsum[warp] = s;
    __syncthreads();
    float total = wsum[0];
    for (int w = 1; w < 8; ++w) total = __fadd_rn(total, wsum[w]);
    float var = __fdiv_rn(total, (float)p.width);
    norm_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-6f)));
  }

  float v[CH][8];
  float m = 0.0f;
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    const int g = wt + j * p.team_warps;
    const bool active = row_ok && g < ngroups;
    const int col0 = g * 256 + lane * 8;
    uint4 raw = make_uint4(0, 0, 0, 0);
    if (active) raw = *reinterpret_cast<const uint4 *>(xr + col0);
    const uint16_t *h = reinterpret_cast<const uint16_t *>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[j][i] = bf16_to_f32(h[i]);
    if (active && p.mode != MODE_PLAIN) {
      if (p.mode == MODE_SWIGLU) {
        uint4 uraw = *reinterpret_cast<const uint4 *>(p.aux + row * p.aux_ld + col0);
        const uint16_t *u = reinterpret_cast<const uint16_t *>(&uraw);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float g0 = v[j][i];
          float act = __fdiv_rn(g0, __fadd_rn(1.0f, exp_cw(-g0)));
          v[j][i] = bf16r(__fmul_rn(bf16r(act), bf16_to_f32(u[i])));
        }
      } else if (p.mode == MODE_ATTN_GATE) {
        const int head = col0 >> 8, within = col0 & 255;
        uint4 qraw = *reinterpret_cast<const uint4 *>(p.aux + row * p.aux_ld + head * 512 + 256 + within);
        const uint16_t *q = reinterpret_cast<const uint16_t *>(&qraw);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float sg = bf16r(__fdiv_rn(1.0f, __fadd_rn(1.0f, exp_cw(-bf16_to_f32(q[i])))));
          v[j][i] = bf16r(__fmul_rn(v[j][i], sg));
        }
      } else {
        uint4 wraw = *reinterpret_cast<const uint4 *>(p.aux + col0);
        const uint16_t *w = reinterpret_cast<const uint16_t *>(&wraw);
        uint16_t nh[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float wf = __fadd_rn(bf16_to_f32(w[i]), 1.0f);
          float nn = __fmul_rn(__fsub_rn(v[j][i], 0.0f), norm_inv);
          nh[i] = f32_to_bf16(__fmaf_rn(nn, wf, 0.0f));
          v[j][i] = bf16_to_f32(nh[i]);
        }
        if (p.mode == MODE_NORM_STORE)
          *reinterpret_cast<uint4 *>(p.norm_out + row * p.norm_ld + col0) = *reinterpret_cast<uint4 *>(nh);
      }
    }
    hadamard256_lane(v[j], lane);
    if (active) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float a = fabsf(v[j][i]);
        m = maxnum(m, a < __int_as_float(0x7f800000) ? a : __int_as_float(0x7f800000));
      }
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) m = maxnum(m, __shfl_xor_sync(0xffffffffu, m, off));
  if (lane == 0) red[team * p.team_warps + wt] = m;
  __syncthreads();
  float rmax = 0.0f;
  for (int w = 0; w < p.team_warps; ++w) rmax = maxnum(rmax, red[team * p.team_warps + w]);
  if (!row_ok) return;

  const float qmax = bits == 8 ? 127.0f : 7.0f;
  const float scale = __fdiv_rn(maxnum(__fmul_rn(rmax, 0.0625f), 1e-30f), qmax);
  const bool valid = scale < __int_as_float(0x7f800000);
  const float inv = __fdiv_rn(0.0625f, scale);
  uint32_t *orow = p.out + row * words;
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    const int g = wt + j * p.team_warps;
    if (g >= ngroups) continue;
    const int col0 = g * 256 + lane * 8;
    int code[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float sc = valid ? __fmul_rn(v[j][i], inv) : 0.0f;
      float c = minnum(maxnum(rintf(sc), -qmax), qmax);
      code[i] = (int)c;
    }
    if (bits == 4) {
      uint32_t w = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) w |= ((uint32_t)code[i] & 0xFu) << (4 * i);
      orow[col0 >> 3] = w;
      if (p.op8) {
        // word q = col0/8 is word (q & 3) of 32-code group q >> 2
        uint8_t *grp = p.op8 + row * p.op_ld + (int64_t)(col0 >> 5) * 32;
        const int i4 = (col0 >> 3) & 3;
        *reinterpret_cast<uint32_t *>(grp + 4 * i4) = nib_lo16(w);
        *reinterpret_cast<uint32_t *>(grp + 16 + 4 * i4) = nib_hi16(w);
      }
    } else {
      uint32_t w0 = 0, w1 = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        w0 |= ((uint32_t)code[i] & 0xFFu) << (8 * i);
        w1 |= ((uint32_t)code[i + 4] & 0xFFu) << (8 * i);
      }
      *reinterpret_cast<uint2 *>(orow + (col0 >> 2)) = make_uint2(w0, w1);
    }
  }
  // Stride padding words are zeroed; the scale follows all code rows.
  const int tid_in_team = wt * 32 + lane;
  for (int w = p.width / P + tid_in_team; w < words; w += p.team_warps * 32) orow[w] = 0u;
  if (tid_in_team == 0) reinterpret_cast<float *>(p.out + p.rows * words)[row] = scale;
}

int launch_prepare(const PrepareArgs &a0, cudaStream_t stream) {
  PrepareArgs a = a0;
  const int ngroups = a.width >> 8;
  const bool norm = a.mode == MODE_NORM || a.mode == MODE_NORM_STORE;
  int tw, rpb;
  if (norm) {
    tw = 8;
    rpb = 1;
  } else if (ngroups >= 16) {
    tw = 16;
    rpb = 1;
  } else if (ngroups >= 8) {
    tw = 8;
    rpb = 1;
  } else {
    tw = ngroups;
    rpb = 8 / ngroups;
  }
  const int ch = (ngroups + tw - 1) / tw;
  a.team_warps = tw;
  a.rows_per_block = rpb;
  const int threads = tw * 32 * rpb;
  const int64_t blocks = (a.rows + rpb - 1) / rpb;
  const size_t smem = sizeof(float) * (size_t)(tw * rpb + 8);
  if (blocks == 0) return 0;
  if (blocks > 0x7fffffffLL) return CLEFQ_ERR_SHAPE;
  switch (ch) {
#define CQ_CASE(N) \
  case N: prepare_kernel<N><<<(unsigned)blocks, threads, smem, stream>>>(a); break;
    CQ_CASE(1) CQ_CASE(2) CQ_CASE(3) CQ_CASE(4) CQ_CASE(5) CQ_CASE(6) CQ_CASE(7) CQ_CASE(8)
#undef CQ_CASE
    default:
      return CLEFQ_ERR_SHAPE;
  }
  return cudaGetLastError() == cudaSuccess ? 0 : CLEFQ_ERR_CUDA;
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
      float a = bf16_to_f32(gh[k]);
      float act = __fdiv_rn(a, __fadd_rn(1.0f, exp_cw(-a)));
      oh[k] = f32_to_bf16(__fmul_rn(bf16r(act), bf16_to_f32(uh[k])));
    }
    reinterpret_cast<uint4 *>(out)[i] = o;
  }
}
__global__ void swiglu_tail_kernel(const uint16_t *g, const uint16_t *u, uint16_t *out, int64_t start, int64_t n) {
  int64_t i = start + blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i < n) {
    float a = bf16_to_f32(g[i]);
    float act = __fdiv_rn(a, __fadd_rn(1.0f, exp_cw(-a)));
    out[i] = f32_to_bf16(__fmul_rn(bf16r(act), bf16_to_f32(u[i])));
  }
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
  return cudaGetLastError() == cudaSuccess ? 0 : CLEFQ_ERR_CUDA;
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
  return cudaGetLastError() == cudaSuccess ? 0 : CLEFQ_ERR_CUDA;
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
  return cudaGetLastError() == cudaSuccess ? 0 : CLEFQ_ERR_CUDA;
}

}  // namespace cq
