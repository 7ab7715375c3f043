// clefq: scalar numerics shared by the device kernels and the host-side table generator.
//
// Every rounding that is part of the reference contract is spelled out: BF16 round to
// nearest even, and exp() as Cody & Waite (1980) two-constant argument reduction with a
// degree-7 Taylor polynomial.  On the device the multiplies and fused multiply-adds use
// the _rn intrinsics so nvcc cannot contract or reassociate them; on the host the same
// steps use fmaf() and plain IEEE binary32 operations (the generator is compiled with
// -ffp-contract=off), so a table computed on the host holds exactly the values the device
// expression produces.
#pragma once
#include <stdint.h>
#include <string.h>
#include <math.h>

#if defined(__CUDACC__)
#define CQ_HD __host__ __device__ __forceinline__
#else
#define CQ_HD static inline
#endif

namespace cq {

CQ_HD float u2f(uint32_t u) {
#if defined(__CUDA_ARCH__)
  return __uint_as_float(u);
#else
  float f;
  memcpy(&f, &u, 4);
  return f;
#endif
}
CQ_HD uint32_t f2u(float f) {
#if defined(__CUDA_ARCH__)
  return __float_as_uint(f);
#else
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
#endif
}
CQ_HD float fma_rn(float a, float b, float c) {
#if defined(__CUDA_ARCH__)
  return __fmaf_rn(a, b, c);
#else
  return fmaf(a, b, c);
#endif
}
CQ_HD float mul_rn(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fmul_rn(a, b);
#else
  return a * b;
#endif
}
CQ_HD float add_rn(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fadd_rn(a, b);
#else
  return a + b;
#endif
}
CQ_HD float div_rn(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fdiv_rn(a, b);
#else
  return a / b;
#endif
}

// BF16 <-> F32, round to nearest even (the reference's `half` crate and Loom fptrunc);
// NaN keeps its sign and top payload bits with the quiet bit set.
CQ_HD float bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }
CQ_HD uint16_t f32_to_bf16(float f) {
  uint32_t u = f2u(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
CQ_HD float bf16r(float f) { return bf16_to_f32(f32_to_bf16(f)); }

// exp(x): x = n ln2 + r with ln2 split into a 13-bit head and its remainder (Cody & Waite),
// |r| <= ln2/2, e^r by its degree-7 Taylor polynomial in Horner form with fused
// multiply-adds, then exact scaling by 2^n split into two powers of two so that results
// near the subnormal range round once.  Error below 2 ulp over the normal range.
CQ_HD float pow2i(int n) { return u2f((uint32_t)(n + 127) << 23); }
CQ_HD float exp_cw(float x) {
  if (x != x) return x;
  if (x > 88.72283935546875f) return u2f(0x7f800000u);
  if (x < -103.972084045410156f) return 0.0f;
  const float log2e = 1.44269502162933349609375f;
  const float ln2_hi = 0.693145751953125f;
  const float ln2_lo = 1.428606765330187045e-06f;
  float n = rintf(mul_rn(x, log2e));
  float r = fma_rn(-n, ln2_hi, x);
  r = fma_rn(-n, ln2_lo, r);
  float p = 1.0f / 5040.0f;
  p = fma_rn(p, r, 1.0f / 720.0f);
  p = fma_rn(p, r, 1.0f / 120.0f);
  p = fma_rn(p, r, 1.0f / 24.0f);
  p = fma_rn(p, r, 1.0f / 6.0f);
  p = fma_rn(p, r, 0.5f);
  p = fma_rn(p, r, 1.0f);
  p = fma_rn(p, r, 1.0f);
  int ni = (int)n;
  int n1 = ni / 2;
  int n2 = ni - n1;
  return mul_rn(mul_rn(p, pow2i(n1)), pow2i(n2));
}

// SiLU of one BF16 input rounded to BF16: bf16(g / (1 + exp(-g))), the activation half of
// the reference's SwiGLU (kernels/swiglu.loom:41-50, prepare_integer_register.loom).
CQ_HD uint16_t silu_bf16(uint16_t g_bits) {
  const float g = bf16_to_f32(g_bits);
  return f32_to_bf16(div_rn(g, add_rn(1.0f, exp_cw(-g))));
}

}  // namespace cq
