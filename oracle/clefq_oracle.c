/*
 * clefq CPU oracle -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C (OpenMP) restatement of clef-hrx's INT4/INT8 quantized matmul path and its
 * Omni MoE operators.  It is the parity checker for the CUDA library and the timed CPU
 * baseline ("port"); nothing in the product links or calls it.  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU legs may load it.
 *
 * Every function cites the reference file:line it follows (paths relative to the
 * clef-hrx project root).  Floating point: IEEE binary32, round-to-nearest-even, no
 * contraction (built with -ffp-contract=off), no fast-math.
 *
 * Parity anchor: the reference ships no golden vectors for this path and cannot run in
 * this image (Rust + the un-vendored hrx-rs 0.11.0 crate + a gfx1151 GPU).  The oracle is
 * pinned against the reference's own in-test CPU oracles and known-answer tests, restated
 * independently in numpy by tests/golden/make_golden.py (src/quantized.rs:790-824 rotation,
 * :1000-1015 quantizer, :1369-1407 retile formula, :1048-1064 integer-dot epilogue,
 * benches/kernels/omni_route_serial.loom serial top-k).  `exp` follows the reference's
 * `expf<afn>` only to within its error class: its exact bits are unpinned (the reference's
 * approximate exp is defined by hrx-rs, absent here); this oracle and the CUDA kernels share
 * one published algorithm (Cody-Waite reduction + degree-7 Taylor polynomial) so that they
 * agree bit for bit with each other.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#if defined(__x86_64__)
#include <immintrin.h>
#endif

#define CQO_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------------------------ */
/* BF16 <-> F32, round to nearest even (the `half` 2.7.1 crate's from_f32 / to_f32:     */
/* Cargo.lock:1186-1187).  NaN keeps its sign and payload top bits, quiet bit forced.   */
/* ------------------------------------------------------------------------------------ */
static inline float f32_of_bits(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t bits_of_f32(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bf16_to_f32(uint16_t h) { return f32_of_bits((uint32_t)h << 16); }
static inline uint16_t f32_to_bf16(float f) {
  uint32_t u = bits_of_f32(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
static inline float bf16r(float f) { return bf16_to_f32(f32_to_bf16(f)); }

/* maxnum / minnum: IEEE-754 2008 maxNum/minNum (return the non-NaN operand). */
static inline float maxnum(float a, float b) { return fmaxf(a, b); }
static inline float minnum(float a, float b) { return fminf(a, b); }

/* ------------------------------------------------------------------------------------ */
/* exp(x): Cody & Waite (1980) two-constant argument reduction x = n ln2 + r,           */
/* |r| <= ln2/2, then the degree-7 Taylor polynomial of e^r in Horner form with fused   */
/* multiply-adds, then an exact scaling by 2^n split in two powers of two.              */
/* Error below 2 ulp over the normal range; the CUDA kernels evaluate the same steps.    */
/* ------------------------------------------------------------------------------------ */
static inline float pow2i(int n) { return f32_of_bits((uint32_t)(n + 127) << 23); }
static float cq_exp(float x) {
  if (x != x) return x;
  if (x > 88.72283935546875f) return INFINITY;
  if (x < -103.972084045410156f) return 0.0f;
  const float log2e = 1.44269502162933349609375f;
  const float ln2_hi = 0.693145751953125f;          /* 13 significant bits */
  const float ln2_lo = 1.428606765330187045e-06f;   /* ln2 - ln2_hi */
  float n = rintf(x * log2e);
  float r = fmaf(-n, ln2_hi, x);
  r = fmaf(-n, ln2_lo, r);
  float p = 1.0f / 5040.0f;
  p = fmaf(p, r, 1.0f / 720.0f);
  p = fmaf(p, r, 1.0f / 120.0f);
  p = fmaf(p, r, 1.0f / 24.0f);
  p = fmaf(p, r, 1.0f / 6.0f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  int ni = (int)n;
  int n1 = ni / 2;
  int n2 = ni - n1;
  return (p * pow2i(n1)) * pow2i(n2);
}

/* ------------------------------------------------------------------------------------ */
/* prepare (A1)                                                                          */
/* kernels/prepare_integer.loom:55-291 (two-pass), prepare_integer_register.loom:58-311  */
/* (fused variants), src/quantized.rs:626-686 (output storage: codes then f32 scales).   */
/* ------------------------------------------------------------------------------------ */
enum { CQO_PLAIN = 0, CQO_SWIGLU = 1, CQO_ATTN_GATE = 2, CQO_NORM = 3, CQO_NORM_STORE = 4 };

/* Radix-4 Hadamard over one 256-group, strides 1, 4, 16, 64 in that order
 * (prepare_integer.loom:86-244; src/quantized.rs:801-824). */
static void hadamard256(float *g) {
  for (int s = 1; s <= 64; s *= 4) {
    for (int base = 0; base < 256; base += 4 * s) {
      for (int i = 0; i < s; ++i) {
        int j = base + i;
        float a = g[j], b = g[j + s], c = g[j + 2 * s], d = g[j + 3 * s];
        float s01 = a + b, s23 = c + d, d01 = a - b, d23 = c - d;
        g[j] = s01 + d23;
        g[j + s] = s01 - d23;
        g[j + 2 * s] = d01 + s23;
        g[j + 3 * s] = s23 - d01;
      }
    }
  }
}

/* The RMSNorm sum of squares in the exact order the CUDA kernel reduces it:
 * 256 strided partial sums (thread t takes columns t, t+256, ... with fma), then a
 * xor-butterfly inside each 32-lane warp (offsets 16..1), then the 8 warp totals in
 * ascending warp order.  The reference's own order (prepare_integer_register.loom:58-74,
 * 128 lanes then a workgroup reduce) is a different parallel order: parity to it is a
 * tolerance, as in its own test (src/quantized.rs:1553-1774). */
static float norm_sum_squares(const uint16_t *x, int64_t width) {
  float part[256];
  for (int t = 0; t < 256; ++t) {
    float s = 0.0f;
    for (int64_t j = t; j < width; j += 256) {
      float v = bf16_to_f32(x[j]);
      s = fmaf(v, v, s);
    }
    part[t] = s;
  }
  float warp_total[8];
  for (int w = 0; w < 8; ++w) {
    float v[32];
    for (int l = 0; l < 32; ++l) v[l] = part[w * 32 + l];
    for (int off = 16; off >= 1; off >>= 1) {
      float nv[32];
      for (int l = 0; l < 32; ++l) nv[l] = v[l] + v[l ^ off];
      memcpy(v, nv, sizeof v);
    }
    warp_total[w] = v[0];
  }
  float total = warp_total[0];
  for (int w = 1; w < 8; ++w) total = total + warp_total[w];
  return total;
}

/* Pre-op value of column i (prepare_integer_register.loom:104-177). */
static inline float preop(int mode, const uint16_t *xr, const uint16_t *auxr, int64_t i, float norm_inv,
                          uint16_t *norm_row) {
  float v = bf16_to_f32(xr[i]);
  switch (mode) {
    case CQO_SWIGLU: {
      float u = bf16_to_f32(auxr[i]);
      float act = v / (1.0f + cq_exp(-v));
      return bf16r(bf16r(act) * u);
    }
    case CQO_ATTN_GATE: {
      int64_t head = i / 256, within = i % 256;
      float q = bf16_to_f32(auxr[head * 512 + 256 + within]);
      float sg = bf16r(1.0f / (1.0f + cq_exp(-q)));
      return bf16r(v * sg);
    }
    case CQO_NORM:
    case CQO_NORM_STORE: {
      float w = bf16_to_f32(auxr[i]) + 1.0f;
      float nn = (v - 0.0f) * norm_inv;
      uint16_t h = f32_to_bf16(fmaf(nn, w, 0.0f));
      if (norm_row) norm_row[i] = h;
      return bf16_to_f32(h);
    }
    default:
      return v;
  }
}

CQO_API int cqo_prepare(int mode, int bits, const uint16_t *x, int64_t x_ld, const uint16_t *aux, int64_t aux_ld,
                        int64_t rows, int64_t width, int64_t stride, uint32_t *out, uint16_t *norm_out,
                        int64_t norm_ld, int threads) {
  if (!(bits == 4 || bits == 8) || width % 256 || width < 256 || stride < width || rows < 0) return -1;
  const int P = 32 / bits;
  if (stride % P) return -1;
  const int64_t words = stride / P;
  const float qmax = bits == 8 ? 127.0f : 7.0f;
  const uint32_t mask = bits == 8 ? 0xffu : 0xfu;
  float *scales = (float *)(out + rows * words);
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
  for (int64_t row = 0; row < rows; ++row) {
    const uint16_t *xr = x + row * x_ld;
    const uint16_t *auxr = aux ? aux + (mode == CQO_NORM || mode == CQO_NORM_STORE ? 0 : row * aux_ld) : NULL;
    uint16_t *nrow = (mode == CQO_NORM_STORE && norm_out) ? norm_out + row * norm_ld : NULL;
    float norm_inv = 1.0f;
    if (mode == CQO_NORM || mode == CQO_NORM_STORE) {
      float ss = norm_sum_squares(xr, width);
      float var = ss / (float)width;
      norm_inv = 1.0f / sqrtf(var + 1e-6f);
    }
    float *h = (float *)malloc(sizeof(float) * (size_t)width);
    float m = 0.0f;
    for (int64_t i = 0; i < width; ++i) h[i] = preop(mode, xr, auxr, i, norm_inv, nrow);
    for (int64_t g = 0; g < width; g += 256) hadamard256(h + g);
    /* prepare_integer.loom:218-234: non-finite magnitudes count as +inf. */
    for (int64_t i = 0; i < width; ++i) {
      float a = fabsf(h[i]);
      m = maxnum(m, a < INFINITY ? a : INFINITY);
    }
    /* prepare_integer.loom:278-283 */
    float scale = maxnum(m * 0.0625f, 1e-30f) / qmax;
    int valid = scale < INFINITY;
    float inv = 0.0625f / scale;
    uint32_t *wr = out + row * words;
    for (int64_t w = 0; w < words; ++w) {
      uint32_t acc = 0;
      if (w * P < width) {
        for (int p = 0; p < P; ++p) {
          /* prepare_integer.loom:255-266 */
          float scaled = valid ? h[w * P + p] * inv : 0.0f;
          float c = minnum(maxnum(rintf(scaled), -qmax), qmax);
          int code = (int)c;
          acc |= ((uint32_t)code & mask) << (p * bits);
        }
      }
      wr[w] = acc; /* stride padding words: zero */
    }
    scales[row] = scale;
    free(h);
  }
  return 0;
}

/* ------------------------------------------------------------------------------------ */
/* retile (A5): kernels/retile_codes.loom:1-5,37-56; src/quantized.rs:542-572            */
/* word (n, q) -> ((n/128)*blocks_k + q/32)*4096 + (n%128)*32 + q%32                      */
/* ------------------------------------------------------------------------------------ */
CQO_API int cqo_retile(const uint32_t *codes, int64_t rows, int64_t in_words, int64_t words, uint32_t *out) {
  if (rows % 128 || words % 32 || in_words < words) return -1;
  int64_t blocks_k = words / 32;
  for (int64_t n = 0; n < rows; ++n)
    for (int64_t q = 0; q < words; ++q)
      out[((n / 128) * blocks_k + q / 32) * 4096 + (n % 128) * 32 + q % 32] = codes[n * in_words + q];
  return 0;
}

/* Sign-extended code k of a packed row (bits 4 or 8). */
static inline int code_at(const uint32_t *row, int64_t k, int bits) {
  int P = 32 / bits;
  uint32_t w = row[k / P] >> ((k % P) * bits);
  if (bits == 4) return (int)((int32_t)(w << 28) >> 28);
  return (int)((int32_t)(w << 24) >> 24);
}

/* Logical weight row n of a tiled code matrix, unpacked to int8. */
static void unpack_tiled_row(const uint32_t *w_tiled, int64_t n, int64_t k, int bits, int8_t *dst) {
  int P = 32 / bits;
  int64_t words = k / P, blocks_k = words / 32;
  for (int64_t q = 0; q < words; ++q) {
    uint32_t w = w_tiled[((n / 128) * blocks_k + q / 32) * 4096 + (n % 128) * 32 + q % 32];
    for (int p = 0; p < P; ++p) {
      uint32_t v = w >> (p * bits);
      dst[q * P + p] = bits == 4 ? (int8_t)((int32_t)(v << 28) >> 28) : (int8_t)((int32_t)(v << 24) >> 24);
    }
  }
}
static void unpack_row(const uint32_t *row, int64_t k, int bits, int8_t *dst) {
  for (int64_t i = 0; i < k; ++i) dst[i] = (int8_t)code_at(row, i, bits);
}

/* int8 dot product; AVX-512 VNNI when the host has it (u8 x s8 with a +128 offset on the
 * first operand, corrected by 128 * sum(b)), else scalar.  Exact int32 either way. */
#if defined(__x86_64__)
__attribute__((target("avx512f,avx512bw,avx512vnni"))) static int32_t dot_vnni(const uint8_t *a_off, const int8_t *b,
                                                                               int64_t k, int32_t b_sum) {
  __m512i acc = _mm512_setzero_si512();
  int64_t i = 0;
  for (; i + 64 <= k; i += 64) {
    __m512i va = _mm512_loadu_si512((const void *)(a_off + i));
    __m512i vb = _mm512_loadu_si512((const void *)(b + i));
    acc = _mm512_dpbusd_epi32(acc, va, vb);
  }
  int32_t s = _mm512_reduce_add_epi32(acc);
  for (; i < k; ++i) s += (int32_t)a_off[i] * (int32_t)b[i];
  return s - 128 * b_sum;
}
#endif
static int have_vnni(void) {
#if defined(__x86_64__)
  static int cached = -1;
  if (cached < 0) cached = __builtin_cpu_supports("avx512vnni") && __builtin_cpu_supports("avx512bw");
  return cached;
#else
  return 0;
#endif
}
static int32_t dot_i8(const int8_t *a, const uint8_t *a_off, const int8_t *b, int64_t k, int32_t b_sum) {
#if defined(__x86_64__)
  if (have_vnni()) return dot_vnni(a_off, b, k, b_sum);
#endif
  (void)a_off; (void)b_sum;
  int32_t s = 0;
  for (int64_t i = 0; i < k; ++i) s += (int32_t)a[i] * (int32_t)b[i];
  return s;
}

/* ------------------------------------------------------------------------------------ */
/* Dense GEMM (A3): kernels/gemm_integer.loom:394-433                                    */
/*   y = (f32(acc) * ws[n]) * as[m] + 0;  BF16 with finite saturation to +-3.3895e38;    */
/*   optional residual bf16(f32(res) + f32(bf16(y))); optional F32 output y.             */
/* ------------------------------------------------------------------------------------ */
static const float BF16_MAX_F = 3.3895313892515355e38f;
static inline uint16_t bf16_saturated(float y) {
  float sat = maxnum(minnum(y, BF16_MAX_F), -BF16_MAX_F);
  return f32_to_bf16(fabsf(y) < INFINITY ? sat : y);
}

CQO_API int cqo_gemm(int bits, const uint32_t *a, int64_t a_ld_words, const float *a_scales, int64_t m,
                     const uint32_t *w_tiled, const float *w_scales, int64_t n, int64_t k, const uint16_t *residual,
                     int out_f32, void *out, int32_t *acc_out, int threads) {
  if (!(bits == 4 || bits == 8) || n % 128 || k % (bits == 4 ? 256 : 128)) return -1;
  int8_t *wu = (int8_t *)malloc((size_t)(n * k));
  int32_t *wsum = (int32_t *)malloc(sizeof(int32_t) * (size_t)n);
  int8_t *au = (int8_t *)malloc((size_t)(m * k + 1));
  uint8_t *ao = (uint8_t *)malloc((size_t)(m * k + 1));
  if (!wu || !wsum || !au || !ao) { free(wu); free(wsum); free(au); free(ao); return -2; }
  int nt = threads > 0 ? threads : 1;
#pragma omp parallel for schedule(static) num_threads(nt)
  for (int64_t j = 0; j < n; ++j) {
    unpack_tiled_row(w_tiled, j, k, bits, wu + j * k);
    int32_t s = 0;
    for (int64_t i = 0; i < k; ++i) s += wu[j * k + i];
    wsum[j] = s;
  }
#pragma omp parallel for schedule(static) num_threads(nt)
  for (int64_t r = 0; r < m; ++r) {
    unpack_row(a + r * a_ld_words, k, bits, au + r * k);
    for (int64_t i = 0; i < k; ++i) ao[r * k + i] = (uint8_t)(au[r * k + i] + 128);
  }
#pragma omp parallel for collapse(2) schedule(static) num_threads(nt)
  for (int64_t r0 = 0; r0 < m; r0 += 16) {
    for (int64_t c0 = 0; c0 < n; c0 += 64) {
      for (int64_t r = r0; r < r0 + 16 && r < m; ++r) {
        for (int64_t c = c0; c < c0 + 64 && c < n; ++c) {
          int32_t acc = dot_i8(au + r * k, ao + r * k, wu + c * k, k, wsum[c]);
          if (acc_out) acc_out[r * n + c] = acc;
          float y = ((float)acc * w_scales[c]) * a_scales[r] + 0.0f;
          if (out_f32) {
            ((float *)out)[r * n + c] = y;
          } else {
            uint16_t h = bf16_saturated(y);
            if (residual) h = f32_to_bf16(bf16_to_f32(residual[r * n + c]) + bf16_to_f32(h));
            ((uint16_t *)out)[r * n + c] = h;
          }
        }
      }
    }
  }
  free(wu); free(wsum); free(au); free(ao);
  return 0;
}

/* ------------------------------------------------------------------------------------ */
/* SwiGLU (A8): kernels/swiglu.loom:41-50, src/ops.rs:9-29                               */
/* ------------------------------------------------------------------------------------ */
CQO_API void cqo_swiglu(const uint16_t *g, const uint16_t *u, int64_t count, uint16_t *out, int threads) {
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
  for (int64_t i = 0; i < count; ++i) {
    float a = bf16_to_f32(g[i]);
    float act = a / (1.0f + cq_exp(-a));
    out[i] = f32_to_bf16(bf16r(act) * bf16_to_f32(u[i]));
  }
}

/* ------------------------------------------------------------------------------------ */
/* Router (A5): benches/kernels/omni_route_serial.loom (the serial spec the parallel     */
/* kernels/omni_route.loom:84-147 must equal): top-k by repeated strict '>' scans in     */
/* ascending expert id from (-3.402823466e38, id 0); then p_j = exp(l_j - l_0) summed in */
/* rank order and p_j / sum rounded to BF16.  routes[t] = ids (as f32) || probabilities. */
/* ------------------------------------------------------------------------------------ */
CQO_API int cqo_route(const void *logits, int logits_f32, int64_t tokens, int experts, int topk, float *routes,
                      int threads) {
  if (topk <= 0 || topk > experts || experts > 128) return -1;
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
  for (int64_t t = 0; t < tokens; ++t) {
    float *o = routes + t * 2 * topk;
    for (int r = 0; r < topk; ++r) {
      float bv = -3.402823466e38f;
      int bi = 0;
      for (int e = 0; e < experts; ++e) {
        int used = 0;
        for (int j = 0; j < r; ++j) if ((int)o[j] == e) used = 1;
        float v = logits_f32 ? ((const float *)logits)[t * experts + e]
                             : bf16_to_f32(((const uint16_t *)logits)[t * experts + e]);
        if (!used && v > bv) { bv = v; bi = e; }
      }
      o[r] = (float)bi;
      o[topk + r] = bv;
    }
    float mx = o[topk];
    float sum = 0.0f;
    for (int j = 0; j < topk; ++j) {
      float p = cq_exp(o[topk + j] - mx);
      o[topk + j] = p;
      sum = sum + p;
    }
    for (int j = 0; j < topk; ++j) o[topk + j] = bf16r(o[topk + j] / sum);
  }
  return 0;
}

/* ------------------------------------------------------------------------------------ */
/* Grouping (A6): kernels/omni_group_routes_ordered.loom:50-97                           */
/*   groups[e] = [count, route ids t*topk+rank ascending t]  (stride tokens+1)           */
/*   order[t][j] = rank whose expert id is the j-th smallest of token t's ids            */
/* ------------------------------------------------------------------------------------ */
CQO_API int cqo_group(const float *routes, int64_t tokens, int topk, int experts, float *groups, float *order) {
  int64_t stride = tokens + 1;
  for (int e = 0; e < experts; ++e) {
    int64_t count = 0;
    for (int64_t t = 0; t < tokens; ++t) {
      const float *rt = routes + t * 2 * topk;
      int rank = topk, less = 0;
      for (int r = 0; r < topk; ++r) {
        if ((int)rt[r] == e) rank = r;
        if (rt[r] < (float)e) ++less;
      }
      if (rank < topk) {
        groups[e * stride + 1 + count] = (float)(t * topk + rank);
        if (order) order[t * topk + less] = (float)rank;
        ++count;
      }
    }
    groups[e * stride] = (float)count;
  }
  return 0;
}

/* Tasks (A6): kernels/omni_expert_tasks.loom:30-61 -- [total, (expert, row0) per 16-row
 * tile, experts ascending]; unused tail entries are left untouched. */
CQO_API int cqo_tasks(const float *groups, int64_t tokens, int experts, float *tasks) {
  int64_t stride = tokens + 1, total = 0;
  for (int e = 0; e < experts; ++e) {
    int64_t count = (int64_t)groups[e * stride];
    int64_t tiles = (count + 15) / 16;
    for (int64_t i = 0; i < tiles; ++i) {
      tasks[1 + 2 * (total + i)] = (float)e;
      tasks[2 + 2 * (total + i)] = (float)(16 * i);
    }
    total += tiles;
  }
  tasks[0] = (float)total;
  return 0;
}

/* ------------------------------------------------------------------------------------ */
/* Grouped expert GEMM (A4): kernels/omni_expert_i4.loom:111-125,442-462                 */
/*   for expert e, route r in groups[e]: xr = input_routed ? r : r / topk                */
/*   out[r][c] = bf16(f32(acc) * (as[xr] * ws[e*n + c]))      (no saturation, no +0)     */
/* ------------------------------------------------------------------------------------ */
CQO_API int cqo_expert(int bits, const uint32_t *a, int64_t a_ld_words, const float *a_scales, const uint32_t *w_tiled,
                       const float *w_scales, const float *groups, int64_t tokens, int topk, int experts, int64_t k,
                       int64_t n, int input_routed, uint16_t *out, int threads) {
  if (bits != 4 || n % 128 || k % 256) return -1;
  int64_t stride = tokens + 1;
  int nt = threads > 0 ? threads : 1;
  for (int e = 0; e < experts; ++e) {
    int64_t count = (int64_t)groups[e * stride];
    if (!count) continue;
    int8_t *wu = (int8_t *)malloc((size_t)(n * k));
    int32_t *wsum = (int32_t *)malloc(sizeof(int32_t) * (size_t)n);
#pragma omp parallel for schedule(static) num_threads(nt)
    for (int64_t c = 0; c < n; ++c) {
      unpack_tiled_row(w_tiled, (int64_t)e * n + c, k, bits, wu + c * k);
      int32_t s = 0;
      for (int64_t i = 0; i < k; ++i) s += wu[c * k + i];
      wsum[c] = s;
    }
#pragma omp parallel num_threads(nt)
    {
      int8_t *au = (int8_t *)malloc((size_t)k);
      uint8_t *ao = (uint8_t *)malloc((size_t)k);
#pragma omp for schedule(static)
      for (int64_t i = 0; i < count; ++i) {
        int64_t r = (int64_t)groups[e * stride + 1 + i];
        int64_t xr = input_routed ? r : r / topk;
        unpack_row(a + xr * a_ld_words, k, bits, au);
        for (int64_t q = 0; q < k; ++q) ao[q] = (uint8_t)(au[q] + 128);
        for (int64_t c = 0; c < n; ++c) {
          int32_t acc = dot_i8(au, ao, wu + c * k, k, wsum[c]);
          float sc = a_scales[xr] * w_scales[(int64_t)e * n + c];
          out[r * n + c] = f32_to_bf16((float)acc * sc);
        }
      }
      free(au); free(ao);
    }
    free(wu); free(wsum);
  }
  return 0;
}

/* ------------------------------------------------------------------------------------ */
/* Combine (A7): kernels/omni_combine_ordered.loom:51-79 (order given) and               */
/* kernels/omni_combine.loom:40-72 (ascending expert order found per token).             */
/*   s = 0; for j: r = order[t][j]; s = bf16(s + bf16(f32(v[t*topk+r][c]) * p[t][r]))   */
/* ------------------------------------------------------------------------------------ */
CQO_API int cqo_combine(const uint16_t *values, const float *routes, const float *order, int64_t tokens, int topk,
                        int64_t width, uint16_t *out, int threads) {
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
  for (int64_t t = 0; t < tokens; ++t) {
    const float *rt = routes + t * 2 * topk;
    int ranks[64];
    if (order) {
      for (int j = 0; j < topk; ++j) ranks[j] = (int)order[t * topk + j];
    } else {
      float prev = -1.0f;
      for (int j = 0; j < topk; ++j) {
        float best = 1000000.0f;
        int at = 0;
        for (int r = 0; r < topk; ++r) {
          float e = rt[r];
          if (e > prev && e < best) { best = e; at = r; }
        }
        ranks[j] = at;
        prev = best;
      }
    }
    for (int64_t c = 0; c < width; ++c) {
      float s = 0.0f;
      for (int j = 0; j < topk; ++j) {
        int r = ranks[j];
        float v = bf16_to_f32(values[(t * topk + r) * width + c]);
        float pf = bf16r(v * rt[topk + r]);
        s = bf16r(s + pf);
      }
      out[t * width + c] = f32_to_bf16(s);
    }
  }
  return 0;
}

/* Exposed for tests of the shared exp algorithm. */
CQO_API void cqo_exp(const float *x, int64_t count, float *out) {
  for (int64_t i = 0; i < count; ++i) out[i] = cq_exp(x[i]);
}
