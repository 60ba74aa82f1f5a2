/*
 * svl_oracle.c — CPU restatement of semantic-voice-local's streaming language-model step
 * (Kyutai STT LanguageModel and Pocket-TTS FlowLm over the shared StreamingTransformer).
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA path and the timed CPU
 * baseline. Only tests/, __graft_entry__.smoke() and bench.py's CPU legs load it; the
 * product library never links or calls it.
 *
 * Parity status: pinned to the reference's own unit-test bounds through torch-f64 fixtures
 * (tests/golden/); the candle-internal pieces (Q8_0 QMatMul, rope_i, rms/layer norm order,
 * argmax ties) are restated from their published algorithms and are "parity unpinned"
 * against candle itself, which cannot be built here (Rust toolchain and candle 0.11.1 absent).
 *
 * Reference paths are relative to crates/semantic-voice-local/src/ of the reference repo.
 * Build: see oracle/Makefile (-O3 -march=x86-64-v3 -ffp-contract=off -fopenmp). Rust never
 * contracts a*b+c into an FMA, so neither may this file except where the reference calls
 * mul_add (its FMA path, taken on every AVX2+FMA CPU: nn/kernels/mod.rs:12-35).
 */
#include "svl_oracle.h"

#include <math.h>
#include <omp.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#if defined(__AVX2__) && defined(__FMA__)
#include <immintrin.h>
#define ORC_AVX2 1
#endif

static __thread char g_err[512];
static void set_err(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
}
const char* orc_last_error(void) { return g_err; }
void orc_set_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
}

/* Test-only knob: 1 sums the RMS-norm squares in reverse order. Comparing the oracle with
 * itself under the two orders measures how far a 1-ulp reduction-order difference carries
 * through the discontinuous activation rounding of bf16 / quantised models. */
static int g_variant = 0;
void orc_set_reduction_variant(int v) { g_variant = v; }

/* ------------------------------------------------------------------ number formats */

/* IEEE binary16 <-> binary32, round to nearest even (the `half` crate's f16::from_f32). */
uint16_t orc_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t exp = (x >> 23) & 0xffu;
  uint32_t man = x & 0x7fffffu;
  if (exp == 0xff) return (uint16_t)(sign | 0x7c00u | (man ? 0x200u | (man >> 13) : 0));
  int32_t e = (int32_t)exp - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7c00u);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    man |= 0x800000u;
    uint32_t shift = (uint32_t)(14 - e);
    uint32_t half = man >> shift;
    uint32_t rem = man & ((1u << shift) - 1);
    uint32_t mid = 1u << (shift - 1);
    if (rem > mid || (rem == mid && (half & 1))) half++;
    return (uint16_t)(sign | half);
  }
  uint32_t h = sign | ((uint32_t)e << 10) | (man >> 13);
  uint32_t rem = man & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1))) h++;
  return (uint16_t)h;
}

float orc_f16_to_f32(uint16_t h) {
  uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  uint32_t x;
  if (exp == 0) {
    if (man == 0) {
      x = sign;
    } else {
      int e = -1;
      do { man <<= 1; e++; } while (!(man & 0x400u));
      x = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ffu) << 13);
    }
  } else if (exp == 31) {
    x = sign | 0x7f800000u | (man << 13);
  } else {
    x = sign | ((exp - 15 + 127) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &x, 4);
  return f;
}

/* f32 -> bf16 -> f32, round to nearest even (the `half` crate's bf16::from_f32). */
float orc_round_bf16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  if ((x & 0x7fffffffu) > 0x7f800000u) {
    x |= 0x00400000u;
  } else {
    x += 0x7fffu + ((x >> 16) & 1u);
  }
  x &= 0xffff0000u;
  memcpy(&f, &x, 4);
  return f;
}

/* ------------------------------------------------------------------ kernel helpers */

/* kernels::dot (nn/kernels/mod.rs:68-91): 16 independent FMA lanes, a non-fused tail sum,
 * then a pairwise lane reduction, and acc[0] + tail last. */
static float dot_scalar(const float* a, const float* b, int n) {
  float acc[16] = {0};
  int chunks = n / 16;
  for (int c = 0; c < chunks; c++)
    for (int i = 0; i < 16; i++) acc[i] = fmaf(a[c * 16 + i], b[c * 16 + i], acc[i]);
  float sum = 0.0f;
  for (int i = chunks * 16; i < n; i++) sum += a[i] * b[i];
  for (int w = 8; w >= 1; w /= 2)
    for (int i = 0; i < w; i++) acc[i] += acc[i + w];
  return acc[0] + sum;
}

float orc_dot(const float* a, const float* b, int n) {
#ifdef ORC_AVX2
  /* Same lanes and reduction tree as dot_scalar, in two 8-wide registers. */
  __m256 lo = _mm256_setzero_ps(), hi = _mm256_setzero_ps();
  int chunks = n / 16;
  for (int c = 0; c < chunks; c++) {
    lo = _mm256_fmadd_ps(_mm256_loadu_ps(a + c * 16), _mm256_loadu_ps(b + c * 16), lo);
    hi = _mm256_fmadd_ps(_mm256_loadu_ps(a + c * 16 + 8), _mm256_loadu_ps(b + c * 16 + 8), hi);
  }
  float sum = 0.0f;
  for (int i = chunks * 16; i < n; i++) sum += a[i] * b[i];
  __m256 s8 = _mm256_add_ps(lo, hi);                                   /* i += i+8 */
  __m128 s4 = _mm_add_ps(_mm256_castps256_ps128(s8), _mm256_extractf128_ps(s8, 1)); /* i+4 */
  __m128 s2 = _mm_add_ps(s4, _mm_movehl_ps(s4, s4));                    /* i += i+2 */
  __m128 s1 = _mm_add_ss(s2, _mm_shuffle_ps(s2, s2, 1));                /* i += i+1 */
  return _mm_cvtss_f32(s1) + sum;
#else
  return dot_scalar(a, b, n);
#endif
}

/* Exposed so the CPU tests can check the vector path against the scalar statement. */
float orc_dot_scalar(const float* a, const float* b, int n) { return dot_scalar(a, b, n); }

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* exp_parts / exp (nn/kernels/mod.rs:96-131): Cody-Waite reduction x = k ln2 + r with a
 * two-part ln2, expm1(r) by its Taylor series to degree 8, 2^k from the exponent bits. */
static inline void exp_parts(float x, float* two_k, float* expm1_r) {
  const float LN2_HI = 0.69314575f;
  const float LN2_LO = 1.4286068e-6f;
  const float ROUND = 12582912.0f; /* 1.5 * 2^23 */
  const float LOG2E = 1.44269504088896340736f;
  float shifted = fmaf(x, LOG2E, ROUND);
  float k = shifted - ROUND;
  int32_t k_int = (int32_t)(f2u(shifted) - f2u(ROUND));
  float r = fmaf(-k, LN2_LO, fmaf(-k, LN2_HI, x));
  static const float coef[7] = {1.0f / 5040.0f, 1.0f / 720.0f, 1.0f / 120.0f, 1.0f / 24.0f,
                                1.0f / 6.0f, 0.5f, 1.0f};
  float p = 1.0f / 40320.0f;
  for (int i = 0; i < 7; i++) p = fmaf(p, r, coef[i]);
  *two_k = u2f((uint32_t)(k_int + 127) << 23);
  *expm1_r = p * r;
}

float orc_exp(float x) {
  float c = x != x ? x : (x < -87.0f ? -87.0f : (x > 88.0f ? 88.0f : x));
  float two_k, e;
  exp_parts(c, &two_k, &e);
  float y = fmaf(two_k, e, two_k);
  if (x > 88.72f) y = INFINITY;
  return x < -87.0f ? 0.0f : y;
}

/* Activation::Elu (nn/kernels/activation.rs:60-67): x above 0, else 2^k expm1(r) + (2^k - 1)
 * of x clamped to [-20, 0]. */
float orc_elu(float x) {
  if (x != x) return x;
  if (x > 0.0f) return x;
  float c = x < -20.0f ? -20.0f : x;
  float two_k, e;
  exp_parts(c, &two_k, &e);
  return fmaf(two_k, e, two_k - 1.0f);
}

/* Activation::Silu / GeluTanh (nn/kernels/activation.rs:71-83). */
float orc_silu(float x) { return x / (1.0f + orc_exp(-x)); }
float orc_gelu_tanh(float x) {
  const float SQRT_2_OVER_PI = 0.7978846f;
  float y = SQRT_2_OVER_PI * fmaf(0.044715f * x, x * x, x);
  return x / (1.0f + orc_exp(-2.0f * y));
}
/* candle's gelu_erf: evaluated in f64, rounded to f32 (transformer.rs:446-447). */
static float gelu_erf(float x) {
  double v = x;
  return (float)((v * (1.0 + erf(v / 1.4142135623730951))) / 2.0);
}

/* ------------------------------------------------------------------ dense matvec */

/* kernels::matvec (nn/kernels/matvec.rs:29-58): one row x [k] times w [n][k]^T, rows in
 * blocks of clamp(n / (4 threads), 8, 256) spread over the threads, bias added after. */
void orc_matvec(const float* x, const float* w, const float* bias, int n, int k, float* out) {
  int threads = omp_get_max_threads();
  int rows = n / (4 * threads);
  rows = rows < 8 ? 8 : (rows > 256 ? 256 : rows);
  int blocks = (n + rows - 1) / rows;
#pragma omp parallel for schedule(dynamic, 1) if (blocks > 1 && (int64_t)n * k > 65536)
  for (int b = 0; b < blocks; b++) {
    int r0 = b * rows, r1 = r0 + rows > n ? n : r0 + rows;
    for (int r = r0; r < r1; r++) {
      out[r] = orc_dot(x, w + (int64_t)r * k, k);
      if (bias) out[r] += bias[r];
    }
  }
}

/* ------------------------------------------------------------------ Q8_0 / Q4_1 */

/* Block formats of ggml, as candle's k_quants uses them (nn/mod.rs:76-88 selects Q8_0):
 *   Q8_0: d = max|x| / 127 (stored f16), q = round(x / d) with id = 1/d in f32.
 *   Q4_1: d = (max - min) / 15, m = min, q = min(15, trunc((x - min) * id + 0.5)),
 *         qs[j] = q[j] | q[j + 16] << 4.
 *   Q8_1 (activation side of Q4_1): Q8_0 plus s = d * sum(q) stored f16. */
#define QK 32
typedef struct { uint16_t d; int8_t qs[QK]; } __attribute__((packed)) blk_q8_0;
typedef struct { uint16_t d, m; uint8_t qs[QK / 2]; } __attribute__((packed)) blk_q4_1;
typedef struct { uint16_t d, s; int8_t qs[QK]; } __attribute__((packed)) blk_q8_1;

static void quantize_q8_0_block(const float* x, blk_q8_0* y) {
  float amax = 0.0f;
  for (int j = 0; j < QK; j++) {
    float a = fabsf(x[j]);
    amax = amax > a ? amax : a;
  }
  float d = amax / 127.0f;
  float id = d != 0.0f ? 1.0f / d : 0.0f;
  y->d = orc_f32_to_f16(d);
  for (int j = 0; j < QK; j++) y->qs[j] = (int8_t)roundf(x[j] * id);
}

void orc_quantize_q8_0(const float* x, int64_t n, uint8_t* blocks) {
  blk_q8_0* y = (blk_q8_0*)blocks;
#pragma omp parallel for schedule(static) if (n > (1 << 20))
  for (int64_t b = 0; b < n / QK; b++) quantize_q8_0_block(x + b * QK, y + b);
}

static void quantize_q8_1_block(const float* x, blk_q8_1* y) {
  float amax = 0.0f;
  for (int j = 0; j < QK; j++) {
    float a = fabsf(x[j]);
    amax = amax > a ? amax : a;
  }
  float d = amax / 127.0f;
  float id = d != 0.0f ? 1.0f / d : 0.0f;
  y->d = orc_f32_to_f16(d);
  int32_t sum = 0;
  for (int j = 0; j < QK / 2; j++) {
    int8_t v0 = (int8_t)roundf(x[j] * id), v1 = (int8_t)roundf(x[j + QK / 2] * id);
    y->qs[j] = v0;
    y->qs[j + QK / 2] = v1;
    sum += v0 + v1;
  }
  y->s = orc_f32_to_f16((float)sum * d);
}

static void quantize_q4_1_block(const float* x, blk_q4_1* y) {
  float mn = INFINITY, mx = -INFINITY;
  for (int j = 0; j < QK; j++) {
    mn = x[j] < mn ? x[j] : mn;
    mx = x[j] > mx ? x[j] : mx;
  }
  float d = (mx - mn) / 15.0f;
  float id = d != 0.0f ? 1.0f / d : 0.0f;
  y->d = orc_f32_to_f16(d);
  y->m = orc_f32_to_f16(mn);
  for (int j = 0; j < QK / 2; j++) {
    int q0 = (int)(int8_t)((x[j] - mn) * id + 0.5f);
    int q1 = (int)(int8_t)((x[j + QK / 2] - mn) * id + 0.5f);
    q0 = q0 > 15 ? 15 : q0;
    q1 = q1 > 15 ? 15 : q1;
    y->qs[j] = (uint8_t)(q0 | (q1 << 4));
  }
}

void orc_quantize_q4_1(const float* x, int64_t n, uint8_t* blocks) {
  blk_q4_1* y = (blk_q4_1*)blocks;
#pragma omp parallel for schedule(static) if (n > (1 << 20))
  for (int64_t b = 0; b < n / QK; b++) quantize_q4_1_block(x + b * QK, y + b);
}

/* Q8_0 x Q8_0 block dot in the order of candle's AVX2 vec_dot: per block eight lanes of
 * four-product integer sums, each scaled by d_w*d_x into its own FMA accumulator, then the
 * hsum tree ((l0+l4)+(l2+l6)) + ((l1+l5)+(l3+l7)). */
static float vec_dot_q8_0(const blk_q8_0* w, const blk_q8_0* x, int nb) {
  float acc[8] = {0};
  for (int b = 0; b < nb; b++) {
    float dd = orc_f16_to_f32(w[b].d) * orc_f16_to_f32(x[b].d);
    for (int l = 0; l < 8; l++) {
      int32_t s = 0;
      for (int e = 0; e < 4; e++) s += (int32_t)w[b].qs[4 * l + e] * (int32_t)x[b].qs[4 * l + e];
      acc[l] = fmaf(dd, (float)s, acc[l]);
    }
  }
  float r0 = acc[0] + acc[4], r1 = acc[1] + acc[5], r2 = acc[2] + acc[6], r3 = acc[3] + acc[7];
  return (r0 + r2) + (r1 + r3);
}

#ifdef ORC_AVX2
static float vec_dot_q8_0_avx2(const blk_q8_0* w, const blk_q8_0* x, int nb) {
  __m256 acc = _mm256_setzero_ps();
  const __m256i ones = _mm256_set1_epi16(1);
  for (int b = 0; b < nb; b++) {
    __m256 d = _mm256_set1_ps(orc_f16_to_f32(w[b].d) * orc_f16_to_f32(x[b].d));
    __m256i bw = _mm256_loadu_si256((const __m256i*)w[b].qs);
    __m256i bx = _mm256_loadu_si256((const __m256i*)x[b].qs);
    __m256i aw = _mm256_sign_epi8(bw, bw);
    __m256i sx = _mm256_sign_epi8(bx, bw);
    __m256i p16 = _mm256_maddubs_epi16(aw, sx);
    __m256 q = _mm256_cvtepi32_ps(_mm256_madd_epi16(p16, ones));
    acc = _mm256_fmadd_ps(d, q, acc);
  }
  __m128 r = _mm_add_ps(_mm256_extractf128_ps(acc, 1), _mm256_castps256_ps128(acc));
  r = _mm_add_ps(r, _mm_movehl_ps(r, r));
  r = _mm_add_ss(r, _mm_movehdup_ps(r));
  return _mm_cvtss_f32(r);
}
#endif

/* Q4_1 x Q8_1 block dot in the order of ggml's AVX2 vec_dot_q4_1_q8_1 (Q4_1 has no
 * counterpart in the reference; this is the published x86 form of the format's dot). The
 * 32 nibbles unpack to values 0..15 (low nibbles of bytes 0..15) and 16..31 (high nibbles);
 * lane l sums the four products of values 4l..4l+3 and accumulates d_w*d_x times that sum
 * with an FMA, block after block; m_w * s_x is summed separately (product rounded, then
 * added). Result: the hsum tree of the lanes (as in vec_dot_q8_0) plus that sum. */
static float vec_dot_q4_1(const blk_q4_1* w, const blk_q8_1* x, int nb) {
  float acc[8] = {0};
  float summs = 0.0f;
  for (int b = 0; b < nb; b++) {
    float mprod = orc_f16_to_f32(w[b].m) * orc_f16_to_f32(x[b].s);
    summs = summs + mprod;
    float dd = orc_f16_to_f32(w[b].d) * orc_f16_to_f32(x[b].d);
    for (int l = 0; l < 8; l++) {
      int32_t s = 0;
      for (int e = 0; e < 4; e++) {
        int v = 4 * l + e;
        int q = v < QK / 2 ? (w[b].qs[v] & 0x0f) : (w[b].qs[v - QK / 2] >> 4);
        s += (int32_t)q * (int32_t)x[b].qs[v];
      }
      acc[l] = fmaf(dd, (float)s, acc[l]);
    }
  }
  float r0 = acc[0] + acc[4], r1 = acc[1] + acc[5], r2 = acc[2] + acc[6], r3 = acc[3] + acc[7];
  return ((r0 + r2) + (r1 + r3)) + summs;
}

static void matvec_q8_0_blocks(const blk_q8_0* xq, const uint8_t* wblocks, int n, int k,
                               float* out) {
  int nb = k / QK;
  const blk_q8_0* w = (const blk_q8_0*)wblocks;
#pragma omp parallel for schedule(static) if ((int64_t)n * k > 65536)
  for (int r = 0; r < n; r++) {
#ifdef ORC_AVX2
    out[r] = vec_dot_q8_0_avx2(w + (int64_t)r * nb, xq, nb);
#else
    out[r] = vec_dot_q8_0(w + (int64_t)r * nb, xq, nb);
#endif
  }
}

/* QMatMul::forward for one row (nn/mod.rs:97): the activation row is quantised to Q8_0,
 * then each output is an integer block dot product. */
void orc_matvec_q8_0(const float* x, const uint8_t* wblocks, int n, int k, float* out) {
  int nb = k / QK;
  blk_q8_0* xq = (blk_q8_0*)malloc(sizeof(blk_q8_0) * (size_t)nb);
  for (int b = 0; b < nb; b++) quantize_q8_0_block(x + b * QK, xq + b);
  matvec_q8_0_blocks(xq, wblocks, n, k, out);
  free(xq);
}

/* Exposed so the CPU tests can check the AVX2 block dot against the scalar statement. */
float orc_vec_dot_q8_0_scalar(const uint8_t* w, const uint8_t* x, int nb) {
  return vec_dot_q8_0((const blk_q8_0*)w, (const blk_q8_0*)x, nb);
}
float orc_vec_dot_q8_0(const uint8_t* w, const uint8_t* x, int nb) {
#ifdef ORC_AVX2
  return vec_dot_q8_0_avx2((const blk_q8_0*)w, (const blk_q8_0*)x, nb);
#else
  return vec_dot_q8_0((const blk_q8_0*)w, (const blk_q8_0*)x, nb);
#endif
}

void orc_matvec_q4_1(const float* x, const uint8_t* wblocks, int n, int k, float* out) {
  int nb = k / QK;
  blk_q8_1* xq = (blk_q8_1*)malloc(sizeof(blk_q8_1) * (size_t)nb);
  for (int b = 0; b < nb; b++) quantize_q8_1_block(x + b * QK, xq + b);
  const blk_q4_1* w = (const blk_q4_1*)wblocks;
#pragma omp parallel for schedule(static) if ((int64_t)n * k > 65536)
  for (int r = 0; r < n; r++) out[r] = vec_dot_q4_1(w + (int64_t)r * nb, xq, nb);
  free(xq);
}

/* ------------------------------------------------------------------ norms */

/* candle_nn::ops::rms_norm on CPU (used at transformer.rs:286, stt/model.rs:252):
 * m = sqrt(sum(x^2) / d + eps) with a sequential f32 sum, y = x / m * alpha. */
void orc_rms_norm(const float* x, const float* alpha, int d, float eps, float* out) {
  float sum2 = 0.0f;
  if (g_variant == 1)
    for (int i = d - 1; i >= 0; i--) sum2 += x[i] * x[i];
  else
    for (int i = 0; i < d; i++) sum2 += x[i] * x[i];
  float m = sqrtf(sum2 / (float)d + eps);
  for (int i = 0; i < d; i++) out[i] = x[i] / m * alpha[i];
}

/* candle_nn::ops::layer_norm on CPU (transformer.rs:284, tts/flow_lm.rs:176,380):
 * mean and mean square in one sequential pass, var = E[x^2] - mean^2,
 * y = (x - mean) * (1 / sqrt(var + eps)) * w + b. */
void orc_layer_norm(const float* x, const float* w, const float* b, int d, float eps,
                    float* out) {
  float sum = 0.0f, sum2 = 0.0f;
  for (int i = 0; i < d; i++) {
    sum += x[i];
    sum2 += x[i] * x[i];
  }
  float mean = sum / (float)d;
  float var = sum2 / (float)d - mean * mean;
  float inv_std = 1.0f / sqrtf(var + eps);
  for (int i = 0; i < d; i++) out[i] = (x[i] - mean) * inv_std * w[i] + b[i];
}

/* ------------------------------------------------------------------ attention */

static inline size_t sat_sub(size_t a, size_t b) { return a > b ? a - b : 0; }

/* attend (nn/kernels/attention.rs:142-169): scores scale*dot, max, exp(w - max), sequential
 * sum, then out += (w / sum) * v with FMA. */
static void attend(const float* q, const float* keys, const float* values, int64_t stride,
                   int count, int d, float scale, float* out, float* weights) {
  if (count <= 0) return;
  float mx = -INFINITY;
  for (int j = 0; j < count; j++) {
    weights[j] = scale * orc_dot(q, keys + (int64_t)j * stride, d);
    mx = (j == 0 || weights[j] > mx) ? weights[j] : mx;
  }
  float sum = 0.0f;
  for (int j = 0; j < count; j++) {
    weights[j] = orc_exp(weights[j] - mx);
    sum += weights[j];
  }
  for (int j = 0; j < count; j++) {
    float w = weights[j] / sum;
    const float* v = values + (int64_t)j * stride;
    for (int i = 0; i < d; i++) out[i] = fmaf(w, v[i], out[i]);
  }
}

/* Attention::cpu_fwd (nn/kernels/attention.rs:81-137) for batch 1: q [heads][t][d] at
 * positions position..position+t, k/v rows of n keys at positions first_key..first_key+n
 * (head stride and row stride given), query p sees keys j <= p with p - j < context.
 * Output [t][heads][d]. context <= 0 means unlimited. */
void orc_attention(const float* q, const float* k, const float* v, int heads, int kv_heads,
                   int t, int n, int d, int64_t k_head_stride, int64_t k_row_stride,
                   int position, int first_key, int context, float* out) {
  float scale = powf((float)d, -0.5f);
  size_t ctx = context > 0 ? (size_t)context : (size_t)-1;
  int tasks = t * heads;
  memset(out, 0, sizeof(float) * (size_t)tasks * d);
  int big = (int64_t)t * heads * n * d >= (1 << 16);
#pragma omp parallel if (big)
  {
    float* weights = (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
#pragma omp for schedule(static)
    for (int idx = 0; idx < tasks; idx++) {
      int step = idx / heads, head = idx % heads;
      int kv_head = head / (heads / kv_heads);
      size_t query = (size_t)position + step;
      size_t lo = sat_sub(query, sat_sub(ctx, 1));
      if (lo < (size_t)first_key) lo = first_key;
      size_t first = lo - first_key;
      size_t end = sat_sub(query + 1, first_key);
      if (end > (size_t)n) end = n;
      int count = (int)sat_sub(end, first);
      const float* qr = q + ((int64_t)head * t + step) * d;
      const float* kr = k + kv_head * k_head_stride + (int64_t)first * k_row_stride;
      const float* vr = v + kv_head * k_head_stride + (int64_t)first * k_row_stride;
      attend(qr, kr, vr, k_row_stride, count, d, scale, out + (int64_t)idx * d, weights);
    }
    free(weights);
  }
}

/* ------------------------------------------------------------------ model */

enum { DT_F32 = 0, DT_BF16 = 1, DT_Q8_0 = 2, DT_Q4_1 = 3 };

typedef struct {
  int n, k, dtype;
  float* w;     /* f32 (or bf16-valued f32) [n][k] */
  uint8_t* q;   /* quantised blocks */
  float* bias;  /* optional [n] */
} olin;

typedef struct {
  float *norm1_w, *norm1_b, *norm2_w, *norm2_b, *ls1, *ls2;
  olin in_proj, out_proj, ff1, ff2; /* ff1 = linear1 | linear_in, ff2 = linear2 | linear_out */
} olayer;

typedef struct {
  float* freqs;
  olin l1, l2;
  float* alpha;
} otime;

typedef struct {
  float *ln_w, *ln_b;
  olin mlp1, mlp2, mod;
} ores;

struct orc_lm {
  int kind;
  orc_tcfg cfg;
  orc_stt_extra stt;
  orc_tts_extra tts;
  olayer* layers;
  float* inv_freq;
  /* STT */
  float* text_emb;
  float** emb;
  float* out_norm;
  olin text_linear;
  olin* extra;
  /* TTS */
  float* cond_embed_table;
  olin input_linear;
  float *out_norm_w, *out_norm_b;
  olin out_eos;
  float* bos;
  otime time_emb[2];
  int n_time;
  olin cond_embed, input_proj, final_mod, final_linear;
  ores* res;
  /* ownership */
  void** owned;
  int n_owned, cap_owned;
};

typedef struct {
  float *k, *v; /* [kvh][cap][hd] */
  int len, start, cap;
} kvcache;

struct orc_state {
  kvcache* caches;
  int n_layers, kvh, hd, context, position;
};

static void* own(orc_lm* m, void* p) {
  if (m->n_owned == m->cap_owned) {
    m->cap_owned = m->cap_owned ? 2 * m->cap_owned : 64;
    m->owned = (void**)realloc(m->owned, sizeof(void*) * (size_t)m->cap_owned);
  }
  m->owned[m->n_owned++] = p;
  return p;
}

typedef struct {
  const orc_tensor* t;
  int n;
} wmap;

static const orc_tensor* find(wmap* w, const char* name) {
  for (int i = 0; i < w->n; i++)
    if (strcmp(w->t[i].name, name) == 0) return &w->t[i];
  return NULL;
}

/* Fetches a tensor by name and checks its element count, copying it (rounded to bf16 when
 * the model runs in bf16, as the reference's loader converts every tensor to the dtype). */
static float* get(orc_lm* m, wmap* w, const char* name, int64_t numel, int* ok) {
  const orc_tensor* t = find(w, name);
  if (!t) {
    if (*ok) set_err("missing tensor %s", name);
    *ok = 0;
    return NULL;
  }
  if (t->numel != numel) {
    if (*ok) set_err("tensor %s: %lld elements, expected %lld", name, (long long)t->numel,
                     (long long)numel);
    *ok = 0;
    return NULL;
  }
  float* p = (float*)own(m, malloc(sizeof(float) * (size_t)numel));
  memcpy(p, t->data, sizeof(float) * (size_t)numel);
  if (m->cfg.weight_dtype == DT_BF16)
    for (int64_t i = 0; i < numel; i++) p[i] = orc_round_bf16(p[i]);
  return p;
}

/* Linear::from_weight (nn/mod.rs:76-88): quantised when requested and k % 32 == 0. */
static void make_linear(orc_lm* m, wmap* w, olin* L, const char* wname, const char* bname,
                        int n, int k, int quantizable, int* ok) {
  L->n = n;
  L->k = k;
  L->dtype = m->cfg.weight_dtype == DT_BF16 ? DT_BF16 : DT_F32;
  L->w = get(m, w, wname, (int64_t)n * k, ok);
  L->bias = bname ? get(m, w, bname, n, ok) : NULL;
  L->q = NULL;
  if (!*ok) return;
  int qd = m->cfg.weight_dtype;
  if (quantizable && (qd == DT_Q8_0 || qd == DT_Q4_1) && k % QK == 0) {
    size_t bsz = qd == DT_Q8_0 ? sizeof(blk_q8_0) : sizeof(blk_q4_1);
    L->q = (uint8_t*)own(m, malloc(bsz * (size_t)n * (k / QK)));
    if (qd == DT_Q8_0)
      orc_quantize_q8_0(L->w, (int64_t)n * k, L->q);
    else
      orc_quantize_q4_1(L->w, (int64_t)n * k, L->q);
    L->dtype = qd;
  }
}

/* Linear::forward (nn/mod.rs:91-99) on one row. */
static void lin_row(const olin* L, const float* x, float* out) {
  switch (L->dtype) {
    case DT_Q8_0:
      orc_matvec_q8_0(x, L->q, L->n, L->k, out);
      break;
    case DT_Q4_1:
      orc_matvec_q4_1(x, L->q, L->n, L->k, out);
      break;
    case DT_BF16: {
      float* xr = (float*)malloc(sizeof(float) * (size_t)L->k);
      for (int i = 0; i < L->k; i++) xr[i] = orc_round_bf16(x[i]);
      orc_matvec(xr, L->w, L->bias, L->n, L->k, out);
      free(xr);
      break;
    }
    default:
      orc_matvec(x, L->w, L->bias, L->n, L->k, out);
  }
}

static void lin_rows(const olin* L, const float* x, int t, float* out) {
  for (int s = 0; s < t; s++) lin_row(L, x + (int64_t)s * L->k, out + (int64_t)s * L->n);
}

static void norm_rows(const orc_lm* m, const float* w, const float* b, const float* x, int t,
                      float* out) {
  int d = m->cfg.d_model;
  for (int s = 0; s < t; s++) {
    if (m->cfg.norm_kind == 1)
      orc_rms_norm(x + (int64_t)s * d, w, d, m->cfg.norm_eps, out + (int64_t)s * d);
    else
      orc_layer_norm(x + (int64_t)s * d, w, b, d, m->cfg.norm_eps, out + (int64_t)s * d);
  }
}

static int build_transformer(orc_lm* m, wmap* w, const char* prefix) {
  const orc_tcfg* c = &m->cfg;
  int ok = 1;
  int d = c->d_model, qd = c->num_heads * c->head_dim, kvd = c->num_kv_heads * c->head_dim;
  m->layers = (olayer*)own(m, calloc((size_t)c->num_layers, sizeof(olayer)));
  char a[256], b[256];
  for (int l = 0; l < c->num_layers && ok; l++) {
    olayer* L = &m->layers[l];
#define NM(buf, fmt) snprintf(buf, sizeof buf, "%slayers.%d." fmt, prefix, l)
    if (c->norm_kind == 1) {
      NM(a, "norm1.alpha");
      L->norm1_w = get(m, w, a, d, &ok);
      NM(a, "norm2.alpha");
      L->norm2_w = get(m, w, a, d, &ok);
    } else {
      NM(a, "norm1.weight");
      L->norm1_w = get(m, w, a, d, &ok);
      NM(a, "norm1.bias");
      L->norm1_b = get(m, w, a, d, &ok);
      NM(a, "norm2.weight");
      L->norm2_w = get(m, w, a, d, &ok);
      NM(a, "norm2.bias");
      L->norm2_b = get(m, w, a, d, &ok);
    }
    if (c->layer_scale) {
      NM(a, "layer_scale_1.scale");
      L->ls1 = get(m, w, a, d, &ok);
      NM(a, "layer_scale_2.scale");
      L->ls2 = get(m, w, a, d, &ok);
    }
    /* Attention::new (transformer.rs:300-316): moshi names in_proj_weight, Pocket TTS
     * in_proj.weight. */
    NM(a, "self_attn.in_proj_weight");
    if (!find(w, a)) NM(a, "self_attn.in_proj.weight");
    make_linear(m, w, &L->in_proj, a, NULL, qd + 2 * kvd, d, 1, &ok);
    NM(a, "self_attn.out_proj.weight");
    make_linear(m, w, &L->out_proj, a, NULL, d, qd, 1, &ok);
    /* FeedForwardLayer::new (transformer.rs:418-436). */
    if (c->ffn_kind == 2) {
      NM(a, "gating.linear_in.weight");
      make_linear(m, w, &L->ff1, a, NULL, 2 * c->ffn_hidden, d, 1, &ok);
      NM(b, "gating.linear_out.weight");
      make_linear(m, w, &L->ff2, b, NULL, d, c->ffn_hidden, 1, &ok);
    } else {
      NM(a, "linear1.weight");
      make_linear(m, w, &L->ff1, a, NULL, c->ffn_hidden, d, 1, &ok);
      NM(b, "linear2.weight");
      make_linear(m, w, &L->ff2, b, NULL, d, c->ffn_hidden, 1, &ok);
    }
#undef NM
  }
  /* RoPE inverse frequencies in f64, stored f32 (transformer.rs:114-118). */
  int half = c->head_dim / 2;
  m->inv_freq = (float*)own(m, malloc(sizeof(float) * (size_t)half));
  for (int i = 0; i < half; i++)
    m->inv_freq[i] = (float)exp(-log(c->max_period) * 2.0 * (double)i / (double)c->head_dim);
  return ok;
}

static int build_stt(orc_lm* m, wmap* w) {
  int ok = 1, d = m->cfg.d_model;
  const orc_stt_extra* s = &m->stt;
  char a[128];
  /* LanguageModel::new (stt/model.rs:196-233). */
  m->text_emb = get(m, w, "text_emb.weight", (int64_t)(s->text_card + 1) * d, &ok);
  m->emb = (float**)own(m, calloc((size_t)s->n_q, sizeof(float*)));
  for (int c = 0; c < s->n_q; c++) {
    snprintf(a, sizeof a, "emb.%d.weight", c);
    m->emb[c] = get(m, w, a, (int64_t)(s->card + 1) * d, &ok);
  }
  if (!ok) return 0;
  if (!build_transformer(m, w, "transformer.")) return 0;
  m->out_norm = get(m, w, "out_norm.alpha", d, &ok);
  make_linear(m, w, &m->text_linear, "text_linear.weight", NULL, s->text_card, d, 1, &ok);
  m->extra = (olin*)own(m, calloc((size_t)(s->extra_heads_num > 0 ? s->extra_heads_num : 1),
                                  sizeof(olin)));
  for (int i = 0; i < s->extra_heads_num && ok; i++) {
    snprintf(a, sizeof a, "extra_heads.%d.weight", i);
    make_linear(m, w, &m->extra[i], a, NULL, s->extra_heads_dim, d, 0, &ok);
  }
  return ok;
}

static int build_tts(orc_lm* m, wmap* w) {
  int ok = 1, d = m->cfg.d_model;
  const orc_tts_extra* t = &m->tts;
  int dim = t->flow_dim, ld = t->latent_dim;
  char a[160], b[160];
  /* FlowLm::new (tts/flow_lm.rs:45-126), without the low-rank table and z_proj. */
  m->cond_embed_table = get(m, w, "conditioner.embed.weight", (int64_t)(t->text_bins + 1) * d, &ok);
  make_linear(m, w, &m->input_linear, "input_linear.weight", NULL, d, ld, 0, &ok);
  if (!ok) return 0;
  if (!build_transformer(m, w, "transformer.")) return 0;
  m->out_norm_w = get(m, w, "out_norm.weight", d, &ok);
  m->out_norm_b = get(m, w, "out_norm.bias", d, &ok);
  make_linear(m, w, &m->out_eos, "out_eos.weight", "out_eos.bias", 1, d, 0, &ok);
  m->bos = get(m, w, "bos_emb", ld, &ok);
  /* FlowHead::new (tts/flow_lm.rs:239-257). */
  m->n_time = t->flow_kind == 0 ? 2 : (t->flow_kind == 1 ? 1 : 0);
  for (int i = 0; i < m->n_time && ok; i++) {
    otime* e = &m->time_emb[i];
    snprintf(a, sizeof a, "flow_net.time_embed.%d.freqs", i);
    e->freqs = get(m, w, a, 128, &ok);
    snprintf(a, sizeof a, "flow_net.time_embed.%d.mlp.0.weight", i);
    snprintf(b, sizeof b, "flow_net.time_embed.%d.mlp.0.bias", i);
    make_linear(m, w, &e->l1, a, b, dim, 256, 0, &ok);
    snprintf(a, sizeof a, "flow_net.time_embed.%d.mlp.2.weight", i);
    snprintf(b, sizeof b, "flow_net.time_embed.%d.mlp.2.bias", i);
    make_linear(m, w, &e->l2, a, b, dim, dim, 0, &ok);
    snprintf(a, sizeof a, "flow_net.time_embed.%d.mlp.3.alpha", i);
    e->alpha = get(m, w, a, dim, &ok);
  }
  make_linear(m, w, &m->cond_embed, "flow_net.cond_embed.weight", "flow_net.cond_embed.bias",
              dim, d, 0, &ok);
  make_linear(m, w, &m->input_proj, "flow_net.input_proj.weight", "flow_net.input_proj.bias",
              dim, ld, 0, &ok);
  m->res = (ores*)own(m, calloc((size_t)(t->flow_depth > 0 ? t->flow_depth : 1), sizeof(ores)));
  for (int i = 0; i < t->flow_depth && ok; i++) {
    ores* r = &m->res[i];
    snprintf(a, sizeof a, "flow_net.res_blocks.%d.in_ln.weight", i);
    r->ln_w = get(m, w, a, dim, &ok);
    snprintf(a, sizeof a, "flow_net.res_blocks.%d.in_ln.bias", i);
    r->ln_b = get(m, w, a, dim, &ok);
    snprintf(a, sizeof a, "flow_net.res_blocks.%d.mlp.0.weight", i);
    snprintf(b, sizeof b, "flow_net.res_blocks.%d.mlp.0.bias", i);
    make_linear(m, w, &r->mlp1, a, b, dim, dim, 0, &ok);
    snprintf(a, sizeof a, "flow_net.res_blocks.%d.mlp.2.weight", i);
    snprintf(b, sizeof b, "flow_net.res_blocks.%d.mlp.2.bias", i);
    make_linear(m, w, &r->mlp2, a, b, dim, dim, 0, &ok);
    snprintf(a, sizeof a, "flow_net.res_blocks.%d.adaLN_modulation.1.weight", i);
    snprintf(b, sizeof b, "flow_net.res_blocks.%d.adaLN_modulation.1.bias", i);
    make_linear(m, w, &r->mod, a, b, 3 * dim, dim, 0, &ok);
  }
  make_linear(m, w, &m->final_mod, "flow_net.final_layer.adaLN_modulation.1.weight",
              "flow_net.final_layer.adaLN_modulation.1.bias", 2 * dim, dim, 0, &ok);
  make_linear(m, w, &m->final_linear, "flow_net.final_layer.linear.weight",
              "flow_net.final_layer.linear.bias", ld, dim, 0, &ok);
  return ok;
}

void orc_lm_free(orc_lm* m) {
  if (!m) return;
  for (int i = 0; i < m->n_owned; i++) free(m->owned[i]);
  free(m->owned);
  free(m);
}

orc_lm* orc_lm_create(int kind, const orc_tcfg* cfg, const orc_stt_extra* stt,
                      const orc_tts_extra* tts, const orc_tensor* tensors, int n_tensors) {
  if (!cfg || cfg->d_model <= 0 || cfg->num_layers <= 0 || cfg->num_heads <= 0 ||
      cfg->num_kv_heads <= 0 || cfg->head_dim <= 0 || cfg->num_heads % cfg->num_kv_heads ||
      cfg->head_dim % 2) {
    set_err("invalid transformer config");
    return NULL;
  }
  orc_lm* m = (orc_lm*)calloc(1, sizeof(orc_lm));
  m->kind = kind;
  m->cfg = *cfg;
  if (stt) m->stt = *stt;
  if (tts) m->tts = *tts;
  wmap w = {tensors, n_tensors};
  int ok = kind == 0 ? build_stt(m, &w) : build_tts(m, &w);
  if (!ok) {
    orc_lm_free(m);
    return NULL;
  }
  return m;
}

/* Transformer::new (transformer.rs:106-125) alone, its tensors named under `prefix`: the
 * transformer of Mimi's ProjectedTransformer (nn/mimi.rs:74-112). */
orc_lm* orc_transformer_create(const orc_tcfg* cfg, const char* prefix, const orc_tensor* tensors,
                               int n_tensors) {
  if (!cfg || !prefix || cfg->d_model <= 0 || cfg->num_layers <= 0 || cfg->num_heads <= 0 ||
      cfg->num_kv_heads <= 0 || cfg->head_dim <= 0 || cfg->num_heads % cfg->num_kv_heads ||
      cfg->head_dim % 2) {
    set_err("invalid transformer config");
    return NULL;
  }
  orc_lm* m = (orc_lm*)calloc(1, sizeof(orc_lm));
  m->kind = 2;
  m->cfg = *cfg;
  wmap w = {tensors, n_tensors};
  if (!build_transformer(m, &w, prefix)) {
    orc_lm_free(m);
    return NULL;
  }
  return m;
}

/* Transformer::init_state (transformer.rs:127-136). */
orc_state* orc_state_create(orc_lm* m) {
  orc_state* s = (orc_state*)calloc(1, sizeof(orc_state));
  s->n_layers = m->cfg.num_layers;
  s->caches = (kvcache*)calloc((size_t)s->n_layers, sizeof(kvcache));
  s->kvh = m->cfg.num_kv_heads;
  s->hd = m->cfg.head_dim;
  s->context = m->cfg.context;
  return s;
}

/* TransformerState::duplicate (transformer.rs:64-73). */
orc_state* orc_state_duplicate(const orc_state* src) {
  orc_state* s = (orc_state*)malloc(sizeof(orc_state));
  *s = *src;
  s->caches = (kvcache*)calloc((size_t)s->n_layers, sizeof(kvcache));
  for (int l = 0; l < s->n_layers; l++) {
    kvcache* c = &s->caches[l];
    *c = src->caches[l];
    if (c->cap) {
      size_t bytes = sizeof(float) * (size_t)s->kvh * c->cap * s->hd;
      c->k = (float*)malloc(bytes);
      c->v = (float*)malloc(bytes);
      memcpy(c->k, src->caches[l].k, bytes);
      memcpy(c->v, src->caches[l].v, bytes);
    }
  }
  return s;
}

void orc_state_free(orc_state* s) {
  if (!s) return;
  for (int l = 0; l < s->n_layers; l++) {
    free(s->caches[l].k);
    free(s->caches[l].v);
  }
  free(s->caches);
  free(s);
}

int orc_state_position(const orc_state* s) { return s->position; }

/* KvCache::append (transformer.rs:508-550): on overflow keep the last min(len, window)
 * entries in a buffer of capacity 2*window + t (geometric growth without a window), then
 * hand out the last min(len, window + t - 1) entries and the position of the first. */
static void cache_append(kvcache* c, int kvh, int hd, int window, const float* k,
                         const float* v, int t, int* offset, int* visible, int* first_key) {
  if (c->len + t > c->cap) {
    int keep = window > 0 ? (c->len < window ? c->len : window) : c->len;
    int drop = c->len - keep;
    int ncap;
    if (window > 0) {
      ncap = 2 * window + t;
    } else {
      ncap = 2 * c->cap;
      if (ncap < keep + t) ncap = keep + t;
      if (ncap < 64) ncap = 64;
    }
    float* nk = (float*)calloc((size_t)kvh * ncap * hd, sizeof(float));
    float* nv = (float*)calloc((size_t)kvh * ncap * hd, sizeof(float));
    if (c->cap && keep > 0)
      for (int h = 0; h < kvh; h++) {
        memcpy(nk + (size_t)h * ncap * hd, c->k + ((size_t)h * c->cap + drop) * hd,
               sizeof(float) * (size_t)keep * hd);
        memcpy(nv + (size_t)h * ncap * hd, c->v + ((size_t)h * c->cap + drop) * hd,
               sizeof(float) * (size_t)keep * hd);
      }
    free(c->k);
    free(c->v);
    c->k = nk;
    c->v = nv;
    c->cap = ncap;
    c->start += drop;
    c->len = keep;
  }
  for (int h = 0; h < kvh; h++) {
    memcpy(c->k + ((size_t)h * c->cap + c->len) * hd, k + (size_t)h * t * hd,
           sizeof(float) * (size_t)t * hd);
    memcpy(c->v + ((size_t)h * c->cap + c->len) * hd, v + (size_t)h * t * hd,
           sizeof(float) * (size_t)t * hd);
  }
  c->len += t;
  int vis = window > 0 ? (c->len < window + t - 1 ? c->len : window + t - 1) : c->len;
  *visible = vis;
  *offset = c->len - vis;
  *first_key = c->start + *offset;
}

/* Layer::forward (transformer.rs:222-250) with Attention::forward (:318-365) and
 * FeedForwardLayer::forward (:438-464), for one stream and t steps. */
static void layer_forward(const orc_lm* m, const olayer* L, float* xs, int t, kvcache* cache,
                          int position, const float* cosv, const float* sinv) {
  const orc_tcfg* c = &m->cfg;
  int d = c->d_model, H = c->num_heads, KVH = c->num_kv_heads, hd = c->head_dim;
  int qd = H * hd, kvd = KVH * hd, nqkv = qd + 2 * kvd, half = hd / 2;
  float* h = (float*)malloc(sizeof(float) * (size_t)t * d);
  float* qkv = (float*)malloc(sizeof(float) * (size_t)t * nqkv);
  float* q = (float*)malloc(sizeof(float) * (size_t)H * t * hd);
  float* k = (float*)malloc(sizeof(float) * (size_t)KVH * t * hd);
  float* v = (float*)malloc(sizeof(float) * (size_t)KVH * t * hd);
  float* att = (float*)malloc(sizeof(float) * (size_t)t * qd);
  float* upd = (float*)malloc(sizeof(float) * (size_t)t * d);

  norm_rows(m, L->norm1_w, L->norm1_b, xs, t, h);
  lin_rows(&L->in_proj, h, t, qkv);
  /* split q|k|v (:330-338) into [heads][t][hd], then rope_i on q and k (:339-340):
   * out[2i] = x[2i] cos - x[2i+1] sin, out[2i+1] = x[2i] sin + x[2i+1] cos. */
  for (int s = 0; s < t; s++) {
    const float* row = qkv + (size_t)s * nqkv;
    for (int hh = 0; hh < H; hh++) memcpy(q + ((size_t)hh * t + s) * hd, row + hh * hd, sizeof(float) * hd);
    for (int hh = 0; hh < KVH; hh++) {
      memcpy(k + ((size_t)hh * t + s) * hd, row + qd + hh * hd, sizeof(float) * hd);
      memcpy(v + ((size_t)hh * t + s) * hd, row + qd + kvd + hh * hd, sizeof(float) * hd);
    }
  }
  for (int pass = 0; pass < 2; pass++) {
    float* x = pass ? k : q;
    int heads = pass ? KVH : H;
    for (int hh = 0; hh < heads; hh++)
      for (int s = 0; s < t; s++) {
        float* r = x + ((size_t)hh * t + s) * hd;
        const float* cs = cosv + (size_t)s * half;
        const float* sn = sinv + (size_t)s * half;
        for (int i = 0; i < half; i++) {
          float a = r[2 * i], b = r[2 * i + 1];
          float p0 = a * cs[i], p1 = b * sn[i], p2 = a * sn[i], p3 = b * cs[i];
          r[2 * i] = p0 - p1;
          r[2 * i + 1] = p2 + p3;
        }
      }
  }
  if (c->kv_dtype == 1)
    for (size_t i = 0; i < (size_t)KVH * t * hd; i++) {
      k[i] = orc_round_bf16(k[i]);
      v[i] = orc_round_bf16(v[i]);
    }
  int offset, visible, first_key;
  cache_append(cache, KVH, hd, c->context, k, v, t, &offset, &visible, &first_key);
  orc_attention(q, cache->k + (size_t)offset * hd, cache->v + (size_t)offset * hd, H, KVH, t,
                visible, hd, (int64_t)cache->cap * hd, hd, position, first_key, c->context, att);
  lin_rows(&L->out_proj, att, t, upd);
  for (size_t i = 0; i < (size_t)t * d; i++) {
    float u = L->ls1 ? upd[i] * L->ls1[i % d] : upd[i];
    xs[i] = xs[i] + u;
  }
  norm_rows(m, L->norm2_w, L->norm2_b, xs, t, h);
  int F = c->ffn_hidden;
  float* hid = (float*)malloc(sizeof(float) * (size_t)t * L->ff1.n);
  lin_rows(&L->ff1, h, t, hid);
  float* act = (float*)malloc(sizeof(float) * (size_t)t * F);
  for (int s = 0; s < t; s++) {
    const float* hr = hid + (size_t)s * L->ff1.n;
    float* ar = act + (size_t)s * F;
    if (c->ffn_kind == 2) {
      for (int i = 0; i < F; i++) ar[i] = orc_silu(hr[i]) * hr[F + i];
    } else if (c->ffn_kind == 1) {
      for (int i = 0; i < F; i++) ar[i] = gelu_erf(hr[i]);
    } else {
      for (int i = 0; i < F; i++) ar[i] = orc_gelu_tanh(hr[i]);
    }
  }
  lin_rows(&L->ff2, act, t, upd);
  for (size_t i = 0; i < (size_t)t * d; i++) {
    float u = L->ls2 ? upd[i] * L->ls2[i % d] : upd[i];
    xs[i] = xs[i] + u;
  }
  free(hid);
  free(act);
  free(h);
  free(qkv);
  free(q);
  free(k);
  free(v);
  free(att);
  free(upd);
}

/* Transformer::forward_block (transformer.rs:156-186): RoPE table for the positions of the
 * block (freqs = position * inv_freq in f32, then cos and sin), every layer, position += t. */
static void forward_block(const orc_lm* m, orc_state* st, float* xs, int t) {
  if (t == 0) return;
  int half = m->cfg.head_dim / 2;
  float* cosv = (float*)malloc(sizeof(float) * (size_t)t * half);
  float* sinv = (float*)malloc(sizeof(float) * (size_t)t * half);
  for (int s = 0; s < t; s++)
    for (int i = 0; i < half; i++) {
      float f = (float)(st->position + s) * m->inv_freq[i];
      cosv[s * half + i] = cosf(f);
      sinv[s * half + i] = sinf(f);
    }
  for (int l = 0; l < m->cfg.num_layers; l++)
    layer_forward(m, &m->layers[l], xs, t, &st->caches[l], st->position, cosv, sinv);
  st->position += t;
  free(cosv);
  free(sinv);
}

/* Transformer::forward (transformer.rs:139-154): inputs longer than the window go through
 * in window-sized blocks. */
int orc_transformer_forward(orc_lm* m, orc_state* st, float* xs, int t) {
  int ctx = m->cfg.context;
  if (ctx > 0 && t > ctx) {
    for (int s0 = 0; s0 < t; s0 += ctx)
      forward_block(m, st, xs + (size_t)s0 * m->cfg.d_model, t - s0 < ctx ? t - s0 : ctx);
  } else {
    forward_block(m, st, xs, t);
  }
  return 0;
}

/* softmax_last_dim's first probability (stt/model.rs:259-271): max, exp(x - max) with the
 * standard exp, sequential sum. */
static float softmax_p0(const float* x, int n) {
  float mx = x[0];
  for (int i = 1; i < n; i++) mx = x[i] > mx ? x[i] : mx;
  float sum = 0.0f, e0 = 0.0f;
  for (int i = 0; i < n; i++) {
    float e = expf(x[i] - mx);
    if (i == 0) e0 = e;
    sum += e;
  }
  return e0 / sum;
}

/* LanguageModel::step (stt/model.rs:239-277). */
int orc_stt_step(orc_lm* m, orc_state* st, uint32_t text_token, const uint32_t* audio,
                 uint32_t* out_token, float* logits, float* extra) {
  if (m->kind != 0) {
    set_err("not an STT model");
    return 2;
  }
  const orc_stt_extra* s = &m->stt;
  int d = m->cfg.d_model;
  if (text_token > (uint32_t)s->text_card) {
    set_err("text token %u out of range", text_token);
    return 2;
  }
  for (int c = 0; c < s->n_q; c++)
    if (audio[c] > (uint32_t)s->card) {
      set_err("audio token %u out of range", audio[c]);
      return 2;
    }
  float* x = (float*)malloc(sizeof(float) * (size_t)d);
  memcpy(x, m->text_emb + (size_t)text_token * d, sizeof(float) * (size_t)d);
  for (int c = 0; c < s->n_q; c++) {
    const float* e = m->emb[c] + (size_t)audio[c] * d;
    for (int i = 0; i < d; i++) x[i] = x[i] + e[i];
  }
  orc_transformer_forward(m, st, x, 1);
  float* ys = (float*)malloc(sizeof(float) * (size_t)d);
  orc_rms_norm(x, m->out_norm, d, 1e-8f, ys);
  float* lg = logits ? logits : (float*)malloc(sizeof(float) * (size_t)s->text_card);
  lin_row(&m->text_linear, ys, lg);
  /* argmax: the first index of the maximum; NaN never wins. */
  uint32_t best = 0;
  float bv = -INFINITY;
  int have = 0;
  for (int i = 0; i < s->text_card; i++)
    if (lg[i] == lg[i] && (!have || lg[i] > bv)) {
      bv = lg[i];
      best = (uint32_t)i;
      have = 1;
    }
  *out_token = best;
  if (extra && s->extra_heads_num > 0) {
    float* hl = (float*)malloc(sizeof(float) * (size_t)s->extra_heads_dim);
    for (int i = 0; i < s->extra_heads_num; i++) {
      lin_row(&m->extra[i], ys, hl);
      extra[i] = softmax_p0(hl, s->extra_heads_dim);
    }
    free(hl);
  }
  if (!logits) free(lg);
  free(x);
  free(ys);
  return 0;
}

/* ------------------------------------------------------------------ Pocket-TTS head */

/* layer_norm_no_affine (tts/flow_lm.rs:226-231): mean, centred, mean of squares. */
static void ln_no_affine(const float* x, int n, float eps, float* out) {
  float sum = 0.0f;
  for (int i = 0; i < n; i++) sum += x[i];
  /* candle's mean_keepdim multiplies the sum by the f64 scale 1/n, cast to f32. */
  float inv_n = (float)(1.0 / (double)n);
  float mean = sum * inv_n;
  float s2 = 0.0f;
  for (int i = 0; i < n; i++) {
    out[i] = x[i] - mean;
    s2 += out[i] * out[i];
  }
  float den = sqrtf(s2 * inv_n + eps);
  for (int i = 0; i < n; i++) out[i] = out[i] / den;
}

/* TimestepEmbedder::forward (tts/flow_lm.rs:339-351). */
static void time_embed(const otime* e, float t, int dim, float* out) {
  float emb[256], h[1024];
  for (int i = 0; i < 128; i++) {
    float a = e->freqs[i] * t;
    emb[i] = cosf(a);
    emb[128 + i] = sinf(a);
  }
  lin_row(&e->l1, emb, h);
  for (int i = 0; i < dim; i++) h[i] = orc_silu(h[i]);
  lin_row(&e->l2, h, out);
  float sum = 0.0f;
  for (int i = 0; i < dim; i++) sum += out[i];
  float mean = sum * (float)(1.0 / (double)dim), s2 = 0.0f;
  for (int i = 0; i < dim; i++) {
    float c = out[i] - mean;
    s2 += c * c;
  }
  float var = s2 * (float)(1.0 / (double)(dim - 1));
  float r = 1.0f / sqrtf(var + 1e-5f);
  for (int i = 0; i < dim; i++) out[i] = out[i] * r * e->alpha[i];
}

/* FlowHead::forward (tts/flow_lm.rs:259-287) with ResBlock::forward (:373-386). */
static void flow_forward(const orc_lm* m, const float* cond, const float* times, const float* x,
                         float* out) {
  int dim = m->tts.flow_dim;
  float* y = (float*)malloc(sizeof(float) * (size_t)dim);
  float* te = (float*)malloc(sizeof(float) * (size_t)dim);
  float* ts = (float*)calloc((size_t)dim, sizeof(float));
  float* xs = (float*)malloc(sizeof(float) * (size_t)dim);
  float* sy = (float*)malloc(sizeof(float) * (size_t)dim);
  float* mod = (float*)malloc(sizeof(float) * (size_t)3 * dim);
  float* hh = (float*)malloc(sizeof(float) * (size_t)dim);
  float* h2 = (float*)malloc(sizeof(float) * (size_t)dim);
  lin_row(&m->cond_embed, cond, y);
  if (m->n_time > 0) {
    for (int i = 0; i < m->n_time; i++) {
      time_embed(&m->time_emb[i], times[i], dim, te);
      for (int j = 0; j < dim; j++) ts[j] = i == 0 ? te[j] : ts[j] + te[j];
    }
    for (int j = 0; j < dim; j++) y[j] = y[j] + ts[j] * (float)(1.0 / (double)m->n_time);
  }
  lin_row(&m->input_proj, x, xs);
  for (int j = 0; j < dim; j++) sy[j] = orc_silu(y[j]);
  for (int b = 0; b < m->tts.flow_depth; b++) {
    const ores* r = &m->res[b];
    lin_row(&r->mod, sy, mod);
    orc_layer_norm(xs, r->ln_w, r->ln_b, dim, 1e-6f, hh);
    for (int j = 0; j < dim; j++) hh[j] = hh[j] * (mod[dim + j] + 1.0f) + mod[j];
    lin_row(&r->mlp1, hh, h2);
    for (int j = 0; j < dim; j++) h2[j] = orc_silu(h2[j]);
    lin_row(&r->mlp2, h2, hh);
    for (int j = 0; j < dim; j++) xs[j] = xs[j] + mod[2 * dim + j] * hh[j];
  }
  lin_row(&m->final_mod, sy, mod);
  ln_no_affine(xs, dim, 1e-6f, hh);
  for (int j = 0; j < dim; j++) hh[j] = hh[j] * (mod[dim + j] + 1.0f) + mod[j];
  lin_row(&m->final_linear, hh, out);
  free(y);
  free(te);
  free(ts);
  free(xs);
  free(sy);
  free(mod);
  free(hh);
  free(h2);
}

/* FlowLm::step (tts/flow_lm.rs:162-185) with FlowHead::decode (:290-315). */
int orc_tts_step(orc_lm* m, orc_state* st, const float* latent_in, const float* noise,
                 float decode_steps_f, float* latent_out, float* eos_logit) {
  if (m->kind != 1) {
    set_err("not a TTS model");
    return 2;
  }
  int d = m->cfg.d_model, ld = m->tts.latent_dim;
  float* xs = (float*)malloc(sizeof(float) * (size_t)d);
  float* z = (float*)malloc(sizeof(float) * (size_t)d);
  lin_row(&m->input_linear, latent_in ? latent_in : m->bos, xs);
  orc_transformer_forward(m, st, xs, 1);
  orc_layer_norm(xs, m->out_norm_w, m->out_norm_b, d, 1e-5f, z);
  lin_row(&m->out_eos, z, eos_logit);
  int steps = (int)decode_steps_f;
  if (steps < 1) steps = 1;
  float* x = (float*)malloc(sizeof(float) * (size_t)ld);
  float* flow = (float*)malloc(sizeof(float) * (size_t)ld);
  memcpy(x, noise, sizeof(float) * (size_t)ld);
  int kind = m->tts.flow_kind;
  if (kind == 0 || kind == 1) {
    for (int i = 0; i < steps; i++) {
      float times[2];
      if (kind == 0) {
        times[0] = (float)i / (float)steps;
        times[1] = (float)(i + 1) / (float)steps;
      } else {
        times[0] = (float)i / (float)steps;
      }
      flow_forward(m, z, times, x, flow);
      for (int j = 0; j < ld; j++) x[j] = x[j] + flow[j] * (float)(1.0 / (double)steps);
    }
  } else {
    flow_forward(m, z, NULL, x, flow);
    for (int j = 0; j < ld; j++) x[j] = kind == 2 ? flow[j] : x[j] + flow[j];
  }
  memcpy(latent_out, x, sizeof(float) * (size_t)ld);
  free(x);
  free(flow);
  free(xs);
  free(z);
  return 0;
}

/* FlowLm::prompt_text (tts/flow_lm.rs:150-158): embedding rows, one transformer pass. */
int orc_tts_prompt_text(orc_lm* m, orc_state* st, const uint32_t* tokens, int n) {
  int d = m->cfg.d_model;
  float* xs = (float*)malloc(sizeof(float) * (size_t)n * d);
  for (int i = 0; i < n; i++) {
    if (tokens[i] > (uint32_t)m->tts.text_bins) {
      free(xs);
      set_err("text token %u out of range", tokens[i]);
      return 2;
    }
    memcpy(xs + (size_t)i * d, m->cond_embed_table + (size_t)tokens[i] * d, sizeof(float) * d);
  }
  orc_transformer_forward(m, st, xs, n);
  free(xs);
  return 0;
}
