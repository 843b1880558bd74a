/*
 * qgemm_oracle.c -- CPU oracle for the W4A16 path (TEST INFRASTRUCTURE ONLY).
 *
 * Plain-C restatement of the reference's host numerics
 * (titoatwork/qgemm-mx include/qgemm/pack.hpp, include/qgemm/ref_gemm.hpp).
 * Each function cites the reference lines whose decision rule it restates.
 * This file is the checker for the CUDA product path and the "port" CPU
 * baseline; the product never links it.  Build: oracle/Makefile (no
 * -ffast-math, -ffp-contract=off, so IEEE rounding and subnormals hold).
 */
#include "qgemm_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* ------------------------------------------------------------------------ */
/* FP16 <-> FP32 (pack.hpp:183-253)                                          */
/* ------------------------------------------------------------------------ */

/* pack.hpp:183-211: exact widening, subnormal halves renormalised. */
float or_fp16_bits_to_float(uint16_t h) {
  uint32_t s = (uint32_t)(h >> 15) & 1u, e = (uint32_t)(h >> 10) & 0x1Fu,
           m = (uint32_t)h & 0x3FFu, out;
  if (e == 0) {
    if (m == 0) {
      out = s << 31;
    } else {
      uint32_t ex = 113; /* 127 - 15 + 1 */
      while ((m & 0x400u) == 0) { m <<= 1; --ex; }
      out = (s << 31) | (ex << 23) | ((m & 0x3FFu) << 13);
    }
  } else if (e == 31) {
    out = (s << 31) | 0x7F800000u | (m << 13);
  } else {
    out = (s << 31) | ((e + 112u) << 23) | (m << 13);
  }
  return u2f(out);
}

/* pack.hpp:213-253: round-to-nearest-even narrowing; NaN -> 0x7C00|0x200,
 * overflow (also by rounding) -> Inf, values below 2^-25 -> signed zero. */
uint16_t or_float_to_fp16_bits(float f) {
  uint32_t x = f2u(f);
  uint32_t sign = (x >> 16) & 0x8000u;
  int32_t exp = (int32_t)((x >> 23) & 0xFFu) - 112; /* -127 + 15 */
  uint32_t mant = x & 0x7FFFFFu;
  if (((x >> 23) & 0xFFu) == 0xFFu)
    return (uint16_t)(sign | 0x7C00u | (mant ? 0x200u : 0u));
  if (exp <= 0) {
    if (exp < -10) return (uint16_t)sign;
    mant |= 0x800000u;
    uint32_t shift = (uint32_t)(14 - exp);
    uint32_t hm = mant >> shift;
    uint32_t rem = mant & ((1u << shift) - 1u), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (hm & 1u))) ++hm;
    return (uint16_t)(sign | hm);
  }
  if (exp >= 31) return (uint16_t)(sign | 0x7C00u);
  uint32_t hm = mant >> 13, rem = mant & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (hm & 1u))) {
    if (++hm == 0x400u) {
      hm = 0;
      if (++exp >= 31) return (uint16_t)(sign | 0x7C00u);
    }
  }
  return (uint16_t)(sign | ((uint32_t)exp << 10) | hm);
}

/* ------------------------------------------------------------------------ */
/* E2M1 (pack.hpp:260-293)                                                   */
/* ------------------------------------------------------------------------ */

static const float kE2m1Mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};

float or_e2m1_decode(uint8_t code) {
  float mag = kE2m1Mag[code & 7u];
  return (code & 8u) ? -mag : mag;
}

/* pack.hpp:272-293: first candidate (ascending magnitude) with the smallest
 * float-rounded |a - t| wins, so ties go to the smaller magnitude; zero drops
 * the sign; non-finite inputs map to +-6 by sign bit. */
uint8_t or_e2m1_encode(float v) {
  if (!isfinite(v)) return signbit(v) ? 0xFu : 0x7u;
  float a = fabsf(v);
  int best = 0;
  float best_err = fabsf(a - kE2m1Mag[0]);
  for (int i = 1; i < 8; ++i) {
    float err = fabsf(a - kE2m1Mag[i]);
    if (err < best_err) { best_err = err; best = i; }
  }
  uint8_t code = (uint8_t)best;
  if (best != 0 && signbit(v)) code |= 8u;
  return code;
}

/* ------------------------------------------------------------------------ */
/* E8M0 (pack.hpp:299-327)                                                   */
/* ------------------------------------------------------------------------ */

float or_e8m0_decode(uint8_t bits) {
  if (bits == 0xFFu) return u2f(0x7FC00000u); /* quiet NaN */
  return ldexpf(1.0f, (int)bits - 127);
}

/* pack.hpp:308-327: frexp mantissa m in [0.5,1); round up to 2^e when
 * m >= 0.70710678f (float literal), else 2^(e-1); clamp to [0,254]. */
uint8_t or_e8m0_encode(float scale) {
  if (!isfinite(scale)) return 0xFFu;
  if (scale <= 0.0f) return 0;
  int e = 0;
  (void)frexpf(scale, &e);
  float m = ldexpf(scale, -e);
  int pw = (m < 0.7071067811865476f) ? e - 1 : e;
  int bits = pw + 127;
  if (bits < 0) bits = 0;
  if (bits > 254) bits = 254;
  return (uint8_t)bits;
}

/* ------------------------------------------------------------------------ */
/* E4M3 (pack.hpp:333-374)                                                   */
/* ------------------------------------------------------------------------ */

float or_e4m3_decode(uint8_t bits) {
  int s = (bits >> 7) & 1, e = (bits >> 3) & 0xF, m = bits & 7;
  if (e == 0xF && m == 7) return u2f(0x7FC00000u);
  float mag = (e == 0) ? ldexpf((float)m, -9) : ldexpf(1.0f + (float)m * 0.125f, e - 7);
  return s ? -mag : mag;
}

/* pack.hpp:352-374: exhaustive nearest over the 127 finite positive codes in
 * ascending order with strict '<' (ties -> lower code), sign from v < 0,
 * signed zero kept, non-finite -> NaN code by sign bit. */
uint8_t or_e4m3_encode(float v) {
  if (!isfinite(v)) return signbit(v) ? 0xFFu : 0x7Fu;
  float a = fabsf(v);
  if (a == 0.0f) return signbit(v) ? 0x80u : 0x00u;
  int best = 0;
  float best_err = INFINITY;
  for (int c = 0; c < 128; ++c) {
    if (c == 0x7F) continue;
    float err = fabsf(a - or_e4m3_decode((uint8_t)c));
    if (err < best_err) { best_err = err; best = c; }
  }
  uint8_t out = (uint8_t)best;
  if (v < 0.0f) out |= 0x80u;
  return out;
}

/* ------------------------------------------------------------------------ */
/* INT4 nibble (pack.hpp:381-390) and bf16                                   */
/* ------------------------------------------------------------------------ */

int or_int4_from_nibble(uint8_t n) { n &= 0xF; return (n & 8) ? (int)n - 16 : (int)n; }
uint8_t or_int4_to_nibble(int v) {
  if (v < -8) v = -8;
  if (v > 7) v = 7;
  return (uint8_t)(v & 0xF);
}

uint16_t or_f32_to_bf16_bits(float f) {
  uint32_t u = f2u(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
float or_bf16_bits_to_f32(uint16_t b) { return u2f((uint32_t)b << 16); }

void or_e2m1_encode_n(const float* v, uint8_t* o, size_t n) { for (size_t i = 0; i < n; ++i) o[i] = or_e2m1_encode(v[i]); }
void or_e8m0_encode_n(const float* v, uint8_t* o, size_t n) { for (size_t i = 0; i < n; ++i) o[i] = or_e8m0_encode(v[i]); }
void or_e4m3_encode_n(const float* v, uint8_t* o, size_t n) { for (size_t i = 0; i < n; ++i) o[i] = or_e4m3_encode(v[i]); }
void or_fp16_encode_n(const float* v, uint16_t* o, size_t n) { for (size_t i = 0; i < n; ++i) o[i] = or_float_to_fp16_bits(v[i]); }

/* ------------------------------------------------------------------------ */
/* Packers                                                                   */
/* ------------------------------------------------------------------------ */

/* std::max(a, b) as the reference uses it: (a < b) ? b : a (NaN b ignored). */
static inline float ref_max(float a, float b) { return (a < b) ? b : a; }

/* static_cast<int>(float) on x86-64 (cvttss2si): NaN and values outside
 * [-2^31, 2^31) give INT32_MIN. */
static inline int x86_f2i(float r) {
  if (!(r >= -2147483648.0f && r < 2147483648.0f)) return (int)0x80000000u;
  return (int)r;
}

static inline void put_nibble(uint8_t* data, size_t lin, uint8_t nib) {
  /* pack.hpp:159-169: even linear index -> low nibble, odd -> high nibble */
  uint8_t* b = &data[lin >> 1];
  if ((lin & 1u) == 0) *b = (uint8_t)((*b & 0xF0u) | (nib & 0xFu));
  else *b = (uint8_t)((*b & 0x0Fu) | ((nib & 0xFu) << 4));
}

/* pack.hpp:424-462 */
int or_pack_int4(const float* W, size_t N, size_t K, int group, uint8_t* data,
                 uint16_t* scales) {
  if (group != 64 && group != 128) return OR_EINVAL;
  if (K % (size_t)group != 0 || ((N * K) & 1u)) return OR_EINVAL;
  memset(data, 0, N * K / 2);
  size_t gpr = K / (size_t)group;
  for (size_t n = 0; n < N; ++n)
    for (size_t g = 0; g < gpr; ++g) {
      const float* w = W + n * K + g * (size_t)group;
      float amax = 0.0f;
      for (int t = 0; t < group; ++t) amax = ref_max(amax, fabsf(w[t]));
      float scale = (amax > 0.0f) ? (amax / 7.0f) : 1.0f;
      scales[n * gpr + g] = or_float_to_fp16_bits(scale);
      float inv = 1.0f / scale;
      for (int t = 0; t < group; ++t) {
        int q = x86_f2i(nearbyintf(w[t] * inv));
        if (q < -8) q = -8;
        if (q > 7) q = 7;
        put_nibble(data, n * K + g * (size_t)group + (size_t)t, or_int4_to_nibble(q));
      }
    }
  return OR_OK;
}

/* pack.hpp:465-497 */
int or_pack_mxfp4(const float* W, size_t N, size_t K, uint8_t* data,
                  uint8_t* scales) {
  if (K % 32 != 0) return OR_EINVAL;
  memset(data, 0, N * K / 2);
  size_t blocks = K / 32;
  for (size_t n = 0; n < N; ++n)
    for (size_t b = 0; b < blocks; ++b) {
      const float* w = W + n * K + b * 32;
      float amax = 0.0f;
      for (int t = 0; t < 32; ++t) amax = ref_max(amax, fabsf(w[t]));
      float target = (amax > 0.0f) ? (amax / 6.0f) : or_e8m0_decode(127);
      uint8_t sb = or_e8m0_encode(target);
      scales[n * blocks + b] = sb;
      float inv = 1.0f / or_e8m0_decode(sb);
      for (int t = 0; t < 32; ++t)
        put_nibble(data, n * K + b * 32 + (size_t)t, or_e2m1_encode(w[t] * inv));
    }
  return OR_OK;
}

/* pack.hpp:502-542 */
int or_pack_nvfp4(const float* W, size_t N, size_t K, float tensor_scale,
                  uint8_t* data, uint8_t* scales) {
  if (K % 16 != 0) return OR_EINVAL;
  if (!(tensor_scale > 0.0f) || !isfinite(tensor_scale)) return OR_EINVAL;
  memset(data, 0, N * K / 2);
  float inv_t = 1.0f / tensor_scale;
  size_t blocks = K / 16;
  for (size_t n = 0; n < N; ++n)
    for (size_t b = 0; b < blocks; ++b) {
      const float* w = W + n * K + b * 16;
      float amax = 0.0f;
      for (int t = 0; t < 16; ++t) amax = ref_max(amax, fabsf(w[t] * inv_t));
      float target = (amax > 0.0f) ? (amax / 6.0f) : 1.0f;
      uint8_t sb = or_e4m3_encode(target);
      scales[n * blocks + b] = sb;
      float s = or_e4m3_decode(sb);
      float inv = (s != 0.0f && isfinite(s)) ? (1.0f / s) : 0.0f;
      for (int t = 0; t < 16; ++t)
        put_nibble(data, n * K + b * 16 + (size_t)t, or_e2m1_encode(w[t] * inv_t * inv));
    }
  return OR_OK;
}

float or_nvfp4_tensor_scale(const float* W, size_t n) {
  float amax = 0.0f;
  for (size_t i = 0; i < n; ++i) amax = ref_max(amax, fabsf(W[i]));
  return amax / 2688.0f; /* 448 * 6 */
}

/* ------------------------------------------------------------------------ */
/* Dequantisers (pack.hpp:548-585)                                           */
/* ------------------------------------------------------------------------ */

static inline uint8_t get_nibble(const uint8_t* d, size_t lin) {
  uint8_t b = d[lin >> 1];
  return (lin & 1u) ? (uint8_t)(b >> 4) : (uint8_t)(b & 0xFu);
}

static void dq_rows(int fmt, const uint8_t* data, const void* scales, size_t K,
                    int group, float ts, size_t n0, size_t n1, float* out) {
  for (size_t n = n0; n < n1; ++n) {
    float* o = out + (n - n0) * K;
    if (fmt == 0) {
      const uint8_t* sc = (const uint8_t*)scales + n * (K / 32);
      for (size_t k = 0; k < K; ++k)
        o[k] = or_e2m1_decode(get_nibble(data, n * K + k)) * or_e8m0_decode(sc[k / 32]);
    } else if (fmt == 1) {
      const uint8_t* sc = (const uint8_t*)scales + n * (K / 16);
      for (size_t k = 0; k < K; ++k)
        o[k] = or_e2m1_decode(get_nibble(data, n * K + k)) * or_e4m3_decode(sc[k / 16]) * ts;
    } else {
      const uint16_t* sc = (const uint16_t*)scales + n * (K / (size_t)group);
      for (size_t k = 0; k < K; ++k)
        o[k] = (float)or_int4_from_nibble(get_nibble(data, n * K + k)) *
               or_fp16_bits_to_float(sc[k / (size_t)group]);
    }
  }
}

void or_dequant_int4(const uint8_t* d, const uint16_t* s, size_t N, size_t K, int g, float* out) { dq_rows(2, d, s, K, g, 1.0f, 0, N, out); }
void or_dequant_mxfp4(const uint8_t* d, const uint8_t* s, size_t N, size_t K, float* out) { dq_rows(0, d, s, K, 32, 1.0f, 0, N, out); }
void or_dequant_nvfp4(const uint8_t* d, const uint8_t* s, size_t N, size_t K, float ts, float* out) { dq_rows(1, d, s, K, 16, ts, 0, N, out); }

/* ------------------------------------------------------------------------ */
/* Reference GEMM (ref_gemm.hpp:15-27)                                       */
/* ------------------------------------------------------------------------ */

void or_gemm_ref(const float* X, const float* W, float* Y, size_t M, size_t N, size_t K) {
  for (size_t m = 0; m < M; ++m)
    for (size_t n = 0; n < N; ++n) {
      double acc = 0.0;
      for (size_t k = 0; k < K; ++k) acc += (double)X[m * K + k] * (double)W[n * K + k];
      Y[m * N + n] = (float)acc;
    }
}

/* Threaded "dequant a row slice, then the reference GEMM over it". */
typedef struct {
  int fmt; const uint8_t* data; const void* scales; size_t N, K; int group; float ts;
  const float* Xf; size_t M; float* Y; size_t n0, n1;
} or_job_t;

static void* or_job_run(void* p) {
  or_job_t* j = (or_job_t*)p;
  const size_t R = 16; /* rows dequantised at a time */
  float* wbuf = (float*)malloc(R * j->K * sizeof(float));
  if (!wbuf) return (void*)1;
  for (size_t n = j->n0; n < j->n1; n += R) {
    size_t e = n + R < j->n1 ? n + R : j->n1;
    dq_rows(j->fmt, j->data, j->scales, j->K, j->group, j->ts, n, e, wbuf);
    for (size_t m = 0; m < j->M; ++m) {
      const float* x = j->Xf + m * j->K;
      for (size_t r = n; r < e; ++r) {
        const float* w = wbuf + (r - n) * j->K;
        double acc = 0.0;
        for (size_t k = 0; k < j->K; ++k) acc += (double)x[k] * (double)w[k];
        j->Y[m * j->N + r] = (float)acc;
      }
    }
  }
  free(wbuf);
  return NULL;
}

int or_w4a16_gemm(int fmt, const uint8_t* data, const void* scales, size_t N, size_t K,
                  int group, float tensor_scale, const uint16_t* X_bf16, size_t M,
                  float* Y, size_t n_begin, size_t n_end, int nthreads) {
  int blk = fmt == 0 ? 32 : fmt == 1 ? 16 : group;
  if (fmt < 0 || fmt > 2 || blk <= 0 || K % (size_t)blk || n_end > N || n_begin > n_end)
    return OR_EINVAL;
  if (nthreads < 1) nthreads = 1;
  float* Xf = (float*)malloc(M * K * sizeof(float));
  if (!Xf) return OR_EINVAL;
  for (size_t i = 0; i < M * K; ++i) Xf[i] = or_bf16_bits_to_f32(X_bf16[i]);
  pthread_t th[256];
  or_job_t jobs[256];
  if (nthreads > 256) nthreads = 256;
  size_t rows = n_end - n_begin, per = (rows + (size_t)nthreads - 1) / (size_t)nthreads;
  int launched = 0;
  for (int t = 0; t < nthreads; ++t) {
    size_t a = n_begin + (size_t)t * per, b = a + per;
    if (a >= n_end) break;
    if (b > n_end) b = n_end;
    jobs[t] = (or_job_t){fmt, data, scales, N, K, group, tensor_scale, Xf, M, Y, a, b};
    if (pthread_create(&th[t], NULL, or_job_run, &jobs[t]) != 0) { or_job_run(&jobs[t]); continue; }
    ++launched;
    (void)launched;
  }
  for (int t = 0; t < nthreads; ++t) {
    size_t a = n_begin + (size_t)t * per;
    if (a >= n_end) break;
    pthread_join(th[t], NULL);
  }
  free(Xf);
  return OR_OK;
}

/* ------------------------------------------------------------------------ */
/* Seeded generator: splitmix64 -> xoshiro256**, Box-Muller                 */
/* ------------------------------------------------------------------------ */

static inline uint64_t splitmix64(uint64_t* s) {
  uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
static inline uint64_t rotl64(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }
typedef struct { uint64_t s[4]; } xo_t;
static inline uint64_t xo_next(xo_t* r) {
  uint64_t* s = r->s;
  uint64_t res = rotl64(s[1] * 5, 7) * 9, t = s[1] << 17;
  s[2] ^= s[0]; s[3] ^= s[1]; s[1] ^= s[2]; s[0] ^= s[3]; s[2] ^= t; s[3] = rotl64(s[3], 45);
  return res;
}
static void xo_seed(xo_t* r, uint64_t seed, uint64_t stream) {
  uint64_t sm = seed ^ (stream * 0xD1B54A32D192ED03ull);
  for (int i = 0; i < 4; ++i) r->s[i] = splitmix64(&sm);
}

/* Pair i of the stream: z0 = r cos(2 pi u2), z1 = r sin(2 pi u2), computed in
 * double and rounded once to float. */
static inline void bm_pair(xo_t* r, float mean, float std, float* z0, float* z1) {
  const double two_pi = 6.283185307179586476925286766559;
  double u1 = ((double)(xo_next(r) >> 11) + 0.5) * 0x1.0p-53;
  double u2 = ((double)(xo_next(r) >> 11) + 0.5) * 0x1.0p-53;
  double rad = sqrt(-2.0 * log(u1));
  *z0 = (float)((double)mean + (double)std * rad * cos(two_pi * u2));
  *z1 = (float)((double)mean + (double)std * rad * sin(two_pi * u2));
}

void or_randn(uint64_t seed, uint64_t stream, float mean, float std, float* out, size_t n) {
  xo_t r;
  xo_seed(&r, seed, stream);
  for (size_t i = 0; i < n; i += 2) {
    float a, b;
    bm_pair(&r, mean, std, &a, &b);
    out[i] = a;
    if (i + 1 < n) out[i + 1] = b;
  }
}

void or_randn_bf16(uint64_t seed, uint64_t stream, float mean, float std, uint16_t* out, size_t n) {
  xo_t r;
  xo_seed(&r, seed, stream);
  for (size_t i = 0; i < n; i += 2) {
    float a, b;
    bm_pair(&r, mean, std, &a, &b);
    out[i] = or_f32_to_bf16_bits(a);
    if (i + 1 < n) out[i + 1] = or_f32_to_bf16_bits(b);
  }
}
