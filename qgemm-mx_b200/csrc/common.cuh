// common.cuh -- shared host helpers and exact device codecs.
//
// The device codecs restate the decision rules of titoatwork/qgemm-mx
// include/qgemm/pack.hpp:183-390 so that device packing is bit-identical to
// the host packer.  sm_100a's cvt.*.e2m1x2 / e4m3x2 instructions round to
// nearest-even, while the reference breaks ties toward the smaller magnitude
// (first minimum of a float-rounded |a - t| search), so packing uses explicit
// searches instead.  Everything is compiled without fast-math: IEEE division,
// reciprocal and subnormals are required for parity.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/qgemm_b200.h"

namespace qg {

// ---------------------------------------------------------------------------
// Host-side status plumbing
// ---------------------------------------------------------------------------

void set_error(const char* fmt, ...);
qgemm_status_t fail(qgemm_status_t s, const char* fmt, ...);

#define QG_CUDA_RET(expr)                                                     \
  do {                                                                        \
    cudaError_t _e = (expr);                                                  \
    if (_e != cudaSuccess)                                                    \
      return ::qg::fail(QGEMM_ERR_CUDA, "%s:%d %s -> %s", __FILE__, __LINE__, \
                        #expr, cudaGetErrorString(_e));                       \
  } while (0)

// Check the launch that was just issued (does not synchronise).
#define QG_LAUNCH_RET()                                                       \
  do {                                                                        \
    cudaError_t _e = cudaGetLastError();                                      \
    if (_e != cudaSuccess)                                                    \
      return ::qg::fail(QGEMM_ERR_CUDA, "%s:%d launch failed: %s", __FILE__,  \
                        __LINE__, cudaGetErrorString(_e));                    \
  } while (0)

inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

struct DevProps {
  int sm_count = 0;
  size_t l2_bytes = 0;
};
qgemm_status_t device_props(DevProps* p);

// Every GEMM workspace starts with the split-tile tickets of whichever kernel
// a call runs, in a region sized from N alone: the largest ticket count of
// any path (the grouped decode kernel's 32 problems x N/128 tiles, the
// LDG-fed decode kernel's N/32 tiles, at least 512 for the tile-per-CTA
// tcgen05 kernel's split tiles).  Each call returns its tickets to zero and
// keeps its other scratch behind the region, so calls of any M, grouped
// calls included, can share one workspace.
size_t ws_ticket_bytes(size_t N);

// Layout checks shared by the entry points (null if fine, else a message).
inline const char* layout_error(const qgemm_weights_t* w) {
  if (w->layout == QGEMM_LAYOUT_CANONICAL) return nullptr;
  if (w->layout != QGEMM_LAYOUT_SCALE_CHECKED) return "unknown layout";
  if (w->format != QGEMM_FMT_MXFP4 && w->format != QGEMM_FMT_NVFP4)
    return "the scale-checked layout is MXFP4 / NVFP4 only";
  return nullptr;
}

// ---------------------------------------------------------------------------
// Bit helpers
// ---------------------------------------------------------------------------

__host__ __device__ __forceinline__ uint32_t f2u(float f) {
#ifdef __CUDA_ARCH__
  return __float_as_uint(f);
#else
  uint32_t u; std::memcpy(&u, &f, 4); return u;
#endif
}
__host__ __device__ __forceinline__ float u2f(uint32_t u) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(u);
#else
  float f; std::memcpy(&f, &u, 4); return f;
#endif
}

// ---------------------------------------------------------------------------
// Device codecs (exact)
// ---------------------------------------------------------------------------

// E2M1 magnitudes, ascending (pack.hpp:260-262).
__device__ __forceinline__ float e2m1_mag(int i) {
  switch (i) {
    case 0: return 0.0f; case 1: return 0.5f; case 2: return 1.0f; case 3: return 1.5f;
    case 4: return 2.0f; case 5: return 3.0f; case 6: return 4.0f; default: return 6.0f;
  }
}

__device__ __forceinline__ float e2m1_decode(uint32_t code) {
  float m = e2m1_mag(code & 7u);
  return (code & 8u) ? -m : m;
}

// Rule of pack.hpp:272-293: scan magnitudes in ascending order keeping the
// first smallest float-rounded |a - t|; zero drops the sign; non-finite goes
// to +-6 by sign bit.  Unrolled so the candidates are immediates.
__device__ __forceinline__ uint32_t e2m1_encode(float v) {
  if (!isfinite(v)) return signbit(v) ? 0xFu : 0x7u;
  const float a = fabsf(v);
  uint32_t best = 0;
  float be = fabsf(a - 0.0f);
#pragma unroll
  for (int i = 1; i < 8; ++i) {
    const float e = fabsf(a - e2m1_mag(i));
    if (e < be) { be = e; best = (uint32_t)i; }
  }
  if (best != 0 && signbit(v)) best |= 8u;
  return best;
}

// 2^(bits-127), 0xFF = NaN (pack.hpp:299-305).  Built from bits: exact.
__device__ __forceinline__ float e8m0_decode(uint32_t bits) {
  bits &= 0xFFu;
  if (bits == 0xFFu) return u2f(0x7FC00000u);
  if (bits == 0) return u2f(0x00400000u);  // 2^-127, subnormal
  return u2f(bits << 23);
}

// Rule of pack.hpp:308-327 written on the exponent field: with
// scale = m * 2^e (m in [0.5,1), frexp convention) the result is 2^e when
// m >= 0.70710678f, else 2^(e-1); m >= 0.70710678f  <=>  the 23-bit fraction
// of the normalised significand is >= 0x3504F3 (0.70710678f = 0x3F3504F3).
__device__ __forceinline__ uint32_t e8m0_encode(float s) {
  if (!isfinite(s)) return 0xFFu;
  if (s <= 0.0f) return 0u;
  uint32_t u = f2u(s);
  int ef = (int)(u >> 23);
  uint32_t frac = u & 0x7FFFFFu;
  int e;  // frexp exponent
  if (ef != 0) {
    e = ef - 126;
  } else {  // subnormal: normalise
    int p = 31 - __clz((int)frac);       // position of the leading one (0..22)
    e = p - 148;
    frac = (frac << (23 - p)) & 0x7FFFFFu;
  }
  int pw = (frac >= 0x3504F3u) ? e : e - 1;
  int bits = pw + 127;
  bits = bits < 0 ? 0 : (bits > 254 ? 254 : bits);
  return (uint32_t)bits;
}

// E4M3 decode (pack.hpp:333-350), from bits.
__device__ __forceinline__ float e4m3_decode(uint32_t bits) {
  const uint32_t s = (bits >> 7) & 1u, e = (bits >> 3) & 0xFu, m = bits & 7u;
  if (e == 0xFu && m == 7u) return u2f(0x7FC00000u);
  float mag = (e == 0) ? (float)m * 0.001953125f  // m * 2^-9, exact
                       : u2f(((e + 120u) << 23) | (m << 20));
  return s ? -mag : mag;
}

// IEEE half bits -> float (pack.hpp:183-211); exact.
__device__ __forceinline__ float fp16_bits_to_float(uint32_t h) {
  const uint32_t s = (h >> 15) & 1u, e = (h >> 10) & 0x1Fu;
  uint32_t m = h & 0x3FFu;
  uint32_t out;
  if (e == 0) {
    if (m == 0) {
      out = s << 31;
    } else {
      const int p = 31 - __clz((int)m);  // leading one, 0..9
      out = (s << 31) | ((uint32_t)(p + 103) << 23) | ((m << (23 - p)) & 0x7FFFFFu);
    }
  } else if (e == 31) {
    out = (s << 31) | 0x7F800000u | (m << 13);
  } else {
    out = (s << 31) | ((e + 112u) << 23) | (m << 13);
  }
  return u2f(out);
}

// float -> IEEE half bits with the rounding and special cases of
// pack.hpp:213-253 (RNE; NaN -> 0x7C00|0x200; below 2^-25 -> signed zero).
__device__ __forceinline__ uint32_t float_to_fp16_bits(float f) {
  const uint32_t x = f2u(f);
  const uint32_t sign = (x >> 16) & 0x8000u;
  int exp = (int)((x >> 23) & 0xFFu) - 112;
  uint32_t mant = x & 0x7FFFFFu;
  if (((x >> 23) & 0xFFu) == 0xFFu) return sign | 0x7C00u | (mant ? 0x200u : 0u);
  if (exp <= 0) {
    if (exp < -10) return sign;
    mant |= 0x800000u;
    const uint32_t shift = (uint32_t)(14 - exp);
    uint32_t hm = mant >> shift;
    const uint32_t rem = mant & ((1u << shift) - 1u), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (hm & 1u))) ++hm;
    return sign | hm;
  }
  if (exp >= 31) return sign | 0x7C00u;
  uint32_t hm = mant >> 13;
  const uint32_t rem = mant & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (hm & 1u))) {
    if (++hm == 0x400u) {
      hm = 0;
      if (++exp >= 31) return sign | 0x7C00u;
    }
  }
  return sign | ((uint32_t)exp << 10) | hm;
}

__device__ __forceinline__ int int4_from_nibble(uint32_t n) {
  n &= 0xFu;
  return (n & 8u) ? (int)n - 16 : (int)n;
}

// static_cast<int>(float) as compiled for x86-64 (cvttss2si): NaN and values
// outside [-2^31, 2^31) give INT32_MIN.  The reference relies on this in
// pack_int4 when a group's scale underflows or overflows.
__device__ __forceinline__ int x86_float_to_int(float r) {
  if (!(r >= -2147483648.0f && r < 2147483648.0f)) return (int)0x80000000u;
  return (int)r;
}

// std::max(a, b) as the reference calls it: (a < b) ? b : a.
__device__ __forceinline__ float ref_max(float a, float b) { return (a < b) ? b : a; }

}  // namespace qg
