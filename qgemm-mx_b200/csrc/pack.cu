// pack.cu -- device quantize+pack, dequant and codec kernels, bit-exact to
// titoatwork/qgemm-mx include/qgemm/pack.hpp.
//
// Layout (pack.hpp:14-25): element (n,k) has linear index n*K+k; byte i holds
// elements 2i (low nibble) and 2i+1 (high nibble); scales are a separate
// array indexed n*(K/block)+k/block.  One thread handles 8 consecutive
// elements (= one 32-bit word of packed output); a scale block of B elements
// is handled by B/8 adjacent lanes that combine their |w| maxima with warp
// shuffles.  All kernels are grid-stride and HBM-bound (4 B read per element,
// 0.5 B + scale written).
#include <cstdarg>
#include <cstring>

#include "common.cuh"

namespace qg {

// E4M3 positive values by code, 0..126 (pack.hpp:333-350).
constexpr float e4m3_pos_value(int c) {
  int e = (c >> 3) & 0xF, m = c & 7;
  if (e == 0) return (float)m * 0.001953125f;
  float v = 1.0f + (float)m * 0.125f;
  for (int i = 7; i < e; ++i) v *= 2.0f;
  for (int i = e; i < 7; ++i) v *= 0.5f;
  return v;
}
#define QG_E4(c) e4m3_pos_value(c)
#define QG_E4x8(b) QG_E4(b), QG_E4(b + 1), QG_E4(b + 2), QG_E4(b + 3), QG_E4(b + 4), QG_E4(b + 5), QG_E4(b + 6), QG_E4(b + 7)
__constant__ float c_e4m3_pos[128] = {
    QG_E4x8(0),  QG_E4x8(8),  QG_E4x8(16), QG_E4x8(24), QG_E4x8(32),  QG_E4x8(40),
    QG_E4x8(48), QG_E4x8(56), QG_E4x8(64), QG_E4x8(72), QG_E4x8(80),  QG_E4x8(88),
    QG_E4x8(96), QG_E4x8(104), QG_E4x8(112), QG_E4x8(120)};
#undef QG_E4x8
#undef QG_E4

// Rule of pack.hpp:352-374: ascending scan over the 127 finite positive codes
// keeping the first smallest float-rounded |a - value|.
__device__ __forceinline__ uint32_t e4m3_encode(float v) {
  if (!isfinite(v)) return signbit(v) ? 0xFFu : 0x7Fu;
  const float a = fabsf(v);
  if (a == 0.0f) return signbit(v) ? 0x80u : 0x00u;
  uint32_t best = 0;
  float be = __int_as_float(0x7F800000);
#pragma unroll 8
  for (int c = 0; c < 127; ++c) {
    const float e = fabsf(a - c_e4m3_pos[c]);
    if (e < be) { be = e; best = (uint32_t)c; }
  }
  if (v < 0.0f) best |= 0x80u;
  return best;
}


// ---------------------------------------------------------------------------
// Host status plumbing
// ---------------------------------------------------------------------------

static thread_local char t_msg[512] = {0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(t_msg, sizeof(t_msg), fmt, ap);
  va_end(ap);
}

qgemm_status_t fail(qgemm_status_t s, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(t_msg, sizeof(t_msg), fmt, ap);
  va_end(ap);
  return s;
}

qgemm_status_t device_props(DevProps* p) {
  static thread_local int cached_dev = -1;
  static thread_local DevProps cached;
  int dev = 0;
  QG_CUDA_RET(cudaGetDevice(&dev));
  if (dev != cached_dev) {
    int sms = 0, l2 = 0;
    QG_CUDA_RET(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    QG_CUDA_RET(cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, dev));
    cached.sm_count = sms;
    cached.l2_bytes = (size_t)l2;
    cached_dev = dev;
  }
  *p = cached;
  return QGEMM_OK;
}

static const char* t_msg_get() { return t_msg; }

// ---------------------------------------------------------------------------
// Element loads: 8 consecutive floats starting at element index e (multiple
// of 8).  VEC uses two 16-byte loads and needs a 16-byte aligned W.
// ---------------------------------------------------------------------------

template <bool VEC>
__device__ __forceinline__ void load8(const float* __restrict__ W, size_t e, float (&w)[8]) {
  if (VEC) {
    const float4* p = reinterpret_cast<const float4*>(W + e);
    float4 a = __ldcs(p), b = __ldcs(p + 1);  // streamed once
    w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
    w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
  } else {
#pragma unroll
    for (int t = 0; t < 8; ++t) w[t] = W[e + t];
  }
}

// ---------------------------------------------------------------------------
// MXFP4 (pack.hpp:465-497): 4 lanes per 32-element block.
// ---------------------------------------------------------------------------

template <bool VEC>
__global__ void __launch_bounds__(256) k_pack_mxfp4(const float* __restrict__ W, size_t octets,
                                                    uint32_t* __restrict__ data,
                                                    uint8_t* __restrict__ scales) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t base = (size_t)blockIdx.x * blockDim.x; base < octets; base += stride) {
    const size_t o = base + threadIdx.x;
    const bool live = o < octets;
    float w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (live) load8<VEC>(W, o * 8, w);
    float amax = 0.0f;
#pragma unroll
    for (int t = 0; t < 8; ++t) amax = ref_max(amax, fabsf(w[t]));
    amax = ref_max(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 1));
    amax = ref_max(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 2));
    if (!live) continue;
    const float target = (amax > 0.0f) ? (amax / 6.0f) : 1.0f;
    const uint32_t sb = e8m0_encode(target);
    const float inv = 1.0f / e8m0_decode(sb);
    uint32_t word = 0;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const float x = w[t] * inv;
      uint32_t c;
      if (isnan(x)) {
        // x86 multiply returns a NaN operand unchanged: W's own NaN keeps its
        // sign; otherwise the NaN is the (positive) decoded 0xFF scale.
        c = (isnan(w[t]) && signbit(w[t])) ? 0xFu : 0x7u;
      } else {
        c = e2m1_encode(x);
      }
      word |= c << (4 * t);
    }
    data[o] = word;
    if ((o & 3) == 0) scales[o >> 2] = (uint8_t)sb;
  }
}

// ---------------------------------------------------------------------------
// NVFP4 (pack.hpp:502-542): 2 lanes per 16-element block.  The two lanes of
// a block split the 127-code E4M3 search (lane 0: codes 0..63, lane 1:
// 64..126); the lower-code lane wins ties, which is the reference's
// first-minimum rule.
// ---------------------------------------------------------------------------

template <bool VEC>
__global__ void __launch_bounds__(256) k_pack_nvfp4(const float* __restrict__ W, size_t octets,
                                                    float inv_t, uint32_t* __restrict__ data,
                                                    uint8_t* __restrict__ scales) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  const int half = threadIdx.x & 1;
  for (size_t base = (size_t)blockIdx.x * blockDim.x; base < octets; base += stride) {
    const size_t o = base + threadIdx.x;
    const bool live = o < octets;
    float w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (live) load8<VEC>(W, o * 8, w);
    float amax = 0.0f;
#pragma unroll
    for (int t = 0; t < 8; ++t) amax = ref_max(amax, fabsf(w[t] * inv_t));
    amax = ref_max(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 1));
    const float target = (amax > 0.0f) ? (amax / 6.0f) : 1.0f;
    // split first-minimum search over the positive codes
    uint32_t best;
    {
      const float a = fabsf(target);
      float be = __int_as_float(0x7F800000);
      uint32_t bc = 0;
      const int c0 = half ? 64 : 0, c1 = half ? 127 : 64;
      for (int c = c0; c < c1; ++c) {
        const float e = fabsf(a - c_e4m3_pos[c]);
        if (e < be) { be = e; bc = (uint32_t)c; }
      }
      const float obe = __shfl_xor_sync(0xFFFFFFFFu, be, 1);
      const uint32_t obc = __shfl_xor_sync(0xFFFFFFFFu, bc, 1);
      // lane 0 holds the lower codes: the other half wins only if strictly less
      if (half == 0) best = (obe < be) ? obc : bc;
      else best = (be < obe) ? bc : obc;
    }
    if (!live) continue;
    // target is finite and >= 0 except when amax is +inf: e4m3_encode rules.
    uint32_t sb;
    if (!isfinite(target)) sb = 0x7Fu;           // +inf -> NaN code
    else if (target == 0.0f) sb = 0x00u;         // +0
    else sb = best;                              // target > 0: no sign bit
    const float s = e4m3_decode(sb);
    const float inv = (s != 0.0f && isfinite(s)) ? (1.0f / s) : 0.0f;
    uint32_t word = 0;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const float y = w[t] * inv_t;
      const float x = y * inv;
      uint32_t c;
      if (isnan(x)) {
        // x86: a NaN operand propagates with its sign; an invalid operation
        // (inf*0) yields the default NaN, which has the sign bit set.
        const bool neg = isnan(y) ? (isnan(w[t]) ? (bool)signbit(w[t]) : true) : true;
        c = neg ? 0xFu : 0x7u;
      } else {
        c = e2m1_encode(x);
      }
      word |= c << (4 * t);
    }
    data[o] = word;
    if ((o & 1) == 0) scales[o >> 1] = (uint8_t)sb;
  }
}

// ---------------------------------------------------------------------------
// INT4 (pack.hpp:424-462): G/8 lanes per group (G = 64 or 128).
// ---------------------------------------------------------------------------

template <bool VEC, int G>
__global__ void __launch_bounds__(256) k_pack_int4(const float* __restrict__ W, size_t octets,
                                                   uint32_t* __restrict__ data,
                                                   uint16_t* __restrict__ scales) {
  constexpr int LANES = G / 8;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t base = (size_t)blockIdx.x * blockDim.x; base < octets; base += stride) {
    const size_t o = base + threadIdx.x;
    const bool live = o < octets;
    float w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (live) load8<VEC>(W, o * 8, w);
    float amax = 0.0f;
#pragma unroll
    for (int t = 0; t < 8; ++t) amax = ref_max(amax, fabsf(w[t]));
#pragma unroll
    for (int d = 1; d < LANES; d <<= 1) amax = ref_max(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, d));
    if (!live) continue;
    const float scale = (amax > 0.0f) ? (amax / 7.0f) : 1.0f;
    const float inv = 1.0f / scale;
    uint32_t word = 0;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      int q = x86_float_to_int(rintf(w[t] * inv));
      q = q < -8 ? -8 : (q > 7 ? 7 : q);
      word |= ((uint32_t)q & 0xFu) << (4 * t);
    }
    data[o] = word;
    if ((o & (LANES - 1)) == 0) scales[o / LANES] = (uint16_t)float_to_fp16_bits(scale);
  }
}

// ---------------------------------------------------------------------------
// NVFP4 tensor scale: max|W| (NaN skipped, as std::max does) / (448*6).
// Non-negative float bit patterns order like the floats, so an unsigned
// atomicMax over the bits is an exact max.
// ---------------------------------------------------------------------------

__global__ void k_amax(const float* __restrict__ W, size_t n, unsigned* __restrict__ out) {
  float m = 0.0f;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    m = ref_max(m, fabsf(W[i]));
#pragma unroll
  for (int d = 16; d; d >>= 1) m = ref_max(m, __shfl_xor_sync(0xFFFFFFFFu, m, d));
  if ((threadIdx.x & 31) == 0 && m > 0.0f) atomicMax(out, f2u(m));
}

__global__ void k_amax_finish(float* out) { out[0] = u2f(f2u(out[0])) / 2688.0f; }

// ---------------------------------------------------------------------------
// Dequant (pack.hpp:548-585): one thread per packed 32-bit word.
// ---------------------------------------------------------------------------

template <int FMT>  // 0 MXFP4, 1 NVFP4, 2 INT4
__global__ void __launch_bounds__(256) k_dequant(const uint32_t* __restrict__ data,
                                                 const void* __restrict__ scales, size_t octets,
                                                 size_t K, int group, float ts,
                                                 float* __restrict__ out) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t o = (size_t)blockIdx.x * blockDim.x + threadIdx.x; o < octets; o += stride) {
    const uint32_t word = data[o];
    const size_t e = o * 8, n = e / K, k = e % K;
    float v[8];
    if (FMT == 0) {
      const float s = e8m0_decode(static_cast<const uint8_t*>(scales)[n * (K / 32) + k / 32]);
#pragma unroll
      for (int t = 0; t < 8; ++t) v[t] = e2m1_decode(word >> (4 * t)) * s;
    } else if (FMT == 1) {
      const float s = e4m3_decode(static_cast<const uint8_t*>(scales)[n * (K / 16) + k / 16]);
#pragma unroll
      for (int t = 0; t < 8; ++t) v[t] = (e2m1_decode(word >> (4 * t)) * s) * ts;
    } else {
      const float s = fp16_bits_to_float(static_cast<const uint16_t*>(scales)[n * (K / group) + k / group]);
#pragma unroll
      for (int t = 0; t < 8; ++t) v[t] = (float)int4_from_nibble(word >> (4 * t)) * s;
    }
    float4* p = reinterpret_cast<float4*>(out + e);
    p[0] = make_float4(v[0], v[1], v[2], v[3]);
    p[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
}

// ---------------------------------------------------------------------------
// Element-wise codecs (tests and tools).
// ---------------------------------------------------------------------------

__global__ void k_codec(int kind, const float* __restrict__ in, void* __restrict__ out, size_t n) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float v = in[i];
    switch (kind) {
      case 0: static_cast<uint8_t*>(out)[i] = (uint8_t)e2m1_encode(v); break;
      case 1: static_cast<uint8_t*>(out)[i] = (uint8_t)e8m0_encode(v); break;
      case 2: static_cast<uint8_t*>(out)[i] = (uint8_t)e4m3_encode(v); break;
      default: static_cast<uint16_t*>(out)[i] = (uint16_t)float_to_fp16_bits(v); break;
    }
  }
}

// ---------------------------------------------------------------------------
// Code-level packing (pack.hpp:611-674): already-quantised codes to the
// canonical layout and back.  One thread per output byte pair of codes;
// even linear index in the low nibble (pack_nibble, pack.hpp:159-168).
// FP4 codes keep their low 4 bits; INT4 codes are clamped to [-8, 7] and
// stored two's complement (int4_to_nibble, pack.hpp:386-390).
// ---------------------------------------------------------------------------

__global__ void k_pack_codes(int int4, const void* __restrict__ codes, uint8_t* __restrict__ data, size_t nbytes) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < nbytes; i += stride) {
    uint32_t lo, hi;
    if (int4) {
      const int* q = static_cast<const int*>(codes);
      const int a = min(max(q[2 * i], -8), 7), b = min(max(q[2 * i + 1], -8), 7);
      lo = (uint32_t)a & 0xFu;
      hi = (uint32_t)b & 0xFu;
    } else {
      const uint8_t* c = static_cast<const uint8_t*>(codes);
      lo = c[2 * i] & 0xFu;
      hi = c[2 * i + 1] & 0xFu;
    }
    data[i] = (uint8_t)(lo | (hi << 4));
  }
}

__global__ void k_unpack_codes(int int4, const uint8_t* __restrict__ data, void* __restrict__ codes, size_t nbytes) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < nbytes; i += stride) {
    const uint32_t b = data[i];
    if (int4) {
      int* q = static_cast<int*>(codes);
      q[2 * i] = int4_from_nibble(b & 0xFu);  // int4_from_nibble, pack.hpp:381-384
      q[2 * i + 1] = int4_from_nibble(b >> 4);
    } else {
      uint8_t* c = static_cast<uint8_t*>(codes);
      c[2 * i] = (uint8_t)(b & 0xFu);
      c[2 * i + 1] = (uint8_t)(b >> 4);
    }
  }
}

// FP32 group scales to FP16 bits (float_to_fp16_bits, pack.hpp:213-258).
__global__ void k_scales_fp16(const float* __restrict__ in, uint16_t* __restrict__ out, size_t n) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = (uint16_t)float_to_fp16_bits(in[i]);
}

static unsigned grid_for(size_t work, int per_block, int sms) {
  size_t g = (work + per_block - 1) / per_block;
  const size_t cap = (size_t)sms * 8;
  if (g > cap) g = cap;
  return (unsigned)(g ? g : 1);
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace qg

using namespace qg;

extern "C" {

const char* qgemm_version(void) { return "qgemm-b200 0.1.0 (sm_100a)"; }

const char* qgemm_status_string(qgemm_status_t s) {
  switch (s) {
    case QGEMM_OK: return "ok";
    case QGEMM_ERR_INVALID_ARG: return "invalid argument";
    case QGEMM_ERR_UNSUPPORTED_SHAPE: return "unsupported shape";
    case QGEMM_ERR_CUDA: return "CUDA error";
    case QGEMM_ERR_NCCL: return "NCCL error";
    case QGEMM_ERR_TIMEOUT: return "device wait timed out";
    case QGEMM_ERR_WORKSPACE: return "workspace missing or too small";
  }
  return "unknown status";
}

const char* qgemm_last_error_message(void) { return t_msg_get(); }

qgemm_status_t qgemm_pack_mxfp4(const float* W, size_t N, size_t K, uint8_t* data,
                                uint8_t* scales, void* stream) {
  if (K % 32 != 0) return fail(QGEMM_ERR_INVALID_ARG, "pack_mxfp4: K must be divisible by 32");
  if (N * K == 0) return QGEMM_OK;
  if (!W || !data || !scales) return fail(QGEMM_ERR_INVALID_ARG, "pack_mxfp4: null pointer");
  if ((reinterpret_cast<uintptr_t>(data) & 3u) != 0)
    return fail(QGEMM_ERR_INVALID_ARG, "pack_mxfp4: data must be 4-byte aligned");
  DevProps dp;
  qgemm_status_t st = device_props(&dp);
  if (st != QGEMM_OK) return st;
  const size_t oct = N * K / 8;
  const unsigned g = grid_for(oct, 256, dp.sm_count);
  if (aligned16(W))
    k_pack_mxfp4<true><<<g, 256, 0, as_stream(stream)>>>(W, oct, reinterpret_cast<uint32_t*>(data), scales);
  else
    k_pack_mxfp4<false><<<g, 256, 0, as_stream(stream)>>>(W, oct, reinterpret_cast<uint32_t*>(data), scales);
  QG_LAUNCH_RET();
  return QGEMM_OK;
}

qgemm_status_t qgemm_pack_nvfp4(const float* W, size_t N, size_t K, float tensor_scale,
                                uint8_t* data, uint8_t* scales, void* stream) {
  if (K % 16 != 0) return fail(QGEMM_ERR_INVALID_ARG, "pack_nvfp4: K must be divisible by 16");
  if (!(tensor_scale > 0.0f) || !std::isfinite(tensor_scale))
    return fail(QGEMM_ERR_INVALID_ARG, "pack_nvfp4: tensor_scale must be finite and > 0");
  if (N * K == 0) return QGEMM_OK;
  if (!W || !data || !scales) return fail(QGEMM_ERR_INVALID_ARG, "pack_nvfp4: null pointer");
  if ((reinterpret_cast<uintptr_t>(data) & 3u) != 0)
    return fail(QGEMM_ERR_INVALID_ARG, "pack_nvfp4: data must be 4-byte aligned");
  DevProps dp;
  qgemm_status_t st = device_props(&dp);
  if (st != QGEMM_OK) return st;
  const size_t oct = N * K / 8;
  const unsigned g = grid_for(oct, 256, dp.sm_count);
  const float inv_t = 1.0f / tensor_scale;  // pack.hpp:517, host IEEE divide
  if (aligned16(W))
    k_pack_nvfp4<true><<<g, 256, 0, as_stream(stream)>>>(W, oct, inv_t, reinterpret_cast<uint32_t*>(data), scales);
  else
    k_pack_nvfp4<false><<<g, 256, 0, as_stream(stream)>>>(W, oct, inv_t, reinterpret_cast<uint32_t*>(data), scales);
  QG_LAUNCH_RET();
  return QGEMM_OK;
}

qgemm_status_t qgemm_pack_int4(const float* W, size_t N, size_t K, int32_t group, uint8_t* data,
                               uint16_t* scales, void* stream) {
  if (group != 64 && group != 128) return fail(QGEMM_ERR_INVALID_ARG, "pack_int4: group must be 64 or 128");
  if (K % (size_t)group != 0) return fail(QGEMM_ERR_INVALID_ARG, "pack_int4: K must be divisible by group");
  if (N * K == 0) return QGEMM_OK;
  if (!W || !data || !scales) return fail(QGEMM_ERR_INVALID_ARG, "pack_int4: null pointer");
  if ((reinterpret_cast<uintptr_t>(data) & 3u) != 0 || (reinterpret_cast<uintptr_t>(scales) & 1u) != 0)
    return fail(QGEMM_ERR_INVALID_ARG, "pack_int4: misaligned output");
  DevProps dp;
  qgemm_status_t st = device_props(&dp);
  if (st != QGEMM_OK) return st;
  const size_t oct = N * K / 8;
  const unsigned g = grid_for(oct, 256, dp.sm_count);
  uint32_t* d32 = reinterpret_cast<uint32_t*>(data);
  cudaStream_t s = as_stream(stream);
  const bool v = aligned16(W);
  if (group == 64) {
    if (v) k_pack_int4<true, 64><<<g, 256, 0, s>>>(W, oct, d32, scales);
    else k_pack_int4<false, 64><<<g, 256, 0, s>>>(W, oct, d32, scales);
  } else {
    if (v) k_pack_int4<true, 128><<<g, 256, 0, s>>>(W, oct, d32, scales);
    else k_pack_int4<false, 128><<<g, 256, 0, s>>>(W, oct, d32, scales);
  }
  QG_LAUNCH_RET();
  return QGEMM_OK;
}

qgemm_status_t qgemm_nvfp4_tensor_scale(const float* W, size_t n, float* out, void* stream) {
  if (!out || (n && !W)) return fail(QGEMM_ERR_INVALID_ARG, "nvfp4_tensor_scale: null pointer");
  cudaStream_t s = as_stream(stream);
  QG_CUDA_RET(cudaMemsetAsync(out, 0, sizeof(float), s));
  if (n) {
    DevProps dp;
    qgemm_status_t st = device_props(&dp);
    if (st != QGEMM_OK) return st;
    k_amax<<<grid_for(n, 256, dp.sm_count), 256, 0, s>>>(W, n, reinterpret_cast<unsigned*>(out));
    QG_LAUNCH_RET();
  }
  k_amax_finish<<<1, 1, 0, s>>>(out);
  QG_LAUNCH_RET();
  return QGEMM_OK;
}

qgemm_status_t qgemm_dequant(const qgemm_weights_t* w, float* out, void* stream) {
  if (!w || !out) return fail(QGEMM_ERR_INVALID_ARG, "dequant: null pointer");
  const size_t N = w->N, K = w->K;
  int group = 0;
  switch (w->format) {
    case QGEMM_FMT_MXFP4: group = 32; break;
    case QGEMM_FMT_NVFP4: group = 16; break;
    case QGEMM_FMT_INT4_G128: group = 128; break;
    case QGEMM_FMT_INT4_G64: group = 64; break;
    default: return fail(QGEMM_ERR_INVALID_ARG, "dequant: unknown format %d", (int)w->format);
  }
  if (K % (size_t)group != 0) return fail(QGEMM_ERR_INVALID_ARG, "dequant: K must be divisible by %d", group);
  if (N * K == 0) return QGEMM_OK;
  if (!w->data || !w->scales) return fail(QGEMM_ERR_INVALID_ARG, "dequant: null pointer");
  if (!aligned16(out) || (reinterpret_cast<uintptr_t>(w->data) & 3u))
    return fail(QGEMM_ERR_INVALID_ARG, "dequant: out must be 16-byte and data 4-byte aligned");
  DevProps dp;
  qgemm_status_t st = device_props(&dp);
  if (st != QGEMM_OK) return st;
  const size_t oct = N * K / 8;
  const unsigned g = grid_for(oct, 256, dp.sm_count);
  cudaStream_t s = as_stream(stream);
  const uint32_t* d32 = reinterpret_cast<const uint32_t*>(w->data);
  if (w->format == QGEMM_FMT_MXFP4) k_dequant<0><<<g, 256, 0, s>>>(d32, w->scales, oct, K, 32, 1.0f, out);
  else if (w->format == QGEMM_FMT_NVFP4) k_dequant<1><<<g, 256, 0, s>>>(d32, w->scales, oct, K, 16, w->tensor_scale, out);
  else k_dequant<2><<<g, 256, 0, s>>>(d32, w->scales, oct, K, group, 1.0f, out);
  QG_LAUNCH_RET();
  return QGEMM_OK;
}

// The block size of a 4-bit format, 0 for an unknown format.
static int format_block(int32_t format) {
  switch (format) {
    case QGEMM_FMT_MXFP4: return 32;
    case QGEMM_FMT_NVFP4: return 16;
    case QGEMM_FMT_INT4_G128: return 128;
    case QGEMM_FMT_INT4_G64: return 64;
    default: return 0;
  }
}

qgemm_status_t qgemm_pack_codes(int32_t format, const void* codes, const void* scales_in, size_t N, size_t K,
                                uint8_t* data, void* scales, void* stream) {
  const int blk = format_block(format);
  if (blk == 0) return fail(QGEMM_ERR_INVALID_ARG, "pack_codes: unknown format %d", (int)format);
  if ((N * K) & 1u) return fail(QGEMM_ERR_INVALID_ARG, "pack_codes: N*K must be even");
  if (K % (size_t)blk != 0) return fail(QGEMM_ERR_INVALID_ARG, "pack_codes: K must be divisible by %d", blk);
  if (N * K == 0) return QGEMM_OK;
  if (!codes || !scales_in || !data || !scales) return fail(QGEMM_ERR_INVALID_ARG, "pack_codes: null pointer");
  DevProps dp;
  qgemm_status_t st = device_props(&dp);
  if (st != QGEMM_OK) return st;
  cudaStream_t s = as_stream(stream);
  const bool int4 = blk >= 64;
  const size_t nbytes = N * K / 2, nscales = N * (K / (size_t)blk);
  k_pack_codes<<<grid_for(nbytes, 256, dp.sm_count), 256, 0, s>>>(int4 ? 1 : 0, codes, data, nbytes);
  QG_LAUNCH_RET();
  if (int4) {
    k_scales_fp16<<<grid_for(nscales, 256, dp.sm_count), 256, 0, s>>>(static_cast<const float*>(scales_in),
                                                                      static_cast<uint16_t*>(scales), nscales);
    QG_LAUNCH_RET();
  } else {
    QG_CUDA_RET(cudaMemcpyAsync(scales, scales_in, nscales, cudaMemcpyDeviceToDevice, s));
  }
  return QGEMM_OK;
}

qgemm_status_t qgemm_unpack_codes(int32_t format, const uint8_t* data, size_t N, size_t K, void* codes,
                                  void* stream) {
  const int blk = format_block(format);
  if (blk == 0) return fail(QGEMM_ERR_INVALID_ARG, "unpack_codes: unknown format %d", (int)format);
  if ((N * K) & 1u) return fail(QGEMM_ERR_INVALID_ARG, "unpack_codes: N*K must be even");
  if (N * K == 0) return QGEMM_OK;
  if (!data || !codes) return fail(QGEMM_ERR_INVALID_ARG, "unpack_codes: null pointer");
  DevProps dp;
  qgemm_status_t st = device_props(&dp);
  if (st != QGEMM_OK) return st;
  const size_t nbytes = N * K / 2;
  k_unpack_codes<<<grid_for(nbytes, 256, dp.sm_count), 256, 0, as_stream(stream)>>>(blk >= 64 ? 1 : 0, data, codes,
                                                                                      nbytes);
  QG_LAUNCH_RET();
  return QGEMM_OK;
}

qgemm_status_t qgemm_codec_encode(int32_t kind, const float* in, void* out, size_t n, void* stream) {
  if (kind < 0 || kind > 3) return fail(QGEMM_ERR_INVALID_ARG, "codec_encode: unknown kind %d", (int)kind);
  if (n == 0) return QGEMM_OK;
  if (!in || !out) return fail(QGEMM_ERR_INVALID_ARG, "codec_encode: null pointer");
  DevProps dp;
  qgemm_status_t st = device_props(&dp);
  if (st != QGEMM_OK) return st;
  k_codec<<<grid_for(n, 256, dp.sm_count), 256, 0, as_stream(stream)>>>(kind, in, out, n);
  QG_LAUNCH_RET();
  return QGEMM_OK;
}

}  // extern "C"
