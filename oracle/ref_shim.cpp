// ref_shim.cpp -- C entry points over the reference's own host code
// (TEST INFRASTRUCTURE ONLY).
//
// Compiled by oracle/Makefile against the reference's unmodified headers
// (titoatwork/qgemm-mx include/qgemm/{pack,ref_gemm,formats}.hpp/.cuh) where
// they lie; the output goes to oracle/_ref/libqgemm_ref.so and never into
// history.  Each function forwards to the reference symbol it names, so tests
// can pin the C oracle against the reference bit for bit, and bench.py can
// time the reference's own CPU path ("dequant_* + gemm_fp32_ref", threaded
// over N-row slices) as the CPU baseline.
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <thread>
#include <vector>

#include "qgemm/formats.cuh"
#include "qgemm/pack.hpp"
#include "qgemm/ref_gemm.hpp"

using namespace qgemm;

extern "C" {

float ref_fp16_bits_to_float(uint16_t h) { return fp16_bits_to_float(h); }
uint16_t ref_float_to_fp16_bits(float f) { return float_to_fp16_bits(f); }
float ref_e2m1_decode(uint8_t c) { return e2m1_decode(c); }
uint8_t ref_e2m1_encode(float v) { return e2m1_encode(v); }
float ref_e8m0_decode(uint8_t b) { return e8m0_decode(b); }
uint8_t ref_e8m0_encode(float s) { return e8m0_encode(s); }
float ref_e4m3_decode(uint8_t b) { return e4m3_decode(b); }
uint8_t ref_e4m3_encode(float v) { return e4m3_encode(v); }
int ref_int4_from_nibble(uint8_t n) { return int4_from_nibble(n); }
uint8_t ref_int4_to_nibble(int v) { return int4_to_nibble(v); }

void ref_e2m1_encode_n(const float* v, uint8_t* o, size_t n) { for (size_t i = 0; i < n; ++i) o[i] = e2m1_encode(v[i]); }
void ref_e8m0_encode_n(const float* v, uint8_t* o, size_t n) { for (size_t i = 0; i < n; ++i) o[i] = e8m0_encode(v[i]); }
void ref_e4m3_encode_n(const float* v, uint8_t* o, size_t n) { for (size_t i = 0; i < n; ++i) o[i] = e4m3_encode(v[i]); }
void ref_fp16_encode_n(const float* v, uint16_t* o, size_t n) { for (size_t i = 0; i < n; ++i) o[i] = float_to_fp16_bits(v[i]); }

// pack_* return 0 on success, 1 where the reference throws std::invalid_argument.
int ref_pack_int4(const float* W, size_t N, size_t K, int group, uint8_t* data, uint16_t* scales) {
  try {
    PackedInt4 p = pack_int4(W, N, K, group);
    std::memcpy(data, p.data.data(), p.data.size());
    std::memcpy(scales, p.scales.data(), p.scales.size() * sizeof(uint16_t));
    return 0;
  } catch (const std::invalid_argument&) { return 1; }
}

int ref_pack_mxfp4(const float* W, size_t N, size_t K, uint8_t* data, uint8_t* scales) {
  try {
    PackedMxfp4 p = pack_mxfp4(W, N, K);
    std::memcpy(data, p.data.data(), p.data.size());
    std::memcpy(scales, p.scales.data(), p.scales.size());
    return 0;
  } catch (const std::invalid_argument&) { return 1; }
}

int ref_pack_nvfp4(const float* W, size_t N, size_t K, float ts, uint8_t* data, uint8_t* scales) {
  try {
    PackedNvfp4 p = pack_nvfp4(W, N, K, ts);
    std::memcpy(data, p.data.data(), p.data.size());
    std::memcpy(scales, p.scales.data(), p.scales.size());
    return 0;
  } catch (const std::invalid_argument&) { return 1; }
}

static PackedInt4 mk_int4(const uint8_t* d, const uint16_t* s, size_t N, size_t K, int g) {
  PackedInt4 p; p.N = N; p.K = K; p.group = g;
  p.data.assign(d, d + N * K / 2);
  p.scales.assign(s, s + N * (K / static_cast<size_t>(g)));
  return p;
}
static PackedMxfp4 mk_mx(const uint8_t* d, const uint8_t* s, size_t N, size_t K) {
  PackedMxfp4 p; p.N = N; p.K = K;
  p.data.assign(d, d + N * K / 2);
  p.scales.assign(s, s + N * (K / 32));
  return p;
}
static PackedNvfp4 mk_nv(const uint8_t* d, const uint8_t* s, size_t N, size_t K, float ts) {
  PackedNvfp4 p; p.N = N; p.K = K; p.tensor_scale = ts;
  p.data.assign(d, d + N * K / 2);
  p.scales.assign(s, s + N * (K / 16));
  return p;
}

void ref_dequant_int4(const uint8_t* d, const uint16_t* s, size_t N, size_t K, int g, float* out) { dequant_int4(mk_int4(d, s, N, K, g), out); }
void ref_dequant_mxfp4(const uint8_t* d, const uint8_t* s, size_t N, size_t K, float* out) { dequant_mxfp4(mk_mx(d, s, N, K), out); }
void ref_dequant_nvfp4(const uint8_t* d, const uint8_t* s, size_t N, size_t K, float ts, float* out) { dequant_nvfp4(mk_nv(d, s, N, K, ts), out); }

void ref_gemm_fp32(const float* X, const float* W, float* Y, size_t M, size_t N, size_t K) { gemm_fp32_ref(X, W, Y, M, N, K); }

size_t ref_weight_bytes(int fmt, size_t N, size_t K) {
  const Format f = fmt == 0 ? Format::MXFP4 : fmt == 1 ? Format::NVFP4 : fmt == 2 ? Format::INT4_G128
                 : fmt == 3 ? Format::INT4_G64 : fmt == 4 ? Format::BF16 : Format::FP8_E4M3;
  return weight_bytes(f, N, K);
}
size_t ref_total_bytes(int fmt, size_t M, size_t N, size_t K) {
  const Format f = fmt == 0 ? Format::MXFP4 : fmt == 1 ? Format::NVFP4 : fmt == 2 ? Format::INT4_G128
                 : fmt == 3 ? Format::INT4_G64 : fmt == 4 ? Format::BF16 : Format::FP8_E4M3;
  return total_bytes(f, M, N, K);
}

// The reference's CPU W4A16 path on rows [n_begin, n_end): per slice of R rows,
// dequant_{mxfp4,nvfp4,int4} of that slice, then gemm_fp32_ref into a slice
// buffer, scattered into Y [M,N].  fmt 0 MXFP4, 1 NVFP4, 2 INT4 (group 64/128).
// X is bf16 bits; each worker thread takes a contiguous range of rows.
int ref_w4a16_gemm(int fmt, const uint8_t* data, const void* scales, size_t N, size_t K,
                   int group, float ts, const uint16_t* Xb, size_t M, float* Y,
                   size_t n_begin, size_t n_end, int nthreads) {
  if (nthreads < 1) nthreads = 1;
  std::vector<float> X(M * K);
  for (size_t i = 0; i < M * K; ++i) {
    uint32_t u = static_cast<uint32_t>(Xb[i]) << 16;
    std::memcpy(&X[i], &u, 4);
  }
  const int blk = fmt == 0 ? 32 : fmt == 1 ? 16 : group;
  auto work = [&](size_t a, size_t b) {
    const size_t R = 16;
    std::vector<float> W;
    std::vector<float> Ys;
    for (size_t n = a; n < b; n += R) {
      const size_t e = std::min(b, n + R), rows = e - n;
      const uint8_t* d = data + n * K / 2;
      if (fmt == 0) {
        W = dequant_reference_mxfp4(mk_mx(d, static_cast<const uint8_t*>(scales) + n * (K / 32), rows, K));
      } else if (fmt == 1) {
        W = dequant_reference_nvfp4(mk_nv(d, static_cast<const uint8_t*>(scales) + n * (K / 16), rows, K, ts));
      } else {
        W = dequant_reference_int4(mk_int4(d, static_cast<const uint16_t*>(scales) + n * (K / blk), rows, K, group));
      }
      Ys = gemm_fp32_ref(X, W, M, rows, K);
      for (size_t m = 0; m < M; ++m)
        for (size_t r = 0; r < rows; ++r) Y[m * N + n + r] = Ys[m * rows + r];
    }
  };
  std::vector<std::thread> th;
  const size_t rows = n_end - n_begin;
  const size_t per = (rows + nthreads - 1) / nthreads;
  for (int t = 0; t < nthreads; ++t) {
    const size_t a = n_begin + t * per;
    if (a >= n_end) break;
    th.emplace_back(work, a, std::min(n_end, a + per));
  }
  for (auto& t : th) t.join();
  return 0;
}

// Code-level packers and unpackers (pack.hpp:611-674); 0 on success, -1 when
// the reference throws.
int ref_pack_int4_codes(const int* q, const float* sc, size_t N, size_t K, int g, uint8_t* data, uint16_t* scales) {
  try {
    PackedInt4 p = pack_int4_codes(q, sc, N, K, g);
    std::memcpy(data, p.data.data(), p.data.size());
    std::memcpy(scales, p.scales.data(), p.scales.size() * 2);
    return 0;
  } catch (const std::invalid_argument&) { return -1; }
}
int ref_pack_mxfp4_codes(const uint8_t* c, const uint8_t* sb, size_t N, size_t K, uint8_t* data, uint8_t* scales) {
  try {
    PackedMxfp4 p = pack_mxfp4_codes(c, sb, N, K);
    std::memcpy(data, p.data.data(), p.data.size());
    std::memcpy(scales, p.scales.data(), p.scales.size());
    return 0;
  } catch (const std::invalid_argument&) { return -1; }
}
int ref_pack_nvfp4_codes(const uint8_t* c, const uint8_t* sb, size_t N, size_t K, float ts, uint8_t* data,
                         uint8_t* scales) {
  try {
    PackedNvfp4 p = pack_nvfp4_codes(c, sb, N, K, ts);
    std::memcpy(data, p.data.data(), p.data.size());
    std::memcpy(scales, p.scales.data(), p.scales.size());
    return 0;
  } catch (const std::invalid_argument&) { return -1; }
}
void ref_unpack_int4_codes(const uint8_t* d, size_t N, size_t K, int* q) {
  PackedInt4 p;
  p.N = N; p.K = K;
  p.data.assign(d, d + N * K / 2);
  unpack_int4_codes(p, q);
}
void ref_unpack_e2m1_codes(const uint8_t* d, size_t N, size_t K, uint8_t* c) { unpack_e2m1_codes(d, N, K, c); }

}  // extern "C"
