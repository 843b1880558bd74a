/*
 * qgemm_oracle.h -- CPU oracle for the W4A16 path (TEST INFRASTRUCTURE ONLY).
 *
 * A plain-C restatement of the reference's host codecs, packers, dequantisers
 * and reference GEMM (titoatwork/qgemm-mx include/qgemm/pack.hpp and
 * include/qgemm/ref_gemm.hpp).  Every function names the reference lines whose
 * decision rule it restates.  The oracle is pinned two ways (tests/):
 *   1. against the reference headers themselves, compiled by oracle/Makefile
 *      into oracle/_ref/libqgemm_ref.so, on seeded random and edge inputs;
 *   2. against the known-answer vectors of the reference's own tests
 *      (tests/test_pack_roundtrip.cpp, tests/test_formats.cpp,
 *      tests/test_ref_gemm.cpp), restated in tests/test_oracle_golden.py.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load this library, and only as the checker / the timed CPU baseline.  The
 * CUDA product path never calls into it.
 *
 * Floating-point environment: IEEE-754 binary32/binary64, round-to-nearest,
 * subnormals honoured (build without -ffast-math).  Where the reference's C++
 * has behaviour that is undefined in the language but fixed on x86-64 (a
 * float-to-int conversion of NaN or of an out-of-range value), the oracle
 * states the x86-64 result explicitly (INT32_MIN).
 */
#ifndef QGEMM_ORACLE_H
#define QGEMM_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes returned by the packers (mirror the reference's throws). */
#define OR_OK 0
#define OR_EINVAL 1

/* ---- scalar codecs (pack.hpp:183-390) ---------------------------------- */
float    or_fp16_bits_to_float(uint16_t h);
uint16_t or_float_to_fp16_bits(float f);
float    or_e2m1_decode(uint8_t code);
uint8_t  or_e2m1_encode(float v);
float    or_e8m0_decode(uint8_t bits);
uint8_t  or_e8m0_encode(float scale);
float    or_e4m3_decode(uint8_t bits);
uint8_t  or_e4m3_encode(float v);
int      or_int4_from_nibble(uint8_t n);
uint8_t  or_int4_to_nibble(int v);
uint16_t or_f32_to_bf16_bits(float f);   /* RNE, NaN kept quiet */
float    or_bf16_bits_to_f32(uint16_t b);

/* batch forms used by the codec parity tests */
void or_e2m1_encode_n(const float* v, uint8_t* out, size_t n);
void or_e8m0_encode_n(const float* v, uint8_t* out, size_t n);
void or_e4m3_encode_n(const float* v, uint8_t* out, size_t n);
void or_fp16_encode_n(const float* v, uint16_t* out, size_t n);

/* ---- packers (pack.hpp:424-542).  Outputs must be pre-sized:
 *      data  = N*K/2 bytes, scales = N*(K/block) entries.              ---- */
int or_pack_int4(const float* W, size_t N, size_t K, int group,
                 uint8_t* data, uint16_t* scales);
int or_pack_mxfp4(const float* W, size_t N, size_t K,
                  uint8_t* data, uint8_t* scales);
int or_pack_nvfp4(const float* W, size_t N, size_t K, float tensor_scale,
                  uint8_t* data, uint8_t* scales);

/* NVFP4 per-tensor scale used by the build: max|W| / (448*6). */
float or_nvfp4_tensor_scale(const float* W, size_t n);

/* ---- dequantisers (pack.hpp:548-585) ----------------------------------- */
void or_dequant_int4(const uint8_t* data, const uint16_t* scales, size_t N,
                     size_t K, int group, float* out);
void or_dequant_mxfp4(const uint8_t* data, const uint8_t* scales, size_t N,
                      size_t K, float* out);
void or_dequant_nvfp4(const uint8_t* data, const uint8_t* scales, size_t N,
                      size_t K, float tensor_scale, float* out);

/* ---- reference GEMM (ref_gemm.hpp:15-27): Y[m,n] = sum_k X[m,k] W[n,k],
 *      double accumulation, one rounding to float.                     ---- */
void or_gemm_ref(const float* X, const float* W, float* Y, size_t M, size_t N,
                 size_t K);

/* Fused CPU path "dequant rows of W, then the reference GEMM", threaded over
 * N-row slices.  X is bf16 bits [M,K]; Y is float [M,N].  fmt: 0 MXFP4,
 * 1 NVFP4, 2 INT4 (group 64/128).  Rows [n_begin, n_end) only; Y keeps its
 * full [M,N] stride.  Returns OR_OK or OR_EINVAL. */
int or_w4a16_gemm(int fmt, const uint8_t* data, const void* scales,
                  size_t N, size_t K, int group, float tensor_scale,
                  const uint16_t* X_bf16, size_t M, float* Y,
                  size_t n_begin, size_t n_end, int nthreads);

/* ---- seeded generators (this build's documented generator) ------------
 * splitmix64 seeding of xoshiro256**, Box-Muller on 53-bit uniforms, so
 * numbers do not depend on any C++ library's normal_distribution.        */
void or_randn(uint64_t seed, uint64_t stream, float mean, float std, float* out,
              size_t n);
/* X ~ N(mean,std) rounded to bf16 (RNE); returns bf16 bits. */
void or_randn_bf16(uint64_t seed, uint64_t stream, float mean, float std,
                   uint16_t* out, size_t n);

#ifdef __cplusplus
}
#endif
#endif /* QGEMM_ORACLE_H */
