// accounting.cu -- byte accounting of titoatwork/qgemm-mx
// include/qgemm/formats.cuh:40-109 and the packed-buffer sizes of
// include/qgemm/pack.hpp:113-153.  Same formulas, so roofline numerators
// computed through this library equal the reference's.
#include "common.cuh"

using namespace qg;

namespace {

// formats.cuh:40-65: element bits and amortised scale bits per element.
double element_bits(int32_t f) {
  switch (f) {
    case QGEMM_FMT_BF16: case QGEMM_FMT_FP16: return 16.0;
    case QGEMM_FMT_FP8_E4M3: return 8.0;
    case QGEMM_FMT_INT4_G128: case QGEMM_FMT_INT4_G64:
    case QGEMM_FMT_MXFP4: case QGEMM_FMT_NVFP4: return 4.0;
  }
  return 0.0;
}
double scale_bits(int32_t f) {
  switch (f) {
    case QGEMM_FMT_INT4_G128: return 16.0 / 128.0;
    case QGEMM_FMT_INT4_G64: return 16.0 / 64.0;
    case QGEMM_FMT_MXFP4: return 8.0 / 32.0;
    case QGEMM_FMT_NVFP4: return 8.0 / 16.0;
  }
  return 0.0;
}

}  // namespace

extern "C" {

double qgemm_bytes_per_weight(int32_t f) { return (element_bits(f) + scale_bits(f)) / 8.0; }

size_t qgemm_weight_bytes(int32_t f, size_t N, size_t K) {
  return static_cast<size_t>(qgemm_bytes_per_weight(f) * static_cast<double>(N) * static_cast<double>(K));
}

size_t qgemm_total_bytes(int32_t f, size_t M, size_t N, size_t K) {
  return qgemm_weight_bytes(f, N, K) + M * K * 2 + M * N * 2;
}

double qgemm_flops(size_t M, size_t N, size_t K) {
  return 2.0 * static_cast<double>(M) * static_cast<double>(N) * static_cast<double>(K);
}

qgemm_status_t qgemm_packed_sizes(int32_t f, size_t N, size_t K, size_t* data_bytes, size_t* scale_bytes) {
  size_t blk = 0, sb = 1;
  switch (f) {
    case QGEMM_FMT_MXFP4: blk = 32; sb = 1; break;
    case QGEMM_FMT_NVFP4: blk = 16; sb = 1; break;
    case QGEMM_FMT_INT4_G128: blk = 128; sb = 2; break;
    case QGEMM_FMT_INT4_G64: blk = 64; sb = 2; break;
    default: return fail(QGEMM_ERR_INVALID_ARG, "packed_sizes: not a 4-bit format (%d)", (int)f);
  }
  if ((N * K) & 1u) return fail(QGEMM_ERR_INVALID_ARG, "packed_sizes: N*K must be even");
  if (K % blk != 0) return fail(QGEMM_ERR_INVALID_ARG, "packed_sizes: K must be divisible by %zu", blk);
  if (data_bytes) *data_bytes = N * K / 2;
  if (scale_bytes) *scale_bytes = N * (K / blk) * sb;
  return QGEMM_OK;
}

}  // extern "C"
