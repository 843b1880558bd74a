// layout.cu -- the scale-checked layout (QGEMM_LAYOUT_SCALE_CHECKED): the
// canonical bytes, checked once offline to hold no scale byte outside the
// range the decode kernel decodes by exponent arithmetic.
//
// Derivation (the reference plans a layout derived from the dequantisation
// instruction sequence, docs/D1_LAYOUT_DERIVATION.md:17-52):
//  * codes: the decode kernel feeds each lane one 32-bit word per 32-k block
//    (codes 8j .. 8j+7 of the block), converted by cvt.rn.f16x2.e2m1x2 into
//    two MMA fragments without shuffles, so the canonical nibble order
//    already suits it (a permutation giving one 128-bit load per chunk
//    measured slower); the block-scaled tcgen05 kernel needs every 32
//    consecutive codes in shared memory to share one scale, which any
//    interleaving across blocks breaks.  Codes stay canonical.
//  * scales: the decode kernel turns an E8M0 byte b into 2^(b - 127) by an
//    exponent shift, exact for b in 1 .. 254; 0x00 (2^-127) and 0xFF (NaN)
//    need the exact decoder, and so do NVFP4's E4M3 zero, subnormal and NaN
//    bytes for the f16 widening.  Searching every chunk's scale words for
//    them cost 7-9 % of the decode kernel's time (gate-up and down at M = 1).
//    Per-unit flags stored after the scales, read in the consumer loop, kept
//    only 1.5 % of that; what pays is knowing it for the whole matrix, which
//    one offline scan establishes.  Real checkpoints rarely hold such bytes;
//    matrices that do stay canonical and take the checked decode.
#include <cuda_runtime.h>

#include "common.cuh"

namespace qg {

// *found |= 1 if any scale byte is outside the fast range.
__global__ void k_scan_scales(int fmt, const uint8_t* __restrict__ scales, size_t n, unsigned* found) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  bool special = false;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const uint32_t v = scales[i];
    if (fmt == QGEMM_FMT_MXFP4) special |= (v == 0u || v == 0xFFu);
    else special |= (((v >> 3) & 0xFu) == 0u || (v & 0x7Fu) == 0x7Fu);
  }
  if (__any_sync(0xFFFFFFFFu, special) && (threadIdx.x & 31) == 0) atomicOr(found, 1u);
}

static qgemm_status_t sizes_of(int32_t format, int32_t layout, size_t N, size_t K, size_t* d, size_t* s) {
  if (layout != QGEMM_LAYOUT_CANONICAL && layout != QGEMM_LAYOUT_SCALE_CHECKED)
    return fail(QGEMM_ERR_INVALID_ARG, "layout: unknown layout %d", (int)layout);
  if (layout == QGEMM_LAYOUT_SCALE_CHECKED && format != QGEMM_FMT_MXFP4 && format != QGEMM_FMT_NVFP4)
    return fail(QGEMM_ERR_INVALID_ARG, "layout: the scale-checked layout is MXFP4 / NVFP4 only");
  return qgemm_packed_sizes(format, N, K, d, s);
}

}  // namespace qg

using namespace qg;

extern "C" {

qgemm_status_t qgemm_layout_sizes(int32_t format, int32_t layout, size_t N, size_t K, size_t* data_bytes,
                                  size_t* scale_bytes) {
  if (!data_bytes || !scale_bytes) return fail(QGEMM_ERR_INVALID_ARG, "layout_sizes: null pointer");
  return sizes_of(format, layout, N, K, data_bytes, scale_bytes);
}

qgemm_status_t qgemm_repack(const qgemm_weights_t* src, int32_t layout, uint8_t* data, void* scales, void* stream) {
  if (!src || !data || !scales) return fail(QGEMM_ERR_INVALID_ARG, "repack: null pointer");
  if (src->layout != QGEMM_LAYOUT_CANONICAL) return fail(QGEMM_ERR_INVALID_ARG, "repack: source must be canonical");
  size_t db = 0, sb = 0;
  qgemm_status_t st = sizes_of(src->format, layout, src->N, src->K, &db, &sb);
  if (st != QGEMM_OK) return st;
  if (src->N * src->K == 0) return QGEMM_OK;
  if (!src->data || !src->scales) return fail(QGEMM_ERR_INVALID_ARG, "repack: null source pointer");
  cudaStream_t s = as_stream(stream);
  if (layout == QGEMM_LAYOUT_SCALE_CHECKED) {
    DevProps dp;
    st = device_props(&dp);
    if (st != QGEMM_OK) return st;
    unsigned* found = nullptr;
    QG_CUDA_RET(cudaMallocAsync(reinterpret_cast<void**>(&found), sizeof(unsigned), s));
    unsigned h = 0;
    cudaError_t e = cudaMemsetAsync(found, 0, sizeof(unsigned), s);
    if (e == cudaSuccess) {
      size_t blocks = (sb + 255) / 256;
      if (blocks > (size_t)dp.sm_count * 8) blocks = (size_t)dp.sm_count * 8;
      k_scan_scales<<<(unsigned)(blocks ? blocks : 1), 256, 0, s>>>(src->format,
                                                                    static_cast<const uint8_t*>(src->scales), sb, found);
      e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(&h, found, sizeof(unsigned), cudaMemcpyDeviceToHost, s);
    const cudaError_t ef = cudaFreeAsync(found, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e == cudaSuccess) e = ef;
    if (e != cudaSuccess) return fail(QGEMM_ERR_CUDA, "repack: scale scan: %s", cudaGetErrorString(e));
    if (h) return fail(QGEMM_ERR_INVALID_ARG, "repack: scales hold bytes outside the fast decode's range; keep the canonical layout");
  }
  if (data != src->data) QG_CUDA_RET(cudaMemcpyAsync(data, src->data, db, cudaMemcpyDeviceToDevice, s));
  if (scales != src->scales) QG_CUDA_RET(cudaMemcpyAsync(scales, src->scales, sb, cudaMemcpyDeviceToDevice, s));
  return QGEMM_OK;
}

qgemm_status_t qgemm_unpack(const qgemm_weights_t* src, uint8_t* data, void* scales, void* stream) {
  if (!src || !data || !scales) return fail(QGEMM_ERR_INVALID_ARG, "unpack: null pointer");
  if (const char* e = layout_error(src)) return fail(QGEMM_ERR_INVALID_ARG, "unpack: %s", e);
  size_t db = 0, sb = 0;
  qgemm_status_t st = qgemm_packed_sizes(src->format, src->N, src->K, &db, &sb);
  if (st != QGEMM_OK) return st;
  if (src->N * src->K == 0) return QGEMM_OK;
  if (!src->data || !src->scales) return fail(QGEMM_ERR_INVALID_ARG, "unpack: null source pointer");
  cudaStream_t s = as_stream(stream);
  if (data != src->data) QG_CUDA_RET(cudaMemcpyAsync(data, src->data, db, cudaMemcpyDeviceToDevice, s));
  if (scales != src->scales) QG_CUDA_RET(cudaMemcpyAsync(scales, src->scales, sb, cudaMemcpyDeviceToDevice, s));
  return QGEMM_OK;
}

}  // extern "C"
