// time_graphed_w4a16.cu -- the reference's own benchmark protocol and
// checker driving the B200 library through its C-ABI, written the way a
// maintainer of titoatwork/qgemm-mx adds a bench beside
// src/bench/bench_cublas.cu.
//
// Everything on the reference side is the reference's public header code,
// compiled from its include/ tree:
//   * W is quantised on the host by pack_mxfp4 / pack_nvfp4 / pack_int4
//     (include/qgemm/pack.hpp:424-542); the packed bytes are uploaded
//     unchanged and described by a qgemm_weights_t;
//   * qgemm_gemm_w4a16 runs inside time_graphed and time_looped
//     (include/qgemm/timing.cuh:250-336), cold over rotation_count weight
//     copies and hot on one, as bench_cublas.cu:152-158 times cuBLAS;
//   * the result is checked against gemm_fp32_ref (ref_gemm.hpp:15-27) on
//     the dequantised weights (dequant_reference_*, pack.hpp:588-604) with
//     compare_close (correctness.hpp:317-346), row by row with the W4A16
//     contract's bound: |Y - Y_ref| <= 1e-2 max_n |Y_ref[m, n]|, plus the
//     relative Frobenius bound 1e-3, the reference rounded to bf16 like Y.
//
// Usage: time_graphed_w4a16 <mxfp4|nvfp4|int4_g128|int4_g64> N K M [check_rows]
// check_rows weight rows are checked (half from the start, half from the
// end of W).  Prints one JSON line; exit 0 when the check passes, 1 on a
// mismatch, 2 on a library or argument error.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "qgemm/correctness.hpp"
#include "qgemm/formats.cuh"
#include "qgemm/pack.hpp"
#include "qgemm/ref_gemm.hpp"
#include "qgemm/timing.cuh"
#include "qgemm_b200.h"

using namespace qgemm;

namespace {

uint16_t f32_to_bf16_rne(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
float bf16_to_f32(uint16_t h) {
  const uint32_t u = (uint32_t)h << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

[[noreturn]] void die(const char* what) {
  std::fprintf(stderr, "%s: %s\n", what, qgemm_last_error_message());
  std::exit(2);
}

// The packed bytes of any format, and a sub-matrix of selected weight rows
// dequantised by the reference.
struct HostPacked {
  std::vector<uint8_t> data, scales;  // scales as raw bytes (INT4: FP16 bits)
  float tensor_scale = 1.0f;
  int32_t code = 0;
  Format fmt = Format::MXFP4;
};

HostPacked pack_host(const std::string& name, const std::vector<float>& W, size_t N, size_t K, int* group) {
  HostPacked h;
  if (name == "mxfp4") {
    PackedMxfp4 p = pack_mxfp4(W.data(), N, K);
    h.data = std::move(p.data);
    h.scales = std::move(p.scales);
    h.code = QGEMM_FMT_MXFP4;
    h.fmt = Format::MXFP4;
    *group = 32;
  } else if (name == "nvfp4") {
    float amax = 0.0f;
    for (float v : W) amax = std::max(amax, std::fabs(v));
    PackedNvfp4 p = pack_nvfp4(W.data(), N, K, amax / (448.0f * 6.0f));
    h.data = std::move(p.data);
    h.scales = std::move(p.scales);
    h.tensor_scale = p.tensor_scale;
    h.code = QGEMM_FMT_NVFP4;
    h.fmt = Format::NVFP4;
    *group = 16;
  } else {
    const int g = name == "int4_g64" ? kInt4Group64 : kInt4Group128;
    PackedInt4 p = pack_int4(W.data(), N, K, g);
    h.data = std::move(p.data);
    h.scales.resize(p.scales.size() * 2);
    std::memcpy(h.scales.data(), p.scales.data(), h.scales.size());
    h.code = g == 64 ? QGEMM_FMT_INT4_G64 : QGEMM_FMT_INT4_G128;
    h.fmt = g == 64 ? Format::INT4_G64 : Format::INT4_G128;
    *group = g;
  }
  return h;
}

// Rows `rows` of W, dequantised by the reference's own routines.
std::vector<float> dequant_rows(const HostPacked& h, const std::vector<size_t>& rows, size_t K, int group) {
  const size_t R = rows.size(), bpr = K / 2;
  std::vector<float> out;
  if (h.fmt == Format::MXFP4 || h.fmt == Format::NVFP4) {
    const size_t spr = K / (size_t)group;
    std::vector<uint8_t> d(R * bpr), s(R * spr);
    for (size_t i = 0; i < R; ++i) {
      std::memcpy(&d[i * bpr], &h.data[rows[i] * bpr], bpr);
      std::memcpy(&s[i * spr], &h.scales[rows[i] * spr], spr);
    }
    if (h.fmt == Format::MXFP4) {
      PackedMxfp4 p;
      p.N = R; p.K = K; p.data = d; p.scales = s;
      out = dequant_reference_mxfp4(p);
    } else {
      PackedNvfp4 p;
      p.N = R; p.K = K; p.data = d; p.scales = s; p.tensor_scale = h.tensor_scale;
      out = dequant_reference_nvfp4(p);
    }
  } else {
    const size_t spr = K / (size_t)group;
    PackedInt4 p;
    p.N = R; p.K = K; p.group = group;
    p.data.resize(R * bpr);
    p.scales.resize(R * spr);
    for (size_t i = 0; i < R; ++i) {
      std::memcpy(&p.data[i * bpr], &h.data[rows[i] * bpr], bpr);
      std::memcpy(&p.scales[i * spr], &h.scales[rows[i] * spr * 2], spr * 2);
    }
    out = dequant_reference_int4(p);
  }
  return out;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 5) {
    std::fprintf(stderr, "usage: %s <mxfp4|nvfp4|int4_g128|int4_g64> N K M [check_rows]\n", argv[0]);
    return 2;
  }
  const std::string name = argv[1];
  const size_t N = std::strtoull(argv[2], nullptr, 10), K = std::strtoull(argv[3], nullptr, 10);
  const int M = std::atoi(argv[4]);
  size_t check_rows = argc > 5 ? std::strtoull(argv[5], nullptr, 10) : 256;
  if (N == 0 || K == 0 || M < 1) return 2;
  if (check_rows > N) check_rows = N;

  // W ~ N(0, 0.02), X ~ N(0, 1) rounded to bf16 (seeded)
  std::mt19937_64 rng(1234);
  std::normal_distribution<float> nw(0.0f, 0.02f), nx(0.0f, 1.0f);
  std::vector<float> W(N * K);
  for (auto& v : W) v = nw(rng);
  std::vector<uint16_t> Xb((size_t)M * K);
  std::vector<float> Xf((size_t)M * K);
  for (size_t i = 0; i < Xb.size(); ++i) {
    Xb[i] = f32_to_bf16_rne(nx(rng));
    Xf[i] = bf16_to_f32(Xb[i]);
  }
  int group = 0;
  HostPacked h = pack_host(name, W, N, K, &group);
  W.clear();
  W.shrink_to_fit();

  const DeviceInfo dev = query_device(0);
  QG_CHECK(cudaSetDevice(0));
  const size_t wbytes = h.data.size() + h.scales.size();
  const int rot = rotation_count(wbytes, dev.l2_bytes);
  std::vector<void*> dd(rot), ds(rot);
  std::vector<qgemm_weights_t> w(rot);
  for (int r = 0; r < rot; ++r) {
    QG_CHECK(cudaMalloc(&dd[r], h.data.size()));
    QG_CHECK(cudaMalloc(&ds[r], h.scales.size()));
    QG_CHECK(cudaMemcpy(dd[r], h.data.data(), h.data.size(), cudaMemcpyHostToDevice));
    QG_CHECK(cudaMemcpy(ds[r], h.scales.data(), h.scales.size(), cudaMemcpyHostToDevice));
    w[r] = qgemm_weights_t{h.code, 0, N, K, static_cast<const uint8_t*>(dd[r]), ds[r], h.tensor_scale};
  }
  uint16_t *dX = nullptr, *dY = nullptr;
  QG_CHECK(cudaMalloc(&dX, Xb.size() * 2));
  QG_CHECK(cudaMalloc(&dY, (size_t)M * N * 2));
  QG_CHECK(cudaMemcpy(dX, Xb.data(), Xb.size() * 2, cudaMemcpyHostToDevice));
  const size_t ws_bytes = qgemm_workspace_size(&w[0], M);
  if (ws_bytes == 0) die("qgemm_workspace_size");
  void* ws = nullptr;
  QG_CHECK(cudaMalloc(&ws, ws_bytes));
  if (qgemm_workspace_init(ws, ws_bytes, nullptr) != QGEMM_OK) die("qgemm_workspace_init");

  // The lambda the reference's timing functions call: f(iteration, stream).
  auto gemm = [&](int idx, cudaStream_t st) {
    if (qgemm_gemm_w4a16(&w[idx % rot], dX, M, dY, ws, ws_bytes, st) != QGEMM_OK) die("qgemm_gemm_w4a16");
  };
  auto gemm_hot = [&](int, cudaStream_t st) { gemm(0, st); };
  const int inner = std::max(rot, 8);
  const TimingResult cold = time_graphed(gemm, 10, 40, inner);
  const TimingResult hot = time_graphed(gemm_hot, 10, 40, inner);
  const TimingResult looped = time_looped(gemm, 10, 40, inner);
  int32_t faulted = 0;
  qgemm_umma_status(&faulted);

  // One more call, then the reference's check on the sampled rows.
  cudaStream_t s;
  QG_CHECK(cudaStreamCreate(&s));
  gemm(0, s);
  QG_CHECK(cudaStreamSynchronize(s));
  std::vector<uint16_t> Yb((size_t)M * N);
  QG_CHECK(cudaMemcpy(Yb.data(), dY, Yb.size() * 2, cudaMemcpyDeviceToHost));
  std::vector<size_t> rows;
  for (size_t i = 0; i < check_rows / 2; ++i) rows.push_back(i);
  for (size_t i = N - (check_rows - check_rows / 2); i < N; ++i) rows.push_back(i);
  const std::vector<float> Wd = dequant_rows(h, rows, K, group);
  const size_t R = rows.size();
  std::vector<float> Yref((size_t)M * R);
  gemm_fp32_ref(Xf.data(), Wd.data(), Yref.data(), (size_t)M, R, K);
  bool ok = faulted == 0;
  double worst_ratio = 0.0, num = 0.0, den = 0.0;
  std::vector<float> got(R), ref(R);
  for (int m = 0; m < M; ++m) {
    float rowmax = 0.0f;
    for (size_t j = 0; j < R; ++j) {
      ref[j] = bf16_to_f32(f32_to_bf16_rne(Yref[(size_t)m * R + j]));
      got[j] = bf16_to_f32(Yb[(size_t)m * N + rows[j]]);
      rowmax = std::max(rowmax, std::fabs(ref[j]));
    }
    const CompareResult c = compare_close(got.data(), ref.data(), R, 1e-2f * rowmax, 0.0f);
    ok = ok && c.ok;
    if (rowmax > 0.0f) worst_ratio = std::max(worst_ratio, (double)c.max_abs_err / rowmax);
    for (size_t j = 0; j < R; ++j) {
      num += ((double)got[j] - ref[j]) * ((double)got[j] - ref[j]);
      den += (double)ref[j] * ref[j];
    }
  }
  const double rel = den > 0.0 ? std::sqrt(num / den) : 0.0;
  ok = ok && rel <= 1e-3;
  const size_t moved = total_bytes(h.fmt, (size_t)M, N, K);
  std::printf(
      "{\"format\": \"%s\", \"N\": %zu, \"K\": %zu, \"M\": %d, \"rot\": %d, \"inner\": %d, "
      "\"cold_us\": %.3f, \"hot_us\": %.3f, \"looped_us\": %.3f, \"launch_share_pct\": %.2f, "
      "\"cold_gbs\": %.1f, \"checked_rows\": %zu, \"max_row_ratio\": %.3g, \"rel_frobenius\": %.3g, "
      "\"wait_timed_out\": %s, \"ok\": %s}\n",
      format_name(h.fmt), N, K, M, rot, inner, cold.median_us, hot.median_us, looped.median_us,
      100.0 * (looped.median_us - cold.median_us) / looped.median_us, achieved_gbps(moved, cold.median_us), R,
      worst_ratio, rel, faulted ? "true" : "false", ok ? "true" : "false");
  for (int r = 0; r < rot; ++r) {
    cudaFree(dd[r]);
    cudaFree(ds[r]);
  }
  cudaFree(dX);
  cudaFree(dY);
  cudaFree(ws);
  cudaStreamDestroy(s);
  return ok ? 0 : 1;
}
