// gemv.cu -- decode-path W4A16 GEMM for small M (M <= 16 per launch).
//
// Y[M,N] = X[M,K] . W[N,K]^T with W in the reference's packed layouts
// (titoatwork/qgemm-mx include/qgemm/pack.hpp:14-85) streamed from HBM once.
// The path is HBM-bound; the kernel is built so that (1) every weight byte is
// read once with coalesced loads, (2) every warp gets an equal share of the
// weight stream on any (N, K) (stream-K), and (3) dequantisation costs about
// one instruction per weight, because an instruction-bound kernel cannot keep
// HBM busy.
//
// Two launches per call, chained with programmatic dependent launch:
//  k_xprep  X (bf16) -> f16 with a per-row power-of-two prescale 2^-s_m chosen
//           so that max|x_m| * 2^-s_m lies in [2^14, 2^15).  Every bf16 value
//           at or above max|x_m| * 2^-31 converts exactly (8 significant bits
//           fit f16's 11); smaller ones round to f16's subnormal grid, an
//           error below 2^-39 * max|x_m| per element.  The FP32 epilogue
//           multiplies by 2^s_m, so no information is lost.
//  k_gemv   swap-AB warp MMA (mma.sync m16n8k16, f16 in, fp32 accumulate):
//           16 weight rows are the MMA's M side, <= 8 activation rows per
//           n-tile its N side.  W codes are widened by the hardware
//           cvt.rn.f16x2.e2m1x2 (sign included) or, for INT4, by an f16
//           magic-number conversion; all dequantised values are exact.
//             MXFP4  the E8M0 block scale is applied to the FP32 partial sum of
//                    each 32-block (post-scale): the K-slot mapping puts one
//                    block in each pair of MMAs.
//             NVFP4  e2m1*e4m3 has <= 6 significant bits within [2^-10, 2688]
//                    and is exact in f16: the block scale is folded into the
//                    operand with one f16x2 multiply; the FP32 tensor scale is
//                    applied in the epilogue.
//             INT4   q in [-8,7] is exact in f16; each 64/128-group's FP32
//                    partial sum is scaled by its FP16 scale.
//           Products are exact in the FP32 accumulator, so Y differs from the
//           double-accumulated reference (ref_gemm.hpp:15-27) only by FP32
//           summation order and the tensor scale applied once per output.
//
// K-slot mapping: an m16n8k16 MMA reduces over 16 k slots; lane (g = lane/4,
// j = lane%4) owns slots {2j, 2j+1, 2j+8, 2j+9}.  Any bijection between slots
// and true k works if the weight (A) and activation (B) fragments agree, so
// lanes load contiguous runs of packed codes and k_xprep writes X in the
// matching order.
//
// Schedule: stream-K.  The iteration space (tile of 32 weight rows, 128-k
// chunk) is cut into one contiguous range per warp.  A tile finished inside
// one warp is stored directly; a tile split across warps leaves FP32 partial
// fragments in the workspace, and the warp whose atomic ticket shows it
// arrived last sums all contributors' partials in warp order (deterministic)
// and stores Y.  There is no spin-wait anywhere in this file.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <atomic>

#include "common.cuh"
#include "gemv_core.cuh"
#include "tp.cuh"

namespace qg {

constexpr int kWarpsPerCta = 4;
constexpr int kChunkK = 128;
constexpr int kRowTiles = 2;          // 16-row MMA tiles per warp tile
constexpr int kTileRows = 16 * kRowTiles;
constexpr int kMaxM = 16;             // activation rows per launch

struct GemvArgs {
  const uint8_t* data;
  const void* scales;
  const __half* Xh;     // [mpad, K] f16, prescaled (and permuted for INT4)
  const float* xs;      // [mpad] 2^s_m
  void* Y;
  int M, N, K, ldy;
  float ts;
  float* partials;      // [2 * W_total][slot]
  unsigned* counters;   // [tiles]
  long long T;          // iterations = tiles * C
  int C;                // chunks per tile: ceil(K / 128)
  int ktail;            // K % 128: the last chunk's valid k (0 = a whole chunk)
  int W_total;          // warps that own iterations
};

// ---------------------------------------------------------------------------
// X preparation
// ---------------------------------------------------------------------------

// One CTA per activation row.  For INT4 formats the f16 values of each group
// of 8 are stored in the order (x0,x4,x1,x5,x2,x6,x3,x7) to match the
// (c_i, c_i+4) pairs that int4x8_to_f16 produces.
// Output layouts (lp = layout parameter):
//  0  row-major [M][K].
//  1  tcgen05 operand image (lp = BN): for each block of BN activation rows
//     and each 64-k block, BN rows of 128 bytes whose 16-byte chunk c is
//     stored at chunk c ^ (row % 8) -- the shared-memory image of a
//     128-byte-swizzled K-major tile, so one linear bulk copy stages it.
// (The TMA-fed decode kernel has its own preparation, k_xprep_units.)
// Rows M .. (padded row count) - 1 (one CTA each) are written as zeros.
__device__ __forceinline__ size_t xprep_index(int m, int k, int K, int layout, int lp) {
  if (layout == 0) return (size_t)m * K + k;
  const int mb = m / lp, r = m % lp, kb = k >> 6, c = (k >> 3) & 7;
  return (((size_t)mb * (K >> 6) + kb) * lp + r) * 64 + (size_t)((c ^ (r & 7)) << 3);
}
// One pass: every thread issues all its 16-byte loads of the row before it
// uses any (up to kXpChunks of them, i.e. K <= 256 * 8 * kXpChunks), keeps
// them in registers for the block-wide |x| maximum and converts from there;
// longer rows load the remainder again for the conversion.  Launched as a
// programmatic dependent: it waits for the previous grid before reading X
// (which that grid may have produced) or writing Xh / xs (which it may read).
constexpr int kXpThreads = 256;
constexpr int kXpChunks = 16;
__device__ __forceinline__ void xprep_store(const uint4 v, float inv, int perm, __half* dst) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  float f[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = u2f(w[i] << 16) * inv;
    f[2 * i + 1] = u2f(w[i] & 0xFFFF0000u) * inv;
  }
  __half2 o[4];
  if (perm) {
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = __floats2half2_rn(f[i], f[i + 4]);
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
  }
  *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(o);
}
__device__ __forceinline__ float absmax8(const uint4 v, float a) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    a = fmaxf(a, fabsf(u2f(w[i] << 16)));
    a = fmaxf(a, fabsf(u2f(w[i] & 0xFFFF0000u)));
  }
  return a;
}
__global__ void __launch_bounds__(kXpThreads) k_xprep(const uint16_t* __restrict__ X, int M, int K, int perm,
                                                      int layout, int lp, __half* __restrict__ Xh,
                                                      float* __restrict__ xs) {
  // Dependents may launch at once (this grid is resident when the trigger
  // fires); they read nothing written here before their own wait returns.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int m = blockIdx.x;
  constexpr int kStride = kXpThreads * 8;
  if (m >= M) {  // zero padding rows of the last activation block
    for (int k = threadIdx.x * 8; k < K; k += kStride)
      *reinterpret_cast<uint4*>(Xh + xprep_index(m, k, K, layout, lp)) = make_uint4(0u, 0u, 0u, 0u);
    return;
  }
  __shared__ float red[kXpThreads / 32];
  __shared__ float s_inv;
  const uint16_t* xr = X + (size_t)m * K;
  uint4 v[kXpChunks];
#pragma unroll
  for (int i = 0; i < kXpChunks; ++i) {
    const int k = threadIdx.x * 8 + i * kStride;
    v[i] = k < K ? *reinterpret_cast<const uint4*>(xr + k) : make_uint4(0u, 0u, 0u, 0u);
  }
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < kXpChunks; ++i) amax = absmax8(v[i], amax);
  for (int k = threadIdx.x * 8 + kXpChunks * kStride; k < K; k += kStride)
    amax = absmax8(*reinterpret_cast<const uint4*>(xr + k), amax);
#pragma unroll
  for (int d = 16; d; d >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, d));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x == 0) {
    float a = 0.0f;
    for (int i = 0; i < kXpThreads / 32; ++i) a = fmaxf(a, red[i]);
    int s = 0;
    if (a > 0.0f && isfinite(a)) {
      s = ilogbf(a) - 14;
      s = s < -126 ? -126 : (s > 114 ? 114 : s);
    }
    xs[m] = u2f((uint32_t)(127 + s) << 23);    // 2^s
    s_inv = u2f((uint32_t)(127 - s) << 23);    // 2^-s
  }
  __syncthreads();
  const float inv = s_inv;
#pragma unroll
  for (int i = 0; i < kXpChunks; ++i) {
    const int k = threadIdx.x * 8 + i * kStride;
    if (k < K) xprep_store(v[i], inv, perm, Xh + xprep_index(m, k, K, layout, lp));
  }
  for (int k = threadIdx.x * 8 + kXpChunks * kStride; k < K; k += kStride)
    xprep_store(*reinterpret_cast<const uint4*>(xr + k), inv, perm, Xh + xprep_index(m, k, K, layout, lp));
}

// PDL launch of k_xprep over `rows` CTAs (rows >= M: the extra rows are zeroed).
static cudaError_t launch_xprep(const uint16_t* X, int M, int rows, int K, int perm, int layout, int lp, __half* Xh,
                                float* xs, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)rows);
  cfg.blockDim = dim3(kXpThreads);
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_xprep, X, M, K, perm, layout, lp, Xh, xs);
}

// ---------------------------------------------------------------------------
// The decode kernel
// ---------------------------------------------------------------------------

template <int FMT, int NT, bool F32OUT>
__global__ void __launch_bounds__(kWarpsPerCta * 32) k_gemv(const GemvArgs a) {
  constexpr int R = kRowTiles;
  constexpr int FRAG = R * NT * 4;  // accumulator floats per lane
  const int lane = threadIdx.x & 31;
  const int w = blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
  const int g = lane >> 2, j = lane & 3;
  const int M = a.M, N = a.N, K = a.K, C = a.C;
  const size_t rowb = (size_t)K / 2;
  const bool active = w < a.W_total;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // the next call's kernels may launch
  const long long start = active ? (long long)w * a.T / a.W_total : 0;
  const long long end = active ? (long long)(w + 1) * a.T / a.W_total : 0;

  float acc[R][NT][4];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[r][t][e] = 0.0f;

  // Registers of one iteration: packed words and scale bits of rows g and
  // g+8 of each row tile, and the X fragment of each n-tile.
  uint32_t wq[R][2][4], sc[R][2];
  uint32_t xf[NT][16];

  // Valid k of chunk c: a whole chunk, or K % 128 in the last one.  Past the
  // end of the row the codes and X are zero and the scales neutral (finite),
  // so those slots add nothing; nothing is read there.  With K % 128 != 0 a
  // row's scales are not word-aligned, so they are read a byte (u16) at a time.
  auto chunk_k = [&](int c) { return (a.ktail != 0 && c == C - 1) ? a.ktail : kChunkK; };
  auto load_w = [&](int tile, int c) {
    const int kv = chunk_k(c);
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int n = tile * kTileRows + 16 * r + 8 * h + g;
#pragma unroll
        for (int q = 0; q < 4; ++q) wq[r][h][q] = 0u;
        sc[r][h] = 0u;
        if (n < N) {
          const uint8_t* row = a.data + (size_t)n * rowb + (size_t)c * (kChunkK / 2);
          if constexpr (FMT == 0) {  // 4 bytes of each of the 4 blocks
            const uint8_t* srow = static_cast<const uint8_t*>(a.scales) + (size_t)n * (K / 32) + 4 * c;
            if (kv == kChunkK) {
#pragma unroll
              for (int b = 0; b < 4; ++b) wq[r][h][b] = ldg_first4(row + 16 * b + 4 * j);
            } else {
#pragma unroll
              for (int b = 0; b < 4; ++b)
                if (32 * b < kv) wq[r][h][b] = ldg_first4(row + 16 * b + 4 * j);
            }
            if (a.ktail == 0) {
              sc[r][h] = __ldg(reinterpret_cast<const uint32_t*>(srow));
            } else {
              uint32_t v = 0u;
#pragma unroll
              for (int b = 0; b < 4; ++b) v |= (32 * b < kv ? (uint32_t)__ldg(srow + b) : 127u) << (8 * b);
              sc[r][h] = v;
            }
          } else if constexpr (FMT == 3) {  // 8 bytes of each 64-group
            const uint16_t* srow = static_cast<const uint16_t*>(a.scales) + (size_t)n * (K / 64) + 2 * c;
            const uint2 lo = ldg_stream8(row + 8 * j);
            wq[r][h][0] = lo.x; wq[r][h][1] = lo.y;
            if (kv == kChunkK) {
              const uint2 hi = ldg_stream8(row + 32 + 8 * j);
              wq[r][h][2] = hi.x; wq[r][h][3] = hi.y;
            }
            if (a.ktail == 0)
              sc[r][h] = __ldg(reinterpret_cast<const uint32_t*>(srow));
            else  // K % 64 == 0: a tail chunk holds exactly one group
              sc[r][h] = (uint32_t)__ldg(srow) | (kv == kChunkK ? (uint32_t)__ldg(srow + 1) << 16 : 0u);
          } else if constexpr (FMT == 1) {  // 16 bytes = k 32 j .. 32 j + 31: blocks 2 j, 2 j + 1
            const int vj = kv - 32 * j;          // valid k of the lane's 32: <= 0, 16 or >= 32
            const uint8_t* srow = static_cast<const uint8_t*>(a.scales) + (size_t)n * (K / 16) + 8 * c + 2 * j;
            if ((K & 31) == 0) {                 // rows start on 16-byte boundaries
              if (vj > 0) {
                const uint4 v = ldg_stream16(row + 16 * j);
                wq[r][h][0] = v.x; wq[r][h][1] = v.y; wq[r][h][2] = v.z; wq[r][h][3] = v.w;
                sc[r][h] = __ldg(reinterpret_cast<const uint16_t*>(srow));
              } else {
                sc[r][h] = 0x3838u;              // E4M3 1.0 for both blocks
              }
            } else {                             // K % 32 == 16: 8-byte rows, scale pairs unaligned
              if (vj > 0) {
                const uint2 lo = ldg_stream8(row + 16 * j);
                wq[r][h][0] = lo.x; wq[r][h][1] = lo.y;
                uint32_t s1 = 0x38u;
                if (vj >= 32) {
                  const uint2 hi = ldg_stream8(row + 16 * j + 8);
                  wq[r][h][2] = hi.x; wq[r][h][3] = hi.y;
                  s1 = __ldg(srow + 1);
                }
                sc[r][h] = (uint32_t)__ldg(srow) | (s1 << 8);
              } else {
                sc[r][h] = 0x3838u;
              }
            }
          } else {  // INT4 g128: 16 contiguous bytes (K % 128 == 0)
            const uint4 v = ldg_stream16(row + 16 * j);
            wq[r][h][0] = v.x; wq[r][h][1] = v.y; wq[r][h][2] = v.z; wq[r][h][3] = v.w;
            sc[r][h] = __ldg(static_cast<const uint16_t*>(a.scales) + (size_t)n * (K / 128) + c);
          }
        }
      }
  };
  auto load_x = [&](int c) {
    const int kv = chunk_k(c);
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const int m = 8 * t + g;
      if (m < M) {
        const __half* xr = a.Xh + (size_t)m * K + (size_t)c * kChunkK;
        uint4 v[4];
        if constexpr (FMT == 0) {
#pragma unroll
          for (int b = 0; b < 4; ++b) v[b] = (32 * b < kv) ? ldg_keep16(xr + 32 * b + 8 * j) : z;
        } else if constexpr (FMT == 3) {
          v[0] = ldg_keep16(xr + 16 * j); v[1] = ldg_keep16(xr + 16 * j + 8);
          v[2] = (kv == kChunkK) ? ldg_keep16(xr + 64 + 16 * j) : z;
          v[3] = (kv == kChunkK) ? ldg_keep16(xr + 64 + 16 * j + 8) : z;
        } else {  // NVFP4 / INT4 g128: k 32 j + 8 q .. + 7 (valid in whole 16-blocks)
#pragma unroll
          for (int q = 0; q < 4; ++q) v[q] = (32 * j + 8 * q < kv) ? ldg_keep16(xr + 32 * j + 8 * q) : z;
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          xf[t][4 * q] = v[q].x; xf[t][4 * q + 1] = v[q].y; xf[t][4 * q + 2] = v[q].z; xf[t][4 * q + 3] = v[q].w;
        }
      } else {
#pragma unroll
        for (int q = 0; q < 16; ++q) xf[t][q] = 0u;
      }
    }
  };

  auto store_tile = [&](int tile, float (&v)[R][NT][4]) {
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      float xsc[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int m = 8 * t + 2 * j + e;
        xsc[e] = (m < M) ? a.xs[m] : 0.0f;
        if (FMT == 1) xsc[e] *= a.ts;
      }
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int n = tile * kTileRows + 16 * r + g + ((e & 2) ? 8 : 0);
          const int m = 8 * t + 2 * j + (e & 1);
          if (n < N && m < M) {
            const float y = v[r][t][e] * xsc[e & 1];
            if (F32OUT) static_cast<float*>(a.Y)[(size_t)m * a.ldy + n] = y;
            else static_cast<__nv_bfloat16*>(a.Y)[(size_t)m * a.ldy + n] = __float2bfloat16_rn(y);
          }
        }
    }
  };

  auto slot_of = [&](int wid, int tile) -> size_t {
    const long long s = (long long)wid * a.T / a.W_total;
    return (size_t)(2 * wid + ((int)(s / C) == tile ? 0 : 1));
  };

  auto flush = [&](int tile, bool full) {
    if (full) {
      store_tile(tile, acc);
    } else {
      float4* mine = reinterpret_cast<float4*>(a.partials) + slot_of(w, tile) * (FRAG / 4) * 32;
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t)
          __stcg(mine + ((r * NT + t) * 32 + lane),
                 make_float4(acc[r][t][0], acc[r][t][1], acc[r][t][2], acc[r][t][3]));
      __syncwarp();  // the warp's partial stores, then one acquire-release ticket
      const long long t0 = (long long)tile * C, t1 = t0 + C - 1;
      const int w_lo = (int)(((t0 + 1) * a.W_total - 1) / a.T);
      const int w_hi = (int)(((t1 + 1) * a.W_total - 1) / a.T);
      unsigned ticket = 0;
      if (lane == 0) ticket = ticket_acq_rel(a.counters + tile);
      ticket = __shfl_sync(0xFFFFFFFFu, ticket, 0);
      if ((int)ticket == w_hi - w_lo) {  // last contributor: reduce in warp order
        float sum[R][NT][4];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int t = 0; t < NT; ++t)
#pragma unroll
            for (int e = 0; e < 4; ++e) sum[r][t][e] = 0.0f;
        // CB contributors' partials in flight before the first add (they
        // come from L2); the adds stay in warp order
        constexpr int CB = NT == 1 ? 4 : 2;
#pragma unroll 1
        for (int wb = w_lo; wb <= w_hi; wb += CB) {
          float4 pv[CB][R][NT];
#pragma unroll
          for (int j = 0; j < CB; ++j)
            if (wb + j <= w_hi) {
              const float4* src =
                  reinterpret_cast<const float4*>(a.partials) + slot_of(wb + j, tile) * (FRAG / 4) * 32;
#pragma unroll
              for (int r = 0; r < R; ++r)
#pragma unroll
                for (int t = 0; t < NT; ++t) pv[j][r][t] = __ldcg(src + ((r * NT + t) * 32 + lane));
            }
#pragma unroll
          for (int j = 0; j < CB; ++j)
            if (wb + j <= w_hi) {
#pragma unroll
              for (int r = 0; r < R; ++r)
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                  sum[r][t][0] += pv[j][r][t].x; sum[r][t][1] += pv[j][r][t].y;
                  sum[r][t][2] += pv[j][r][t].z; sum[r][t][3] += pv[j][r][t].w;
                }
            }
        }
        store_tile(tile, sum);
        if (lane == 0) a.counters[tile] = 0u;  // leave the workspace zeroed
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[r][t][e] = 0.0f;
  };

  // Weights do not depend on X: start streaming them before waiting for the
  // X-preparation grid.
  // (tile, c) of the current iteration and of the next one, advanced
  // incrementally: no 64-bit division inside the loop.
  int tile = (int)(start / C), c = (int)(start % C);
  if (start < end) load_w(tile, c);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (start >= end) return;
  load_x(c);

  bool seg_full_start = (c == 0);
  for (long long it = start; it < end; ++it) {
    int ntile = tile, nc = c + 1;
    if (nc == C) { nc = 0; ++ntile; }
    uint32_t cw[R][2][4], cs[R][2], cx[NT][16];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        cs[r][h] = sc[r][h];
#pragma unroll
        for (int q = 0; q < 4; ++q) cw[r][h][q] = wq[r][h][q];
      }
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int q = 0; q < 16; ++q) cx[t][q] = xf[t][q];
    if (it + 1 < end) { load_w(ntile, nc); load_x(nc); }

    chunk_mma<FMT, R, NT>(acc, cw, cs, cx);

    if (c == C - 1 || it + 1 == end) {
      flush(tile, seg_full_start && (c == C - 1));
      seg_full_start = true;  // the next segment starts at chunk 0
    }
    tile = ntile;
    c = nc;
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

struct GemvPlan {
  int fmt = 0, nt = 1;
  int tiles = 0, C = 0;
  long long T = 0;
  int grid = 0, W_total = 0;
  int mpad = 8;
  size_t counter_bytes = 0, partial_bytes = 0, xs_bytes = 0, xh_bytes = 0;
  size_t total() const { return counter_bytes + partial_bytes + xs_bytes + xh_bytes; }
};

static int fmt_code(int32_t format) {
  switch (format) {
    case QGEMM_FMT_MXFP4: return 0;
    case QGEMM_FMT_NVFP4: return 1;
    case QGEMM_FMT_INT4_G128: return 2;
    case QGEMM_FMT_INT4_G64: return 3;
  }
  return -1;
}

template <int FMT, int NT>
static int occupancy_of() {
  static int occ[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 1;
  if (occ[dev] == 0) {
    int v = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, k_gemv<FMT, NT, false>, kWarpsPerCta * 32, 0) !=
            cudaSuccess || v < 1)
      v = 1;
    occ[dev] = v;
  }
  return occ[dev];
}

template <int FMT>
static int occ_for(int nt) { return nt == 1 ? occupancy_of<FMT, 1>() : occupancy_of<FMT, 2>(); }

static size_t pad256(size_t b) { return (b + 255) & ~(size_t)255; }

size_t ws_ticket_bytes(size_t N) {
  size_t n = (N + kTileRows - 1) / kTileRows;
  const size_t grouped = (size_t)32 * ((N + 127) / 128);
  if (grouped > n) n = grouped;
  if (n < 512) n = 512;
  return pad256(n * sizeof(unsigned));
}

// Plan for one launch over mb (<= 16) activation rows.
qgemm_status_t gemv_plan(const qgemm_weights_t* w, int mb, GemvPlan* p) {
  const int f = fmt_code(w->format);
  if (f < 0) return fail(QGEMM_ERR_INVALID_ARG, "gemm: unknown format %d", (int)w->format);
  if (w->K == 0 || w->N == 0) return fail(QGEMM_ERR_INVALID_ARG, "gemm: empty weight matrix");
  // K need not be a multiple of the 128-k chunk: the last chunk may hold
  // K % 128 valid k in whole blocks (32 MXFP4, 16 NVFP4) or 64-groups (INT4 g64).
  const size_t kq = f == 0 ? 32 : f == 1 ? 16 : f == 3 ? 64 : 128;
  if (w->K % kq != 0)
    return fail(QGEMM_ERR_UNSUPPORTED_SHAPE, "gemm: K=%zu is not a multiple of %zu", w->K, kq);
  if (w->K > (size_t)INT32_MAX / 2 || w->N > (size_t)INT32_MAX / 2)
    return fail(QGEMM_ERR_UNSUPPORTED_SHAPE, "gemm: N or K too large");
  DevProps dp;
  qgemm_status_t st = device_props(&dp);
  if (st != QGEMM_OK) return st;
  p->fmt = f;
  p->nt = mb <= 8 ? 1 : 2;
  p->mpad = 8 * p->nt;
  p->tiles = (int)((w->N + kTileRows - 1) / kTileRows);
  p->C = (int)((w->K + kChunkK - 1) / kChunkK);
  p->T = (long long)p->tiles * p->C;
  int occ = 1;
  switch (f) {
    case 0: occ = occ_for<0>(p->nt); break;
    case 1: occ = occ_for<1>(p->nt); break;
    case 2: occ = occ_for<2>(p->nt); break;
    default: occ = occ_for<3>(p->nt); break;
  }
  long long warps = (long long)dp.sm_count * occ * kWarpsPerCta;
  if (warps > p->T) warps = p->T;
  p->W_total = (int)warps;
  p->grid = (int)((warps + kWarpsPerCta - 1) / kWarpsPerCta);
  const size_t slot = (size_t)kRowTiles * p->nt * 4 * 32 * sizeof(float);
  p->counter_bytes = ws_ticket_bytes(w->N);
  p->partial_bytes = pad256(2 * (size_t)p->W_total * slot);
  p->xs_bytes = pad256((size_t)kMaxM * sizeof(float));
  p->xh_bytes = pad256((size_t)kMaxM * w->K * sizeof(__half));
  return QGEMM_OK;
}

// Scratch of the LDG-fed path for a call over M activation rows, launched
// in blocks of 16 rows: [counters | partials | xs | Xh].  A tail block of
// M % 16 rows plans on its own (<= 8 rows: one n-tile, its own occupancy and
// warp count), so the partial region is sized for the larger of the first
// block's and the tail block's plans; every launch checks its plan against it.
struct LdgLayout {
  GemvPlan first;
  size_t partial_bytes = 0;  // reserved partial region
  size_t total = 0;
};
static qgemm_status_t ldg_layout(const qgemm_weights_t* w, int M, LdgLayout* L) {
  qgemm_status_t st = gemv_plan(w, M < kMaxM ? M : kMaxM, &L->first);
  if (st != QGEMM_OK) return st;
  L->partial_bytes = L->first.partial_bytes;
  if (M > kMaxM && (M % kMaxM) != 0) {
    GemvPlan tail;
    st = gemv_plan(w, M % kMaxM, &tail);
    if (st != QGEMM_OK) return st;
    if (tail.partial_bytes > L->partial_bytes) L->partial_bytes = tail.partial_bytes;
  }
  L->total = L->first.counter_bytes + L->partial_bytes + L->first.xs_bytes + L->first.xh_bytes;
  return QGEMM_OK;
}

// Launches of the LDG-fed path over all M rows, in blocks of 16, with the
// scratch at `base` laid out by L.
static qgemm_status_t ldg_run(const qgemm_weights_t* w, const uint16_t* X, int M, void* Y, bool f32,
                              uint8_t* base, const LdgLayout& L, cudaStream_t s, const char* who);

template <int FMT, bool F32>
static cudaError_t launch_fmt(const GemvPlan& p, const GemvArgs& a, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.grid);
  cfg.blockDim = dim3(kWarpsPerCta * 32);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (p.nt == 1) return cudaLaunchKernelEx(&cfg, k_gemv<FMT, 1, F32>, a);
  return cudaLaunchKernelEx(&cfg, k_gemv<FMT, 2, F32>, a);
}

template <bool F32>
static cudaError_t launch_gemv(const GemvPlan& p, const GemvArgs& a, cudaStream_t s) {
  switch (p.fmt) {
    case 0: return launch_fmt<0, F32>(p, a, s);
    case 1: return launch_fmt<1, F32>(p, a, s);
    case 2: return launch_fmt<2, F32>(p, a, s);
    default: return launch_fmt<3, F32>(p, a, s);
  }
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

qgemm_status_t gemm_umma_ts(const qgemm_weights_t* w, const __half* Xh, const float* xs, int M, void* Y, bool f32,
                            int splits, unsigned* tickets, void* partials, cudaStream_t s);
int umma_splits(const qgemm_weights_t* w, int M, int sm_count);
size_t umma_split_workspace(const qgemm_weights_t* w, int M, int splits);  // partials only

bool umma_bs_supported(const qgemm_weights_t* w, int M);
int umma_bs_launches(const qgemm_weights_t* w, int M, int sm_count);
size_t umma_bs_workspace(const qgemm_weights_t* w, int M, int sm_count);
qgemm_status_t gemm_umma_bs(const qgemm_weights_t* w, const uint16_t* X, int M, void* Y, bool f32, void* ws,
                            int sm_count, cudaStream_t s, const TpOut* tp);
bool umma_sk_supported(const qgemm_weights_t* w, int M);
int umma_sk_bn(int M);
size_t umma_sk_workspace(const qgemm_weights_t* w, int M, int sm_count);  // partials only
qgemm_status_t gemm_umma_sk(const qgemm_weights_t* w, const __half* Xh, const float* xs, int M, void* Y, bool f32,
                            unsigned* tickets, void* partials, int sm_count, cudaStream_t s, const TpOut* tp);

bool gemv_tma_supported(const qgemm_weights_t* w, int mb);
size_t gemv_tma_workspace(const qgemm_weights_t* w, int sm_count);
qgemm_status_t gemm_gemv_tma(const qgemm_weights_t* w, const uint16_t* X, int mb, void* Y, int ldy, bool f32,
                             void* ws, int sm_count, cudaStream_t s, const TpOut* tp);
// [counters | partials | X image] (gemv_tma.cu)
static size_t decode_tma_workspace(const qgemm_weights_t* w, int sms) { return gemv_tma_workspace(w, sms); }

// The tcgen05 paths (dequantised W in TMEM) take M >= 32, and NVFP4 / INT4
// from M = 17 (one pass over W instead of two 16-row decode passes; X is
// padded to 32 zero rows): every format on the persistent stream-K kernel
// for M < 128, K % 256 == 0 and at least 2^26 weights (umma_sk.cu), and on the
// tile-per-CTA kernel with K splits otherwise (K % 64 == 0, umma.cu).  Their
// workspace holds the f16 copy of X, its row factors and the split tiles'
// tickets and partial sums.
static bool use_umma(const qgemm_weights_t* w, int M) {
  return (M >= 32 || (M >= 17 && w->format != QGEMM_FMT_MXFP4)) && w->K % 64 == 0;
}
static int umma_ts_rows(int M) { return M < 32 ? 32 : M; }  // the tile kernel's X rows
static int sm_count_or_zero() {
  DevProps dp;
  return device_props(&dp) == QGEMM_OK ? dp.sm_count : 0;
}
static int umma_split_count(const qgemm_weights_t* w, int M) {
  const int sms = sm_count_or_zero();
  return sms > 0 ? umma_splits(w, M, sms) : 1;
}
// [tickets | xs | Xh | split partials]
static size_t umma_xh_bytes(const qgemm_weights_t* w, int M) {
  const int rows = umma_sk_supported(w, M) ? (M + umma_sk_bn(M) - 1) / umma_sk_bn(M) * umma_sk_bn(M)
                                           : umma_ts_rows(M);
  return pad256((size_t)rows * w->K * sizeof(__half));
}
static size_t umma_workspace(const qgemm_weights_t* w, int M) {
  const size_t head = ws_ticket_bytes(w->N) + pad256((size_t)M * sizeof(float)) + umma_xh_bytes(w, M);
  if (umma_sk_supported(w, M)) {
    const int sms = sm_count_or_zero();
    return sms > 0 ? head + umma_sk_workspace(w, M, sms) : 0;
  }
  return head + umma_split_workspace(w, M, umma_split_count(w, M));
}

// tp: tensor-parallel output (kernels that write every rank's Y_full); only
// with the TMA-fed decode and stream-K tcgen05 kernels, Y unused then.
qgemm_status_t gemm_decode_ex(const qgemm_weights_t* w, const uint16_t* X, int M, void* Y, bool f32, void* ws,
                              size_t ws_bytes, cudaStream_t s, const TpOut* tp) {
  if (!w || !X || (!Y && !tp)) return fail(QGEMM_ERR_INVALID_ARG, "gemm: null pointer");
  if (M < 1) return fail(QGEMM_ERR_INVALID_ARG, "gemm: M must be >= 1");
  if (!w->data || !w->scales) return fail(QGEMM_ERR_INVALID_ARG, "gemm: null weight pointer");
  if (const char* le = layout_error(w)) return fail(QGEMM_ERR_INVALID_ARG, "gemm: %s", le);
  if (w->format == QGEMM_FMT_NVFP4 && !std::isfinite(w->tensor_scale))
    return fail(QGEMM_ERR_INVALID_ARG, "gemm: NVFP4 tensor_scale must be finite");
  GemvPlan p;
  qgemm_status_t st = gemv_plan(w, M < kMaxM ? M : kMaxM, &p);
  if (st != QGEMM_OK) return st;
  const uintptr_t sa = reinterpret_cast<uintptr_t>(w->scales);
  const bool scales_ok = (w->format == QGEMM_FMT_NVFP4) ? (sa & 1u) == 0 : (sa & 3u) == 0;
  if (!al16(w->data) || !al16(X) || !scales_ok)
    return fail(QGEMM_ERR_INVALID_ARG, "gemm: data and X must be 16-byte aligned, scales 4-byte aligned");
  if (umma_bs_supported(w, M)) {  // MXFP4, M <= 128: block-scaled tensor cores, no dequantisation
    const int sms = sm_count_or_zero();
    const size_t need = sms > 0 ? umma_bs_workspace(w, M, sms) : 0;
    if (!ws || !al16(ws) || ws_bytes < need || need == 0)
      return fail(QGEMM_ERR_WORKSPACE, "gemm: 16-byte aligned workspace of %zu bytes needed, %zu given", need,
                  ws_bytes);
    return gemm_umma_bs(w, X, M, Y, f32, ws, sms, s, tp);
  }
  if (use_umma(w, M)) {
    const size_t need = umma_workspace(w, M);
    if (!ws || !al16(ws) || ws_bytes < need)
      return fail(QGEMM_ERR_WORKSPACE, "gemm: 16-byte aligned workspace of %zu bytes needed, %zu given", need,
                  ws_bytes);
    unsigned* tickets = static_cast<unsigned*>(ws);
    uint8_t* head = static_cast<uint8_t*>(ws) + ws_ticket_bytes(w->N);
    float* xs = reinterpret_cast<float*>(head);
    __half* xh = reinterpret_cast<__half*>(head + pad256((size_t)M * sizeof(float)));
    void* part = head + pad256((size_t)M * sizeof(float)) + umma_xh_bytes(w, M);
    // INT4: X in the pair order int4x8_to_f16 widens codes in
    const int perm = (w->format == QGEMM_FMT_INT4_G128 || w->format == QGEMM_FMT_INT4_G64) ? 1 : 0;
    if (umma_sk_supported(w, M)) {
      const int bn = umma_sk_bn(M);
      QG_CUDA_RET(launch_xprep(X, M, (M + bn - 1) / bn * bn, (int)w->K, perm, 1, bn, xh, xs, s));
      return gemm_umma_sk(w, xh, xs, M, Y, f32, tickets, part, sm_count_or_zero(), s, tp);
    }
    if (tp) return fail(QGEMM_ERR_UNSUPPORTED_SHAPE, "gemm: no tensor-parallel output on this path");
    QG_CUDA_RET(launch_xprep(X, M, umma_ts_rows(M), (int)w->K, perm, 0, 0, xh, xs, s));
    return gemm_umma_ts(w, xh, xs, M, Y, f32, umma_split_count(w, M), tickets, part, s);
  }
  if (gemv_tma_supported(w, M < kMaxM ? M : kMaxM)) {
    // TMA-fed decode kernel (gemv_tma.cu): X preparation + GEMM per 16
    // activation rows
    const int sms = sm_count_or_zero();
    const size_t need = decode_tma_workspace(w, sms);
    if (sms <= 0 || !ws || !al16(ws) || ws_bytes < need)
      return fail(QGEMM_ERR_WORKSPACE, "gemm: 16-byte aligned workspace of %zu bytes needed, %zu given", need,
                  ws_bytes);
    for (int m0 = 0; m0 < M; m0 += kMaxM) {
      const int mb = (M - m0) < kMaxM ? (M - m0) : kMaxM;
      const uint16_t* Xb = X + (size_t)m0 * w->K;
      if (tp) {  // this block's rows of every rank's Y_full
        TpOut tb = *tp;
        for (int d = 0; d < tb.world; ++d) tb.y[d] += (size_t)m0 * tb.ldy;
        st = gemm_gemv_tma(w, Xb, mb, nullptr, 0, false, ws, sms, s, &tb);
      } else {
        void* Yb = f32 ? (void*)(static_cast<float*>(Y) + (size_t)m0 * w->N)
                       : (void*)(static_cast<uint16_t*>(Y) + (size_t)m0 * w->N);
        st = gemm_gemv_tma(w, Xb, mb, Yb, (int)w->N, f32, ws, sms, s, nullptr);
      }
      if (st != QGEMM_OK) return st;
    }
    return QGEMM_OK;
  }
  if (tp) return fail(QGEMM_ERR_UNSUPPORTED_SHAPE, "gemm: no tensor-parallel output on this path");
  LdgLayout L;
  st = ldg_layout(w, M, &L);
  if (st != QGEMM_OK) return st;
  if (!ws || !al16(ws) || ws_bytes < L.total)
    return fail(QGEMM_ERR_WORKSPACE, "gemm: 16-byte aligned workspace of %zu bytes needed, %zu given", L.total,
                ws_bytes);
  return ldg_run(w, X, M, Y, f32, static_cast<uint8_t*>(ws), L, s, "gemm");
}

static qgemm_status_t ldg_run(const qgemm_weights_t* w, const uint16_t* X, int M, void* Y, bool f32,
                              uint8_t* base, const LdgLayout& L, cudaStream_t s, const char* who) {
  const GemvPlan& p = L.first;
  GemvArgs a;
  a.data = w->data; a.scales = w->scales; a.N = (int)w->N; a.K = (int)w->K; a.ldy = (int)w->N;
  a.ts = w->tensor_scale;
  a.counters = reinterpret_cast<unsigned*>(base);
  a.partials = reinterpret_cast<float*>(base + p.counter_bytes);
  float* xs = reinterpret_cast<float*>(base + p.counter_bytes + L.partial_bytes);
  __half* xh = reinterpret_cast<__half*>(base + p.counter_bytes + L.partial_bytes + p.xs_bytes);
  a.xs = xs; a.Xh = xh;
  const int perm = (w->format == QGEMM_FMT_INT4_G128 || w->format == QGEMM_FMT_INT4_G64) ? 1 : 0;
  for (int m0 = 0; m0 < M; m0 += kMaxM) {
    const int mb = (M - m0) < kMaxM ? (M - m0) : kMaxM;
    GemvPlan pb;
    qgemm_status_t st = gemv_plan(w, mb, &pb);
    if (st != QGEMM_OK) return st;
    if (pb.partial_bytes > L.partial_bytes || pb.counter_bytes != p.counter_bytes)
      return fail(QGEMM_ERR_WORKSPACE, "%s: block plan needs %zu partial bytes, %zu reserved", who,
                  pb.partial_bytes, L.partial_bytes);
    a.T = pb.T; a.C = pb.C; a.ktail = (int)(w->K % kChunkK); a.W_total = pb.W_total; a.M = mb;
    a.Y = f32 ? (void*)(static_cast<float*>(Y) + (size_t)m0 * w->N)
              : (void*)(static_cast<uint16_t*>(Y) + (size_t)m0 * w->N);
    QG_CUDA_RET(launch_xprep(X + (size_t)m0 * w->K, mb, mb, (int)w->K, perm, 0, 0, xh, xs, s));
    const cudaError_t e = f32 ? launch_gemv<true>(pb, a, s) : launch_gemv<false>(pb, a, s);
    if (e != cudaSuccess) return fail(QGEMM_ERR_CUDA, "%s: launch failed: %s", who, cudaGetErrorString(e));
  }
  return QGEMM_OK;
}

qgemm_status_t gemm_decode(const qgemm_weights_t* w, const uint16_t* X, int M, void* Y, bool f32, void* ws,
                           size_t ws_bytes, cudaStream_t s) {
  return gemm_decode_ex(w, X, M, Y, f32, ws, ws_bytes, s, nullptr);
}

size_t gemm_decode_workspace(const qgemm_weights_t* w, int M) {
  if (w && M >= 1 && umma_bs_supported(w, M)) {
    const int sms = sm_count_or_zero();
    return sms > 0 ? umma_bs_workspace(w, M, sms) : 0;
  }
  if (w && use_umma(w, M)) return umma_workspace(w, M);
  if (w && M >= 1 && gemv_tma_supported(w, M < kMaxM ? M : kMaxM)) {
    const int sms = sm_count_or_zero();
    return sms > 0 ? decode_tma_workspace(w, sms) : 0;
  }
  LdgLayout L;
  if (!w || M < 1 || ldg_layout(w, M, &L) != QGEMM_OK) return 0;
  return L.total;
}

// Mirrors gemm_decode's dispatch: launches per call and the GEMM kernel used.
int32_t gemm_launch_count(const qgemm_weights_t* w, int M, int32_t* kernel) {
  if (!w || M < 1 || fmt_code(w->format) < 0) return -1;
  {  // the shapes the GEMM entry accepts (gemv_plan's checks, which every call makes first)
    const int f = fmt_code(w->format);
    const size_t kq = f == 0 ? 32 : f == 1 ? 16 : f == 3 ? 64 : 128;
    if (w->K == 0 || w->N == 0 || w->K % kq != 0 || w->K > (size_t)INT32_MAX / 2 || w->N > (size_t)INT32_MAX / 2)
      return -1;
  }
  int k = 0, n = 0;
  if (umma_bs_supported(w, M)) {
    k = 4;
    n = umma_bs_launches(w, M, sm_count_or_zero());  // k_xprep_bs + k_umma_bs (+ k_bs_fixup for split tiles)
  } else if (use_umma(w, M)) {
    k = umma_sk_supported(w, M) ? 2 : 3;
    n = 2;  // k_xprep + the tcgen05 kernel
  } else {
    k = gemv_tma_supported(w, M < kMaxM ? M : kMaxM) ? 1 : 0;
    n = 2 * ((M + kMaxM - 1) / kMaxM);  // per 16 activation rows: X preparation + decode kernel
  }
  if (kernel) *kernel = k;
  return n;
}

}  // namespace qg

using namespace qg;

extern "C" {

size_t qgemm_workspace_size(const qgemm_weights_t* w, int32_t M) { return gemm_decode_workspace(w, M); }

int32_t qgemm_launch_count(const qgemm_weights_t* w, int32_t M, int32_t* kernel) {
  return gemm_launch_count(w, M, kernel);
}

qgemm_status_t qgemm_workspace_init(void* ws, size_t ws_bytes, void* stream) {
  if (!ws && ws_bytes) return fail(QGEMM_ERR_INVALID_ARG, "workspace_init: null pointer");
  if (ws_bytes) QG_CUDA_RET(cudaMemsetAsync(ws, 0, ws_bytes, as_stream(stream)));
  return QGEMM_OK;
}

qgemm_status_t qgemm_gemm_w4a16(const qgemm_weights_t* w, const uint16_t* X, int32_t M, uint16_t* Y, void* ws,
                                size_t ws_bytes, void* stream) {
  return gemm_decode(w, X, M, Y, false, ws, ws_bytes, as_stream(stream));
}

qgemm_status_t qgemm_gemm_w4a16_f32(const qgemm_weights_t* w, const uint16_t* X, int32_t M, float* Y, void* ws,
                                    size_t ws_bytes, void* stream) {
  return gemm_decode(w, X, M, Y, true, ws, ws_bytes, as_stream(stream));
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free decode GEMM
// ---------------------------------------------------------------------------
//
// Some callers cannot hand the library a workspace: an operator slot whose
// fixed signature carries only inputs, outputs and a stream; a plugin running
// inside a host framework that owns the device memory pool and forbids raw
// cudaMalloc; code that runs while another component captures the stream in
// global mode, where cudaMalloc is an unsafe call.  For them the decode
// kernel's scratch (split-tile partial sums, tile tickets, the f16 copy of X)
// lives in a fixed device array that the library reserves once.
//
// Properties:
//  * 16 MiB of device memory per GPU that loads the library, held until the
//    process exits.  Calls whose plan needs more scratch (about K > 300k, or a
//    device with far more SMs) return QGEMM_ERR_WORKSPACE; the check covers
//    every 16-row block of the call, the tail block's own plan included.
//  * The first call on each device looks up the array's device address with
//    cudaGetSymbolAddress and keeps it for the life of the process; make that
//    first call before any stream capture.  cudaDeviceReset destroys the
//    context the address belongs to: a process that resets a device must not
//    call this entry point on that device again.
//  * Every call shares the array: calls that may overlap on the GPU (other
//    streams, other threads) race and must be serialised by the caller.
//  * The tile tickets that must start at zero are cleared by each call
//    (cudaMemsetAsync on the caller's stream); nothing is allocated.
//  * Always runs the decode kernel (any M, in blocks of 16 activation rows).

namespace qg {

constexpr size_t kNoAllocScratchBytes = (size_t)16 << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

// The array's device address per device ordinal.  Threads that race on the
// first lookup store the same value; the atomics make that well defined.
static qgemm_status_t noalloc_scratch(uint8_t** out) {
  static std::atomic<uint8_t*> ptrs[64];
  int dev = 0;
  QG_CUDA_RET(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(QGEMM_ERR_CUDA, "gemm_noalloc: device ordinal %d out of range", dev);
  uint8_t* p = ptrs[dev].load(std::memory_order_acquire);
  if (!p) {
    void* q = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&q, g_noalloc_scratch);
    if (e != cudaSuccess || !q)
      return fail(QGEMM_ERR_CUDA, "gemm_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    p = static_cast<uint8_t*>(q);
    ptrs[dev].store(p, std::memory_order_release);
  }
  *out = p;
  return QGEMM_OK;
}

}  // namespace qg

extern "C" qgemm_status_t qgemm_gemm_w4a16_noalloc(const qgemm_weights_t* w, const uint16_t* X, int32_t M,
                                                   uint16_t* Y, void* stream) {
  using namespace qg;
  cudaStream_t s = as_stream(stream);
  if (!w || !X || !Y) return fail(QGEMM_ERR_INVALID_ARG, "gemm_noalloc: null pointer");
  if (M < 1) return fail(QGEMM_ERR_INVALID_ARG, "gemm_noalloc: M must be >= 1");
  if (!w->data || !w->scales) return fail(QGEMM_ERR_INVALID_ARG, "gemm_noalloc: null weight pointer");
  if (const char* le = layout_error(w)) return fail(QGEMM_ERR_INVALID_ARG, "gemm_noalloc: %s", le);
  if (w->format == QGEMM_FMT_NVFP4 && !std::isfinite(w->tensor_scale))
    return fail(QGEMM_ERR_INVALID_ARG, "gemm_noalloc: NVFP4 tensor_scale must be finite");
  LdgLayout L;
  qgemm_status_t st = ldg_layout(w, M, &L);
  if (st != QGEMM_OK) return st;
  const uintptr_t sa = reinterpret_cast<uintptr_t>(w->scales);
  const bool scales_ok = (w->format == QGEMM_FMT_NVFP4) ? (sa & 1u) == 0 : (sa & 3u) == 0;
  if (!al16(w->data) || !al16(X) || !scales_ok)
    return fail(QGEMM_ERR_INVALID_ARG, "gemm_noalloc: data and X must be 16-byte aligned, scales 4-byte aligned");
  if (L.total > kNoAllocScratchBytes)
    return fail(QGEMM_ERR_WORKSPACE, "gemm_noalloc: needs %zu bytes of scratch, the fixed array holds %zu",
                L.total, kNoAllocScratchBytes);
  uint8_t* base = nullptr;
  st = noalloc_scratch(&base);
  if (st != QGEMM_OK) return st;
  QG_CUDA_RET(cudaMemsetAsync(base, 0, L.first.counter_bytes, s));
  return ldg_run(w, X, M, Y, false, base, L, s, "gemm_noalloc");
}

// ---------------------------------------------------------------------------
// Grouped GEMM (mixture of experts)
// ---------------------------------------------------------------------------
//
// E experts of one format and shape; expert e multiplies its M[e] rows of X
// (rows offs[e] ..) and writes the same rows of Y.  Decode-sized experts
// (MXFP4 / NVFP4, 1 <= M[e] <= 16) run kGroupChunk at a time through the
// TMA-fed decode kernel with one stream-K iteration space over all their
// units, so a step with many small experts pays two launches and one pipeline
// fill per chunk instead of per expert; every other expert runs as a
// regular call.  All of them share one workspace (tickets at its start).

namespace qg {

size_t gemv_tma_group_workspace(const qgemm_weights_t* w, int sm_count);
qgemm_status_t gemm_gemv_tma_group(const qgemm_weights_t* const* w, const int* M, const size_t* row0, int n,
                                   const uint16_t* X, uint16_t* Y, void* ws, int sm_count, cudaStream_t s);
constexpr int kGroupChunk = 32;  // problems per fused launch (the kernel's parameter block holds 32)

static bool grouped_fused(const qgemm_weights_t* w, int m) {
  return m >= 1 && m <= kMaxM && gemv_tma_supported(w, m);
}

// Workspace for calls whose experts have at most max_m rows: the fused
// launches' and every regular call's, maximised over the experts' pointer
// alignments (which select kernels) and over 1 .. max_m rows.
static size_t grouped_workspace(const qgemm_weights_t* w, int E, int max_m) {
  if (!w || E < 1 || max_m < 1) return 0;
  const int sms = sm_count_or_zero();
  if (sms <= 0) return 0;
  size_t need = ws_ticket_bytes(w[0].N);
  unsigned seen = 0;  // alignment classes done: data 32-byte aligned x scales address mod 16
  for (int e = 0; e < E; ++e) {
    const uintptr_t d = reinterpret_cast<uintptr_t>(w[e].data), sc = reinterpret_cast<uintptr_t>(w[e].scales);
    const unsigned cls = ((d & 31u) == 0 ? 16u : 0u) | (unsigned)(sc & 15u);
    if (seen & (1u << cls)) continue;
    seen |= 1u << cls;
    for (int m = 1; m <= max_m; ++m) {
      const size_t b = grouped_fused(&w[e], m) ? gemv_tma_group_workspace(&w[e], sms) : gemm_decode_workspace(&w[e], m);
      if (b == 0) return 0;
      if (b > need) need = b;
    }
  }
  return need;
}

static qgemm_status_t grouped_gemm(const qgemm_weights_t* w, int E, const uint16_t* X, const int32_t* M,
                                   const int64_t* offs, uint16_t* Y, void* ws, size_t ws_bytes, cudaStream_t s) {
  if (E < 0) return fail(QGEMM_ERR_INVALID_ARG, "grouped_gemm: E must be >= 0");
  if (E == 0) return QGEMM_OK;
  if (!w || !X || !Y || !M || !offs) return fail(QGEMM_ERR_INVALID_ARG, "grouped_gemm: null pointer");
  int max_m = 0;
  for (int e = 0; e < E; ++e) {
    const qgemm_weights_t& we = w[e];
    if (we.format != w[0].format || we.N != w[0].N || we.K != w[0].K)
      return fail(QGEMM_ERR_INVALID_ARG, "grouped_gemm: expert %d differs from expert 0 in format or shape", e);
    if (const char* le = layout_error(&we)) return fail(QGEMM_ERR_INVALID_ARG, "grouped_gemm: expert %d: %s", e, le);
    if (M[e] < 0 || offs[e] < 0)
      return fail(QGEMM_ERR_INVALID_ARG, "grouped_gemm: expert %d has M %d, row offset %lld", e, M[e],
                  (long long)offs[e]);
    if (M[e] > max_m) max_m = M[e];
  }
  if (max_m == 0) return QGEMM_OK;
  const int sms = sm_count_or_zero();
  const size_t need = grouped_workspace(w, E, max_m);
  if (sms <= 0 || need == 0) return fail(QGEMM_ERR_UNSUPPORTED_SHAPE, "grouped_gemm: no plan for this shape");
  if (!ws || !al16(ws) || ws_bytes < need)
    return fail(QGEMM_ERR_WORKSPACE, "grouped_gemm: 16-byte aligned workspace of %zu bytes needed, %zu given", need,
                ws_bytes);
  const size_t N = w[0].N, K = w[0].K;
  const qgemm_weights_t* cw[kGroupChunk];
  int cm[kGroupChunk];
  size_t cr[kGroupChunk];
  int n = 0;
  auto flush = [&]() -> qgemm_status_t {
    if (n == 0) return QGEMM_OK;
    const qgemm_status_t st = gemm_gemv_tma_group(cw, cm, cr, n, X, Y, ws, sms, s);
    n = 0;
    return st;
  };
  for (int e = 0; e < E; ++e) {
    if (M[e] == 0) continue;
    const qgemm_weights_t* we = &w[e];
    if (!we->data || !we->scales || layout_error(we) ||
        (we->format == QGEMM_FMT_NVFP4 && !std::isfinite(we->tensor_scale)) || !al16(we->data))
      return fail(QGEMM_ERR_INVALID_ARG, "grouped_gemm: expert %d: null or misaligned weights, or bad tensor_scale", e);
    if (grouped_fused(we, M[e]) && al16(X)) {
      cw[n] = we; cm[n] = M[e]; cr[n] = (size_t)offs[e];
      if (++n == kGroupChunk) {
        const qgemm_status_t st = flush();
        if (st != QGEMM_OK) return st;
      }
    } else {
      const qgemm_status_t st = gemm_decode(we, X + (size_t)offs[e] * K, M[e], Y + (size_t)offs[e] * N, false, ws,
                                            ws_bytes, s);
      if (st != QGEMM_OK) return st;
    }
  }
  return flush();
}

}  // namespace qg

extern "C" size_t qgemm_grouped_workspace_size(const qgemm_weights_t* w, int32_t E, int32_t max_m) {
  return qg::grouped_workspace(w, E, max_m);
}

extern "C" qgemm_status_t qgemm_grouped_gemm_w4a16(const qgemm_weights_t* w, int32_t E, const uint16_t* X,
                                                   const int32_t* M, const int64_t* offs, uint16_t* Y, void* ws,
                                                   size_t ws_bytes, void* stream) {
  return qg::grouped_gemm(w, E, X, M, offs, Y, ws, ws_bytes, qg::as_stream(stream));
}
