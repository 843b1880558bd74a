// gemv.cu -- decode-path W4A16 GEMM for small M (M <= 32 per launch).
//
// Y[M,N] = X[M,K] . W[N,K]^T with W in the reference's packed layouts
// (titoatwork/qgemm-mx include/qgemm/pack.hpp:14-85) streamed straight from
// HBM once.  The path is HBM-bound, so the design goals are (1) every weight
// byte read exactly once with 16-byte coalesced loads, (2) an equal share of
// the weight stream for every warp on any (N, K), and (3) few ALU
// instructions per weight.
//
// Math: a swap-AB warp MMA (mma.sync m16n8k16, bf16 in, fp32 accumulate).
// The 16 weight rows of a tile are the MMA's M side, the (<= 8 per n-tile)
// activation rows its N side, so tensor cores do the multiply-accumulate and
// CUDA cores only dequantise.  Dequantisation is exact:
//   MXFP4  e2m1 * 2^(e8m0-127) is representable in bf16 (<= 2 significant
//          bits), so the block scale is folded into the bf16 operand;
//   NVFP4  e2m1 * e4m3 has <= 6 significant bits and lies in [2^-10, 2688],
//          so the block scale is folded too; the FP32 tensor scale is applied
//          to the FP32 result;
//   INT4   q in [-8,7] is exact in bf16; q * fp16-scale is not, so each
//          group's FP32 partial sum is scaled by the group scale (post-scale).
// Products of bf16 values are exact in the fp32 accumulator, so Y differs
// from the double-accumulated reference (ref_gemm.hpp:15-27) only by fp32
// summation order (and, for NVFP4, by the tensor scale being applied once per
// output instead of once per weight).
//
// K-slot mapping: an MMA reduces over 16 "k slots"; lane (g = lane/4,
// j = lane%4) owns slots {2j, 2j+1, 2j+8, 2j+9}.  Any bijection between slots
// and true k works as long as the weight (A) and activation (B) fragments use
// the same one, so each lane loads one contiguous 16-byte run of packed codes
// (32 k) per weight row and the matching 64-byte run of X: no shuffles.
//
// Schedule: stream-K.  The iteration space (row tile, 128-k chunk) is cut
// into one contiguous range per warp.  A tile finished inside one warp is
// stored directly; a tile split across warps leaves FP32 partial fragments in
// the workspace, and the warp whose atomic ticket shows it arrived last sums
// all contributors' partials in warp order (deterministic) and stores Y.
// Nobody waits on anybody: there is no spin loop in this kernel.
#include <cuda_bf16.h>

#include "common.cuh"

namespace qg {

constexpr int kWarpsPerCta = 4;
constexpr int kChunkK = 128;

struct GemvArgs {
  const uint8_t* data;
  const void* scales;
  const uint16_t* X;
  void* Y;
  int M, N, K;
  float ts;
  float* partials;      // [2 * W_total][R*NT*32*4] floats
  unsigned* counters;   // [tiles]
  long long T;          // iterations = tiles * C
  int C;                // chunks per tile
  int W_total;          // warps that own iterations
};

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t s) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(s));
  return d;
}
__device__ __forceinline__ uint32_t lop_or_and(uint32_t a, uint32_t b, uint32_t m) {
  // a | (b & m)
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xF8;" : "=r"(d) : "r"(a), "r"(b), "r"(m));
  return d;
}
__device__ __forceinline__ uint32_t hmul2_bf16(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t hsub2_bf16(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 16-byte streaming load of packed weights: read once, keep out of L1.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint2 ldg_stream8(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
// Activations: re-read by every warp, keep cached.
__device__ __forceinline__ uint4 ldg_keep(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

// 8 E2M1 codes (nibble i = k offset i) -> 4 bf16x2 words (c0,c1) (c2,c3)
// (c4,c5) (c6,c7), low half = even code.  Magnitudes through a byte-permute
// lookup of the bf16 bytes of {0,.5,1,1.5,2,3,4,6}; signs by replicating the
// code's sign bit into the high byte.
__device__ __forceinline__ void e2m1x8_to_bf16(uint32_t q, uint32_t (&o)[4]) {
  constexpr uint32_t LO_A = 0xC0800000u, LO_B = 0xC0804000u;  // low bytes
  constexpr uint32_t HI_A = 0x3F3F3F00u, HI_B = 0x40404040u;  // high bytes
  const uint32_t s0 = q & 0x7777u, s1 = (q >> 16) & 0x7777u;
  const uint32_t lo0 = prmt(LO_A, LO_B, s0), lo1 = prmt(LO_A, LO_B, s1);
  uint32_t hi0 = prmt(HI_A, HI_B, s0), hi1 = prmt(HI_A, HI_B, s1);
  const uint32_t q4 = q << 4;  // even codes' sign bits become byte msbs
  hi0 = lop_or_and(hi0, prmt(q4, q, 0xD9C8u), 0x80808080u);
  hi1 = lop_or_and(hi1, prmt(q4, q, 0xFBEAu), 0x80808080u);
  o[0] = prmt(lo0, hi0, 0x5140u);
  o[1] = prmt(lo0, hi0, 0x7362u);
  o[2] = prmt(lo1, hi1, 0x5140u);
  o[3] = prmt(lo1, hi1, 0x7362u);
}

// 8 INT4 codes -> 4 bf16x2 words (c0,c4) (c1,c5) (c2,c6) (c3,c7): the offset
// nibble u = q+8 is placed in the mantissa of bf16 128.0 and 136 subtracted.
__device__ __forceinline__ void int4x8_to_bf16(uint32_t q, uint32_t (&o)[4]) {
  const uint32_t u = q ^ 0x88888888u;
  constexpr uint32_t MAGIC = 0x43004300u, BIAS = 0x43084308u;  // 128, 136
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t w;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(w) : "r"(u >> (4 * i)), "r"(0x000F000Fu), "r"(MAGIC));
    o[i] = hsub2_bf16(w, BIAS);
  }
}

// bf16x2 broadcast of an exact bf16 value given as fp32.
__device__ __forceinline__ uint32_t bf16x2_of(float f) {
  const uint32_t b = f2u(f) >> 16;  // exact for the values used here
  return b | (b << 16);
}

template <int FMT, int NT, int R, bool F32OUT>
__global__ void __launch_bounds__(kWarpsPerCta * 32)
k_gemv(const GemvArgs a) {
  constexpr int TR = 16 * R;                  // rows per tile
  constexpr int FRAG = R * NT * 4;            // accumulator floats per lane
  const int lane = threadIdx.x & 31;
  const int w = blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
  if (w >= a.W_total) return;
  const int g = lane >> 2, j = lane & 3;
  const int M = a.M, N = a.N, K = a.K, C = a.C;
  const size_t rowb = (size_t)K / 2;          // packed bytes per row
  const long long start = (long long)w * a.T / a.W_total;
  const long long end = (long long)(w + 1) * a.T / a.W_total;

  float acc[R][NT][4];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[r][t][e] = 0.0f;

  // ---- per-iteration operands (double-buffered through registers) --------
  uint4 wq[R][2];
  uint32_t sc[R][2];  // raw scale bits per row (format dependent)
  uint32_t xf[NT][16];

  auto load = [&](long long it, uint4 (&wq_)[R][2], uint32_t (&sc_)[R][2], uint32_t (&xf_)[NT][16]) {
    const int tile = (int)(it / C), c = (int)(it % C);
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int n = tile * TR + 16 * r + 8 * h + g;
        wq_[r][h] = make_uint4(0, 0, 0, 0);
        sc_[r][h] = 0;
        if (n < N) {
          const uint8_t* row = a.data + (size_t)n * rowb + (size_t)c * (kChunkK / 2);
          if (FMT == 3) {
            const uint2 lo = ldg_stream8(row + 8 * j), hi = ldg_stream8(row + 32 + 8 * j);
            wq_[r][h] = make_uint4(lo.x, lo.y, hi.x, hi.y);
          } else {
            wq_[r][h] = ldg_stream(row + 16 * j);
          }
          if (FMT == 0) {
            sc_[r][h] = __ldg(static_cast<const uint8_t*>(a.scales) + (size_t)n * (K / 32) + c * 4 + j);
          } else if (FMT == 1) {
            sc_[r][h] = __ldg(reinterpret_cast<const uint16_t*>(static_cast<const uint8_t*>(a.scales) +
                                                                 (size_t)n * (K / 16) + c * 8 + 2 * j));
          } else if (FMT == 2) {
            sc_[r][h] = __ldg(static_cast<const uint16_t*>(a.scales) + (size_t)n * (K / 128) + c);
          } else {
            sc_[r][h] = __ldg(reinterpret_cast<const uint32_t*>(static_cast<const uint16_t*>(a.scales) +
                                                                 (size_t)n * (K / 64) + 2 * c));
          }
        }
      }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const int m = 8 * t + g;
      if (m < M) {
        const uint16_t* xr = a.X + (size_t)m * K + (size_t)c * kChunkK;
        uint4 v[4];
        if (FMT == 3) {
          v[0] = ldg_keep(xr + 16 * j); v[1] = ldg_keep(xr + 16 * j + 8);
          v[2] = ldg_keep(xr + 64 + 16 * j); v[3] = ldg_keep(xr + 64 + 16 * j + 8);
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q) v[q] = ldg_keep(xr + 32 * j + 8 * q);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          xf_[t][4 * q + 0] = v[q].x; xf_[t][4 * q + 1] = v[q].y;
          xf_[t][4 * q + 2] = v[q].z; xf_[t][4 * q + 3] = v[q].w;
        }
      } else {
#pragma unroll
        for (int q = 0; q < 16; ++q) xf_[t][q] = 0u;
      }
    }
  };

  auto store_tile = [&](int tile, float (&v)[R][NT][4]) {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int n = tile * TR + 16 * r + g + ((e & 2) ? 8 : 0);
          const int m = 8 * t + 2 * j + (e & 1);
          if (n < N && m < M) {
            float y = v[r][t][e];
            if (FMT == 1) y *= a.ts;
            if (F32OUT) static_cast<float*>(a.Y)[(size_t)m * N + n] = y;
            else static_cast<__nv_bfloat16*>(a.Y)[(size_t)m * N + n] = __float2bfloat16_rn(y);
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
      __threadfence();
      __syncwarp();
      unsigned ticket = 0;
      const long long t0 = (long long)tile * C, t1 = t0 + C - 1;
      const int w_lo = (int)(((t0 + 1) * a.W_total - 1) / a.T);
      const int w_hi = (int)(((t1 + 1) * a.W_total - 1) / a.T);
      if (lane == 0) ticket = atomicAdd(a.counters + tile, 1u);
      ticket = __shfl_sync(0xFFFFFFFFu, ticket, 0);
      if ((int)ticket == w_hi - w_lo) {  // last contributor: reduce in warp order
        __threadfence();
        float sum[R][NT][4];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int t = 0; t < NT; ++t)
#pragma unroll
            for (int e = 0; e < 4; ++e) sum[r][t][e] = 0.0f;
        for (int ww = w_lo; ww <= w_hi; ++ww) {
          const float4* src = reinterpret_cast<const float4*>(a.partials) + slot_of(ww, tile) * (FRAG / 4) * 32;
#pragma unroll
          for (int r = 0; r < R; ++r)
#pragma unroll
            for (int t = 0; t < NT; ++t) {
              const float4 p = __ldcg(src + ((r * NT + t) * 32 + lane));
              sum[r][t][0] += p.x; sum[r][t][1] += p.y; sum[r][t][2] += p.z; sum[r][t][3] += p.w;
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

  if (start >= end) return;
  load(start, wq, sc, xf);
  long long seg_begin = start;
  for (long long it = start; it < end; ++it) {
    const int tile = (int)(it / C), c = (int)(it % C);
    uint4 cw[R][2];
    uint32_t cs[R][2];
    uint32_t cx[NT][16];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      cw[r][0] = wq[r][0]; cw[r][1] = wq[r][1]; cs[r][0] = sc[r][0]; cs[r][1] = sc[r][1];
    }
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int q = 0; q < 16; ++q) cx[t][q] = xf[t][q];
    if (it + 1 < end) load(it + 1, wq, sc, xf);

    if (FMT >= 2) {  // INT4 operands are in (c_i, c_i+4) pair order
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t x0 = cx[t][4 * q], x1 = cx[t][4 * q + 1], x2 = cx[t][4 * q + 2], x3 = cx[t][4 * q + 3];
          cx[t][4 * q + 0] = prmt(x0, x2, 0x5410u);
          cx[t][4 * q + 1] = prmt(x0, x2, 0x7632u);
          cx[t][4 * q + 2] = prmt(x1, x3, 0x5410u);
          cx[t][4 * q + 3] = prmt(x1, x3, 0x7632u);
        }
    }

    // per-row bf16x2 scale multipliers (MXFP4: one block, NVFP4: two blocks)
    uint32_t smul[R][2][2];
    bool slow[R][2];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        slow[r][h] = false;
        if (FMT == 0) {
          const uint32_t sb = cs[r][h] & 0xFFu;
          slow[r][h] = sb <= 1u;
          const uint32_t b = (sb == 0xFFu) ? 0x7FC0u : (sb << 7);
          smul[r][h][0] = smul[r][h][1] = b | (b << 16);
        } else if (FMT == 1) {
          smul[r][h][0] = bf16x2_of(e4m3_decode(cs[r][h] & 0xFFu));
          smul[r][h][1] = bf16x2_of(e4m3_decode((cs[r][h] >> 8) & 0xFFu));
        }
      }

    float tmp[R][NT][4];
    if (FMT >= 2) {
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
          for (int e = 0; e < 4; ++e) tmp[r][t][e] = 0.0f;
    }

#pragma unroll
    for (int qw = 0; qw < 4; ++qw) {  // 8 codes of each row per step = 2 MMAs
      uint32_t A[R][2][4];
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t q = (qw == 0) ? cw[r][h].x : (qw == 1) ? cw[r][h].y : (qw == 2) ? cw[r][h].z : cw[r][h].w;
          if (FMT >= 2) {
            int4x8_to_bf16(q, A[r][h]);
          } else {
            e2m1x8_to_bf16(q, A[r][h]);
            const uint32_t m2 = smul[r][h][FMT == 1 ? (qw >> 1) : 0];
            if (FMT == 0 && slow[r][h]) {
              const float s = e8m0_decode(cs[r][h]);
#pragma unroll
              for (int p = 0; p < 4; ++p) {
                const float f0 = e2m1_decode(q >> (8 * p)) * s, f1 = e2m1_decode(q >> (8 * p + 4)) * s;
                A[r][h][p] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(f0)) |
                             ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(f1)) << 16);
              }
            } else {
#pragma unroll
              for (int p = 0; p < 4; ++p) A[r][h][p] = hmul2_bf16(A[r][h][p], m2);
            }
          }
        }
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        const int i = 2 * qw + s;  // MMA index within the chunk
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            float (&d)[4] = (FMT >= 2) ? tmp[r][t] : acc[r][t];
            mma_bf16(d, A[r][0][2 * s], A[r][1][2 * s], A[r][0][2 * s + 1], A[r][1][2 * s + 1],
                     cx[t][2 * i], cx[t][2 * i + 1]);
          }
      }
      if (FMT == 3 && qw == 1) {  // end of the first 64-k group
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const float s0 = fp16_bits_to_float(cs[r][0] & 0xFFFFu), s1 = fp16_bits_to_float(cs[r][1] & 0xFFFFu);
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            acc[r][t][0] = fmaf(s0, tmp[r][t][0], acc[r][t][0]);
            acc[r][t][1] = fmaf(s0, tmp[r][t][1], acc[r][t][1]);
            acc[r][t][2] = fmaf(s1, tmp[r][t][2], acc[r][t][2]);
            acc[r][t][3] = fmaf(s1, tmp[r][t][3], acc[r][t][3]);
            tmp[r][t][0] = tmp[r][t][1] = tmp[r][t][2] = tmp[r][t][3] = 0.0f;
          }
        }
      }
    }
    if (FMT >= 2) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const uint32_t b0 = (FMT == 3) ? (cs[r][0] >> 16) : cs[r][0];
        const uint32_t b1 = (FMT == 3) ? (cs[r][1] >> 16) : cs[r][1];
        const float s0 = fp16_bits_to_float(b0 & 0xFFFFu), s1 = fp16_bits_to_float(b1 & 0xFFFFu);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          acc[r][t][0] = fmaf(s0, tmp[r][t][0], acc[r][t][0]);
          acc[r][t][1] = fmaf(s0, tmp[r][t][1], acc[r][t][1]);
          acc[r][t][2] = fmaf(s1, tmp[r][t][2], acc[r][t][2]);
          acc[r][t][3] = fmaf(s1, tmp[r][t][3], acc[r][t][3]);
        }
      }
    }

    const bool tile_ends = (c == C - 1) || (it + 1 == end);
    if (tile_ends) {
      const bool full = ((seg_begin % C) == 0) && (c == C - 1);
      flush(tile, full);
      seg_begin = it + 1;
    }
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

struct GemvPlan {
  int fmt = 0, nt = 1, r = 2;
  int tiles = 0, C = 0;
  long long T = 0;
  int grid = 0, W_total = 0;
  size_t slot_floats = 0;
  size_t partial_bytes = 0, counter_bytes = 0;
};

template <int FMT, int NT, int R, bool F32>
static int occupancy_of() {
  static int occ = 0;
  if (occ == 0) {
    int v = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, k_gemv<FMT, NT, R, F32>, kWarpsPerCta * 32, 0) != cudaSuccess || v < 1)
      v = 1;
    occ = v;
  }
  return occ;
}

static int fmt_code(int32_t format) {
  switch (format) {
    case QGEMM_FMT_MXFP4: return 0;
    case QGEMM_FMT_NVFP4: return 1;
    case QGEMM_FMT_INT4_G128: return 2;
    case QGEMM_FMT_INT4_G64: return 3;
  }
  return -1;
}

static void pick_tile(int M, int* nt, int* r) {
  if (M <= 8) { *nt = 1; *r = 2; }
  else if (M <= 16) { *nt = 2; *r = 2; }
  else { *nt = 4; *r = 1; }
}

// Occupancy is a property of the compiled kernel; approximate with the
// bf16-out instance of each (FMT, NT, R) (both outputs use the same registers
// to within a few).
template <int FMT>
static int occ_for(int nt, int r) {
  if (nt == 1) return occupancy_of<FMT, 1, 2, false>();
  if (nt == 2) return occupancy_of<FMT, 2, 2, false>();
  return occupancy_of<FMT, 4, 1, false>();
}

qgemm_status_t gemv_plan(const qgemm_weights_t* w, int M, GemvPlan* p) {
  const int f = fmt_code(w->format);
  if (f < 0) return fail(QGEMM_ERR_INVALID_ARG, "gemm: unknown format %d", (int)w->format);
  if (w->K == 0 || w->N == 0) return fail(QGEMM_ERR_INVALID_ARG, "gemm: empty weight matrix");
  if (w->K % kChunkK != 0)
    return fail(QGEMM_ERR_UNSUPPORTED_SHAPE, "gemm: K=%zu is not a multiple of %d", w->K, kChunkK);
  if (w->K > (size_t)INT32_MAX / 2 || w->N > (size_t)INT32_MAX / 2)
    return fail(QGEMM_ERR_UNSUPPORTED_SHAPE, "gemm: N or K too large");
  DevProps dp;
  qgemm_status_t st = device_props(&dp);
  if (st != QGEMM_OK) return st;
  const int mb = M > 32 ? 32 : M;
  pick_tile(mb, &p->nt, &p->r);
  p->fmt = f;
  p->tiles = (int)((w->N + 16 * p->r - 1) / (16 * p->r));
  p->C = (int)(w->K / kChunkK);
  p->T = (long long)p->tiles * p->C;
  int occ = 1;
  switch (f) {
    case 0: occ = occ_for<0>(p->nt, p->r); break;
    case 1: occ = occ_for<1>(p->nt, p->r); break;
    case 2: occ = occ_for<2>(p->nt, p->r); break;
    default: occ = occ_for<3>(p->nt, p->r); break;
  }
  long long warps = (long long)dp.sm_count * occ * kWarpsPerCta;
  if (warps > p->T) warps = p->T;
  p->W_total = (int)warps;
  p->grid = (int)((warps + kWarpsPerCta - 1) / kWarpsPerCta);
  p->slot_floats = (size_t)p->r * p->nt * 4 * 32;
  p->partial_bytes = 2 * (size_t)p->W_total * p->slot_floats * sizeof(float);
  p->counter_bytes = ((size_t)p->tiles * sizeof(unsigned) + 255) & ~(size_t)255;
  return QGEMM_OK;
}

template <int FMT, bool F32>
static void launch_fmt(const GemvPlan& p, const GemvArgs& a, cudaStream_t s) {
  if (p.nt == 1) k_gemv<FMT, 1, 2, F32><<<p.grid, kWarpsPerCta * 32, 0, s>>>(a);
  else if (p.nt == 2) k_gemv<FMT, 2, 2, F32><<<p.grid, kWarpsPerCta * 32, 0, s>>>(a);
  else k_gemv<FMT, 4, 1, F32><<<p.grid, kWarpsPerCta * 32, 0, s>>>(a);
}

template <bool F32>
static void launch_gemv(const GemvPlan& p, const GemvArgs& a, cudaStream_t s) {
  switch (p.fmt) {
    case 0: launch_fmt<0, F32>(p, a, s); break;
    case 1: launch_fmt<1, F32>(p, a, s); break;
    case 2: launch_fmt<2, F32>(p, a, s); break;
    default: launch_fmt<3, F32>(p, a, s); break;
  }
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Workspace layout: [counters (256-byte padded)][partials].
qgemm_status_t gemm_decode(const qgemm_weights_t* w, const uint16_t* X, int M, void* Y, bool f32,
                           void* ws, size_t ws_bytes, cudaStream_t s) {
  if (!w || !X || !Y) return fail(QGEMM_ERR_INVALID_ARG, "gemm: null pointer");
  if (M < 1) return fail(QGEMM_ERR_INVALID_ARG, "gemm: M must be >= 1");
  if (!w->data || !w->scales) return fail(QGEMM_ERR_INVALID_ARG, "gemm: null weight pointer");
  if (w->reserved != 0) return fail(QGEMM_ERR_INVALID_ARG, "gemm: reserved field must be 0");
  if (w->format == QGEMM_FMT_NVFP4 && !(std::isfinite(w->tensor_scale)))
    return fail(QGEMM_ERR_INVALID_ARG, "gemm: NVFP4 tensor_scale must be finite");
  GemvPlan p;
  qgemm_status_t st = gemv_plan(w, M, &p);
  if (st != QGEMM_OK) return st;
  if (!al16(w->data) || !al16(X) || (w->format == QGEMM_FMT_NVFP4 && (reinterpret_cast<uintptr_t>(w->scales) & 1u)) ||
      ((w->format == QGEMM_FMT_INT4_G128 || w->format == QGEMM_FMT_INT4_G64) &&
       (reinterpret_cast<uintptr_t>(w->scales) & 3u)))
    return fail(QGEMM_ERR_INVALID_ARG, "gemm: data and X must be 16-byte aligned, scales naturally aligned");
  const size_t need = p.counter_bytes + p.partial_bytes;
  if (!ws || ws_bytes < need)
    return fail(QGEMM_ERR_WORKSPACE, "gemm: workspace of %zu bytes needed, %zu given", need, ws_bytes);
  GemvArgs a;
  a.data = w->data; a.scales = w->scales; a.N = (int)w->N; a.K = (int)w->K;
  a.ts = w->tensor_scale;
  a.counters = static_cast<unsigned*>(ws);
  a.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + p.counter_bytes);
  a.T = p.T; a.C = p.C; a.W_total = p.W_total;
  for (int m0 = 0; m0 < M; m0 += 32) {
    const int mb = (M - m0) < 32 ? (M - m0) : 32;
    GemvPlan pb = p;
    pick_tile(mb, &pb.nt, &pb.r);
    if (pb.nt != p.nt) {  // last partial block may use a narrower tile
      st = gemv_plan(w, mb, &pb);
      if (st != QGEMM_OK) return st;
      if (pb.counter_bytes + pb.partial_bytes > ws_bytes)
        return fail(QGEMM_ERR_WORKSPACE, "gemm: workspace too small for the tail block");
      a.T = pb.T; a.C = pb.C; a.W_total = pb.W_total;
      a.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + pb.counter_bytes);
    }
    a.M = mb;
    a.X = X + (size_t)m0 * w->K;
    a.Y = f32 ? (void*)(static_cast<float*>(Y) + (size_t)m0 * w->N)
              : (void*)(static_cast<uint16_t*>(Y) + (size_t)m0 * w->N);
    if (f32) launch_gemv<true>(pb, a, s);
    else launch_gemv<false>(pb, a, s);
    QG_LAUNCH_RET();
  }
  return QGEMM_OK;
}

size_t gemm_decode_workspace(const qgemm_weights_t* w, int M) {
  GemvPlan p;
  if (!w || gemv_plan(w, M, &p) != QGEMM_OK) return 0;
  size_t need = p.counter_bytes + p.partial_bytes;
  if (M > 32 && (M % 32) != 0) {
    GemvPlan q;
    if (gemv_plan(w, M % 32, &q) == QGEMM_OK && q.counter_bytes + q.partial_bytes > need)
      need = q.counter_bytes + q.partial_bytes;
  }
  return need;
}

}  // namespace qg

using namespace qg;

extern "C" {

size_t qgemm_workspace_size(const qgemm_weights_t* w, int32_t M) { return gemm_decode_workspace(w, M); }

qgemm_status_t qgemm_workspace_init(void* ws, size_t ws_bytes, void* stream) {
  if (!ws && ws_bytes) return fail(QGEMM_ERR_INVALID_ARG, "workspace_init: null pointer");
  if (ws_bytes) QG_CUDA_RET(cudaMemsetAsync(ws, 0, ws_bytes, as_stream(stream)));
  return QGEMM_OK;
}

qgemm_status_t qgemm_gemm_w4a16(const qgemm_weights_t* w, const uint16_t* X, int32_t M, uint16_t* Y,
                                void* ws, size_t ws_bytes, void* stream) {
  return gemm_decode(w, X, M, Y, false, ws, ws_bytes, as_stream(stream));
}

qgemm_status_t qgemm_gemm_w4a16_f32(const qgemm_weights_t* w, const uint16_t* X, int32_t M, float* Y,
                                    void* ws, size_t ws_bytes, void* stream) {
  return gemm_decode(w, X, M, Y, true, ws, ws_bytes, as_stream(stream));
}

}  // extern "C"
