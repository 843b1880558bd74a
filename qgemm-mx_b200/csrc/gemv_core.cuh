// gemv_core.cuh -- the decode kernels' exact per-format arithmetic: warp-MMA
// wrappers, code widening (E2M1 / INT4 -> f16), scale decoding, and one
// 128-k chunk of swap-AB mma.sync work (chunk_mma) shared by the LDG-fed and
// the TMA-fed decode kernels.  The register layouts chunk_mma expects are
// documented at the top of gemv.cu (K-slot mapping).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"

namespace qg {

// Position of 8-f16 chunk idx of X row m in the staged X tile (the image
// k_xprep writes, layout 2 for MXFP4 and 3 for NVFP4): a per-row permutation within each aligned
// group of 8 chunks chosen so that the consumers' 128-bit fragment loads
// (two rows and four lanes per phase) hit eight distinct bank groups.
__host__ __device__ __forceinline__ int xg_pos(int fmt, int idx, int m) {
  const int f = fmt == 0 ? ((m & 1) << 2) : ((((idx >> 3) & 1) << 1) ^ (m & 1));
  return (idx & ~7) | ((idx ^ f) & 7);
}

// ---------------------------------------------------------------------------
// small PTX helpers
// ---------------------------------------------------------------------------

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// d = A.B (accumulator starts at zero)
__device__ __forceinline__ void mma_f16_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  const float z = 0.0f;
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
}

// Split-tile ticket: atomicAdd(p, 1) with acquire-release semantics at GPU
// scope.  Taken by one thread after a barrier of the threads that stored the
// partial sums (the release is cumulative over what the barrier ordered), it
// publishes those stores; for the last contributor its acquire orders the
// partial loads that follow the next barrier.
__device__ __forceinline__ unsigned ticket_acq_rel(unsigned* p) {
  unsigned old;
  asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(old) : "l"(p) : "memory");
  return old;
}

__device__ __forceinline__ uint4 ldg_stream16(const void* p) {  // read once: skip L1
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ uint2 ldg_stream8(const void* p) {
  uint2 v;
  asm("ld.global.nc.L1::no_allocate.L2::256B.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
// 4-byte pieces of one 16-byte block: allocate in L1 so the 3 sibling loads
// of the same sector hit there.
__device__ __forceinline__ uint32_t ldg_first4(const void* p) {
  uint32_t v;
  asm("ld.global.nc.L1::evict_first.L2::256B.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ uint4 ldg_keep16(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

// byte t of q (codes 2t, 2t+1) -> f16x2 (low half = even code)
__device__ __forceinline__ void e2m1x8_to_f16(uint32_t q, uint32_t (&o)[4]) {
  asm("{ .reg .b8 b0, b1, b2, b3;\n"
      "  mov.b32 {b0, b1, b2, b3}, %4;\n"
      "  cvt.rn.f16x2.e2m1x2 %0, b0;\n"
      "  cvt.rn.f16x2.e2m1x2 %1, b1;\n"
      "  cvt.rn.f16x2.e2m1x2 %2, b2;\n"
      "  cvt.rn.f16x2.e2m1x2 %3, b3; }\n"
      : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
      : "r"(q));
}

__device__ __forceinline__ uint32_t hmul2_f16(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// 8 INT4 codes -> f16x2 words (c0,c4) (c1,c5) (c2,c6) (c3,c7).  With
// u = q ^ 0x8 (= value + 8), nibble u placed in the mantissa of f16 1024
// gives 1024 + u, or 1024 + 16u when taken from the upper nibble of a byte;
// one subtract / fused multiply-add recovers the signed value exactly.
__device__ __forceinline__ void int4x8_to_f16(uint32_t q, uint32_t (&o)[4]) {
  const uint32_t lo = q ^ 0x88888888u, hi = lo >> 8;
  constexpr uint32_t MAGIC = 0x64006400u;
  uint32_t w0, w1, w2, w3;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(w0) : "r"(lo), "r"(0x000F000Fu), "r"(MAGIC));
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(w1) : "r"(lo), "r"(0x00F000F0u), "r"(MAGIC));
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(w2) : "r"(hi), "r"(0x000F000Fu), "r"(MAGIC));
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(w3) : "r"(hi), "r"(0x00F000F0u), "r"(MAGIC));
  constexpr uint32_t SUB = 0x64086408u;    // 1032
  constexpr uint32_t K16 = 0x2C002C00u;    // 1/16
  constexpr uint32_t NEG72 = 0xD480D480u;  // -72
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(o[0]) : "r"(w0), "r"(SUB));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(o[1]) : "r"(w1), "r"(K16), "r"(NEG72));
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(o[2]) : "r"(w2), "r"(SUB));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(o[3]) : "r"(w3), "r"(K16), "r"(NEG72));
}

// True if any byte of v equals 0x00 or 0xFF (classic zero-byte test on v and ~v).
__device__ __forceinline__ bool has_00_or_ff(uint32_t v) {
  const uint32_t nv = ~v;
  return (((v - 0x01010101u) & ~v) | ((nv - 0x01010101u) & ~nv)) & 0x80808080u;
}

// 2^(b-127) for an E8M0 byte b in 1..254 (callers route 0x00 / 0xFF through
// the exact e8m0_decode).
__device__ __forceinline__ float e8m0_fast(uint32_t word, int byte) {
  return u2f(((word >> (8 * byte)) & 0xFFu) << 23);
}

// f16x2 broadcast of each of the two E4M3 bytes in the low half of v, exact
// for normal E4M3 codes (exponent field 1..15, not the NaN code): f16 keeps
// the sign, rebiases the exponent by +8 and widens the mantissa.  Returns
// false when either byte is zero, subnormal or NaN (callers then use the
// exact path).
__device__ __forceinline__ bool e4m3x2_to_f16x2_fast(uint32_t v, uint32_t& lo, uint32_t& hi) {
  const uint32_t e0 = (v >> 3) & 0xFu, e1 = (v >> 11) & 0xFu;
  const uint32_t m0 = v & 0x7Fu, m1 = (v >> 8) & 0x7Fu;
  const bool ok = e0 != 0 && e1 != 0 && m0 != 0x7Fu && m1 != 0x7Fu;
  const uint32_t h0 = ((v & 0x80u) << 8) | ((m0 << 7) + 0x2000u);
  const uint32_t h1 = ((v & 0x8000u)) | ((m1 << 7) + 0x2000u);
  lo = h0 | (h0 << 16);
  hi = h1 | (h1 << 16);
  return ok;
}

__device__ __forceinline__ uint32_t f16x2_of(float f) {
  const uint32_t h = (uint32_t)__half_as_ushort(__float2half_rn(f));  // exact for e4m3 values
  return h | (h << 16);
}

// One 128-k chunk for R 16-row tiles and NT 8-column activation tiles:
//   cw[r][h][q]  packed words of weight rows g (h = 0) and g + 8 (h = 1)
//   cs[r][h]     their scale bits for the chunk
//   cx[t][16]    the X fragment words of activation rows 8t + g
// FMT: 0 MXFP4, 1 NVFP4, 2 INT4 g128, 3 INT4 g64.
// SCALES (FP4 formats): how block scales are decoded.
//   kScalesCheck  fast decode, and the exact decoder for the whole warp when
//                 the chunk holds a byte the fast decode does not cover
//                 (found by a per-chunk search);
//   kScalesFast   fast decode only: the weights are in the scale-checked
//                 layout, so no such byte occurs.
constexpr int kScalesCheck = 0, kScalesFast = 1;
template <int FMT, int R, int NT, int SCALES = kScalesCheck>
__device__ __forceinline__ void chunk_mma(float (&acc)[R][NT][4], const uint32_t (&cw)[R][2][4],
                                          const uint32_t (&cs)[R][2], const uint32_t (&cx)[NT][16]) {
  if constexpr (FMT == 0) {
    // block b of the chunk = MMAs (b,0), (b,1); post-scale by 2^(e8m0-127).
    // The chunk's 8 R scales are decoded before the MMA loop so that loop is
    // straight-line code; a 0x00 (2^-127) or 0xFF (NaN) byte anywhere in the
    // warp's chunk sends the whole warp through the exact decoder once.
    float sc[R][2][4];
    bool special = false;
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (SCALES == kScalesCheck) special |= has_00_or_ff(cs[r][h]);
#pragma unroll
        for (int b = 0; b < 4; ++b) sc[r][h][b] = e8m0_fast(cs[r][h], b);
      }
    if (SCALES == kScalesCheck && __any_sync(0xFFFFFFFFu, special)) {
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int b = 0; b < 4; ++b) sc[r][h][b] = e8m0_decode((cs[r][h] >> (8 * b)) & 0xFFu);
    }
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      uint32_t A[R][2][4];
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int h = 0; h < 2; ++h) e2m1x8_to_f16(cw[r][h][b], A[r][h]);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float s0 = sc[r][0][b], s1 = sc[r][1][b];
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          float tmp[4];
          mma_f16_z(tmp, A[r][0][0], A[r][1][0], A[r][0][1], A[r][1][1], cx[t][4 * b + 0], cx[t][4 * b + 1]);
          mma_f16(tmp, A[r][0][2], A[r][1][2], A[r][0][3], A[r][1][3], cx[t][4 * b + 2], cx[t][4 * b + 3]);
          acc[r][t][0] = fmaf(s0, tmp[0], acc[r][t][0]);
          acc[r][t][1] = fmaf(s0, tmp[1], acc[r][t][1]);
          acc[r][t][2] = fmaf(s1, tmp[2], acc[r][t][2]);
          acc[r][t][3] = fmaf(s1, tmp[3], acc[r][t][3]);
        }
      }
    }
  } else if constexpr (FMT == 1) {
    // words 0,1 -> block 2j, words 2,3 -> block 2j+1; fold e4m3 into f16.
    // Zero, subnormal or NaN scale codes anywhere in the warp's chunk send
    // the whole warp through the exact decoder (one uniform branch).
    uint32_t sw[R][2][2];
    bool slow = false;
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int h = 0; h < 2; ++h) slow |= !e4m3x2_to_f16x2_fast(cs[r][h], sw[r][h][0], sw[r][h][1]);
    if (SCALES == kScalesCheck && __any_sync(0xFFFFFFFFu, slow)) {
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          sw[r][h][0] = f16x2_of(e4m3_decode(cs[r][h] & 0xFFu));
          sw[r][h][1] = f16x2_of(e4m3_decode((cs[r][h] >> 8) & 0xFFu));
        }
    }
#pragma unroll
    for (int qw = 0; qw < 4; ++qw) {
      uint32_t A[R][2][4];
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          e2m1x8_to_f16(cw[r][h][qw], A[r][h]);
          const uint32_t m2 = sw[r][h][qw >> 1];
#pragma unroll
          for (int p = 0; p < 4; ++p) A[r][h][p] = hmul2_f16(A[r][h][p], m2);
        }
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        const int i = 2 * qw + s;
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int t = 0; t < NT; ++t)
            mma_f16(acc[r][t], A[r][0][2 * s], A[r][1][2 * s], A[r][0][2 * s + 1], A[r][1][2 * s + 1],
                    cx[t][2 * i], cx[t][2 * i + 1]);
      }
    }
  } else {
    // INT4: FP32 partial per group, post-scaled by the FP16 group scale
    float tmp[R][NT][4];
#pragma unroll
    for (int qw = 0; qw < 4; ++qw) {
      uint32_t A[R][2][4];
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int h = 0; h < 2; ++h) int4x8_to_f16(cw[r][h][qw], A[r][h]);
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        const int i = 2 * qw + s;
        const bool first = (FMT == 2) ? (i == 0) : (i == 0 || i == 4);
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            if (first)
              mma_f16_z(tmp[r][t], A[r][0][2 * s], A[r][1][2 * s], A[r][0][2 * s + 1], A[r][1][2 * s + 1],
                        cx[t][2 * i], cx[t][2 * i + 1]);
            else
              mma_f16(tmp[r][t], A[r][0][2 * s], A[r][1][2 * s], A[r][0][2 * s + 1], A[r][1][2 * s + 1],
                      cx[t][2 * i], cx[t][2 * i + 1]);
          }
      }
      if ((FMT == 3 && qw == 1) || qw == 3) {  // end of a group
        const int sh = (FMT == 3 && qw == 3) ? 16 : 0;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const float s0 = __half2float(__ushort_as_half((unsigned short)((cs[r][0] >> sh) & 0xFFFFu)));
          const float s1 = __half2float(__ushort_as_half((unsigned short)((cs[r][1] >> sh) & 0xFFFFu)));
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            acc[r][t][0] = fmaf(s0, tmp[r][t][0], acc[r][t][0]);
            acc[r][t][1] = fmaf(s0, tmp[r][t][1], acc[r][t][1]);
            acc[r][t][2] = fmaf(s1, tmp[r][t][2], acc[r][t][2]);
            acc[r][t][3] = fmaf(s1, tmp[r][t][3], acc[r][t][3]);
          }
        }
      }
    }
  }

}

}  // namespace qg
