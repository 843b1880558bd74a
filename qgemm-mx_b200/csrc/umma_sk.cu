// umma_sk.cu -- persistent stream-K tcgen05 W4A16 GEMM for 32 <= M < 128
// (MXFP4; NVFP4 and INT4 g128 / g64 from M = 17; K % 256 == 0; weights of
// at least 2^26 codes).
//
// Y[M,N] = X[M,K] . W[N,K]^T with W in the reference's packed layouts
// (titoatwork/qgemm-mx include/qgemm/pack.hpp:14-85); X arrives as the f16
// copy with per-row power-of-two factors xs[m] made by k_xprep (gemv.cu).
//
// Swap-AB: 128 weight rows are the UMMA M side, BN (32 / 64) activation rows
// the N side; the FP32 accumulator D = Y^T tile lives in TMEM.  The
// dequantised operand never touches shared memory: each dequant thread widens
// its row's codes with cvt.rn.f16x2.e2m1x2, folds the block scale with one
// f16x2 multiply and writes TMEM with tcgen05.st; the MMA takes A from TMEM
// and B (X) from shared memory (kind::f16, TS form).
//   NVFP4  e2m1 * e4m3 is exact in f16; the FP32 tensor scale is applied in
//          the epilogue.
//   MXFP4  2^(e8m0-127) is folded relative to a per-row, per-segment base
//          b = max(e8m0) - 140 over the segment's blocks, so every factor is
//          <= 2^13 and e2m1 * factor <= 49152 fits f16; products are exact
//          while e8m0 >= max - 36; the next binade rounds to f16's smallest
//          subnormals and blocks below it are flushed to zero.  The epilogue
//          multiplies row n by 2^b.
//   INT4   q (exact in f16) times the FP16 group scale, rounded to f16
//          (exact while q s needs at most 11 significant bits); rows whose
//          largest scale field e over the segment could overflow f16 are
//          folded by 2^-b, b = max(0, e - 26), multiplied back in the
//          epilogue.  Codes widen in (c_i, c_i+4) pairs, the order of X from
//          k_xprep with the INT4 pair permutation.
//
// Schedule: one CTA per SM, stream-K.  The iteration space (tile, 256-k step)
// is cut into one contiguous range per CTA; a CTA walks its range as
// segments (a tile's run of steps).  A segment covering a whole tile is
// stored directly; a partial segment parks its FP32 tile (already scaled by
// its row factors) in the workspace, and the CTA whose ticket shows it
// arrived last sums all contributors in CTA order (deterministic).
//
// Pacing.  A tcgen05.mma with N <= 64 occupies the tensor pipe ~45 cycles
// whatever N, and the issuing thread blocks for that long; 128 weight rows x
// 256 k (16 MMAs, ~720 cycles) is also what HBM delivers to one SM in that
// time.  So each barrier round trip is amortised over 16 MMAs, and the packed
// W ring is released by the dequant warps as soon as they have read a stage
// (not by the MMAs), so its depth covers HBM latency on its own.
//
// Warp roles (768 threads):
//   warp 0        X producer: one linear bulk copy per step of the X tile
//                 (four BN x 64 f16 sub-tiles, already in the 128-byte
//                 swizzled image k_xprep wrote) into the X ring.
//   warps 1, 2    W producers, alternate steps: one packed-W box per step by
//                 TMA (128 rows x 128 B, 128-byte swizzle) into the W ring.
//                 (A TMA-issuing thread streams about one box row per 8
//                 cycles; two keep ahead of HBM.)  No multicast anywhere.
//   warp 3        TMEM allocation (512 columns) and the MMA issuer: 16
//                 tcgen05.mma (K = 16) per step into accumulator buffer
//                 seg & 1; commits release the X stage, the TMEM A stage and,
//                 at a segment's end, the accumulator.
//   warps 4..19   dequant: warp w covers TMEM lane quadrant w % 4 (32 weight
//                 rows) and 64-k slice (w - 4) / 4 of each step.
//   warps 20..23  epilogue: drain accumulator buffers (double-buffered, so
//                 the next segment's MMAs overlap the drain), split-tile
//                 tickets and reductions; ahead of each segment they compute
//                 the MXFP4 row bases and INT4 row folds (or prefetch NVFP4
//                 scales into L2).
// TMEM: [acc 0 | acc 1 | AST A stages of 128 columns (256 k, f16 pairs)].
//
// Every mbarrier wait is bounded (tc.cuh); on timeout the kernel sets
// g_sk_fault, lets copies in flight land, frees TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "gemv_core.cuh"
#include "tc.cuh"
#include "tp.cuh"

namespace qg {

__device__ unsigned g_sk_fault = 0;

constexpr int kSkBK = 256;                               // k per pipeline step
constexpr int kSkRows = 128;                             // weight rows per tile
constexpr int kSkXProd = 0;
constexpr int kSkWProd0 = 1, kSkWProds = 2;
constexpr int kSkMmaWarp = 3;
constexpr int kSkDqWarp0 = 4;
constexpr int kSkDqWarps = 16;
constexpr int kSkEpiWarps = 4;
constexpr int kSkEpiWarp0 = kSkDqWarp0 + kSkDqWarps;
constexpr int kSkThreads = 32 * (kSkEpiWarp0 + kSkEpiWarps);  // 768

template <int BN>
struct SkCfg {
  static constexpr int W_CODES = kSkRows * kSkBK / 2;    // 16 KB packed codes
  static constexpr int W_SCALE_ROW = 16;                 // scale bytes per row per step (at most 16)
  static constexpr int W_STAGE = W_CODES + kSkRows * W_SCALE_ROW;
  static constexpr int XBOX = BN * 128;                  // 64 k of X (f16), one swizzle row per activation row
  static constexpr int X_STAGE = 4 * XBOX;
  static constexpr int SX = BN == 32 ? 4 : 3;            // X ring depth
  static constexpr int SW = BN == 32 ? 8 : 6;            // W ring depth (even: two W producers)
  static constexpr int AST = (512 - 2 * BN) / 128;       // TMEM A stages
  static constexpr int NBAR = 2 * SX + 2 * SW + 2 * AST + 8;
  static constexpr int BYTES = 1024 + SX * X_STAGE + SW * W_STAGE + NBAR * 8 + 2 * kSkRows * 4 + 16;
  static_assert(BYTES <= 232448, "shared memory");
  static_assert(2 * BN + 128 * AST <= 512, "TMEM columns");
  static_assert(SW % kSkWProds == 0, "each W producer owns whole stages");
};

// scale bytes per weight row per 256-k step: E8M0 / 32, E4M3 / 16, FP16 / 128, FP16 / 64
__host__ __device__ constexpr int sk_scale_bytes(int fmt) { return fmt == 0 ? 8 : fmt == 1 ? 16 : fmt == 2 ? 4 : 8; }

struct SkArgs {
  const uint8_t* scales;
  const uint8_t* xsw;   // X in the swizzled operand layout (k_xprep with swz_bn = BN)
  void* Y;
  const float* xs;
  float* partials;      // [2 * G][128][BN] FP32, scaled by the row factors
  unsigned* counters;   // [tiles] tickets (start and end at zero)
  long long T;          // tiles * KS
  int M, N, K;
  int tiles_n;          // tile t -> rows (t % tiles_n) * 128, activations (t / tiles_n) * BN
  int KS;               // steps per tile (K / 256)
  int G;                // CTAs
  float ts;
  TpOut tp;             // world > 0: store into every rank's Y_full, then tp_finish
};

// Largest E8M0 byte among nbytes scale bytes at p, with NaN codes (0xFF)
// counted as 0.  p is 4-byte aligned and nbytes a multiple of 4.
__device__ __forceinline__ int e8m0_row_max(const uint8_t* p, int nbytes) {
  uint32_t m4 = 0;
  auto fold = [&](uint32_t v) { m4 = __vmaxu4(m4, v & ~__vcmpeq4(v, 0xFFFFFFFFu)); };
  int i = 0;
  while (i < nbytes && (reinterpret_cast<uintptr_t>(p + i) & 15u)) {
    fold(__ldg(reinterpret_cast<const uint32_t*>(p + i)));
    i += 4;
  }
  for (; i + 128 <= nbytes; i += 128) {
    uint4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = __ldg(reinterpret_cast<const uint4*>(p + i) + u);
#pragma unroll
    for (int u = 0; u < 8; ++u) { fold(v[u].x); fold(v[u].y); fold(v[u].z); fold(v[u].w); }
  }
  for (; i + 16 <= nbytes; i += 16) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(p + i));
    fold(v.x); fold(v.y); fold(v.z); fold(v.w);
  }
  for (; i < nbytes; i += 4) fold(__ldg(reinterpret_cast<const uint32_t*>(p + i)));
  m4 = __vmaxu4(m4, m4 >> 16);
  m4 = __vmaxu4(m4, m4 >> 8);
  return (int)(m4 & 0xFFu);
}

// Largest exponent field among the FP16 scales in nbytes bytes at p, with
// infinity / NaN fields (31) counted as 0.  p is 4-byte aligned and nbytes a
// multiple of 4.
__device__ __forceinline__ int f16_row_emax(const uint8_t* p, int nbytes) {
  uint32_t m2 = 0;  // two 16-bit lanes, each the largest field seen there
  auto fold = [&](uint32_t v) {
    uint32_t e = (v >> 10) & 0x001F001Fu;
    e &= ~__vcmpeq2(e, 0x001F001Fu);
    m2 = __vmaxu2(m2, e);
  };
  int i = 0;
  while (i < nbytes && (reinterpret_cast<uintptr_t>(p + i) & 15u)) {
    fold(__ldg(reinterpret_cast<const uint32_t*>(p + i)));
    i += 4;
  }
  for (; i + 16 <= nbytes; i += 16) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(p + i));
    fold(v.x); fold(v.y); fold(v.z); fold(v.w);
  }
  for (; i < nbytes; i += 4) fold(__ldg(reinterpret_cast<const uint32_t*>(p + i)));
  return (int)max(m2 & 0xFFFFu, m2 >> 16);
}

template <int FMT, int BN, bool F32OUT>
__global__ void __launch_bounds__(kSkThreads, 1)
k_umma_sk(const __grid_constant__ CUtensorMap map_w, const SkArgs a) {
  using C = SkCfg<BN>;
  constexpr int SX = C::SX, SW = C::SW, AST = C::AST;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = su32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;  // swizzled tiles want 1024-byte alignment
  uint8_t* gbase = smem_raw + (base - raw);
  // [X ring: SX x (four BN x 128 B sub-tiles)] [W ring: SW x (128 rows x 128 B)]
  auto X_addr = [&](int s) { return base + (uint32_t)(s * C::X_STAGE); };
  auto W_off = [&](int s) { return SX * C::X_STAGE + s * C::W_STAGE; };
  uint64_t* bars = reinterpret_cast<uint64_t*>(gbase + SX * C::X_STAGE + SW * C::W_STAGE);
  auto fullx_bar = [&](int s) { return su32(&bars[s]); };
  auto emptyx_bar = [&](int s) { return su32(&bars[SX + s]); };
  auto fullw_bar = [&](int s) { return su32(&bars[2 * SX + s]); };
  auto emptyw_bar = [&](int s) { return su32(&bars[2 * SX + SW + s]); };
  auto aready_bar = [&](int s) { return su32(&bars[2 * SX + 2 * SW + s]); };
  auto afree_bar = [&](int s) { return su32(&bars[2 * SX + 2 * SW + AST + s]); };
  constexpr int B8 = 2 * SX + 2 * SW + 2 * AST;
  auto accf_bar = [&](int b) { return su32(&bars[B8 + b]); };
  auto acce_bar = [&](int b) { return su32(&bars[B8 + 2 + b]); };
  auto basef_bar = [&](int b) { return su32(&bars[B8 + 4 + b]); };
  auto basee_bar = [&](int b) { return su32(&bars[B8 + 6 + b]); };
  int* sbase = reinterpret_cast<int*>(bars + C::NBAR);                 // [2][128] row base exponents
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sbase + 2 * kSkRows);
  unsigned* s_ticket = tmem_slot + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long it0 = (long long)blockIdx.x * a.T / a.G;
  const long long it1 = (long long)(blockIdx.x + 1) * a.T / a.G;
  const int niter = (int)(it1 - it0);
  const int KS = a.KS;
  unsigned* fault = &g_sk_fault;

  if (threadIdx.x == 0) {
    for (int s = 0; s < SX; ++s) { mbar_init(fullx_bar(s), 1); mbar_init(emptyx_bar(s), 1); }
    for (int s = 0; s < SW; ++s) {  // full: expect_tx arrival + 32 cp.async arrivals (scale bytes)
      mbar_init(fullw_bar(s), 1 + 32);
      mbar_init(emptyw_bar(s), kSkDqWarps);
    }
    for (int s = 0; s < AST; ++s) { mbar_init(aready_bar(s), kSkDqWarps); mbar_init(afree_bar(s), 1); }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf_bar(b), 1);
      mbar_init(acce_bar(b), kSkEpiWarps);
      mbar_init(basef_bar(b), kSkEpiWarps);
      mbar_init(basee_bar(b), kSkDqWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kSkMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                 "r"(512u));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // the next call's kernels may launch now; they take SMs as this grid's
  // CTAs finish and read nothing it writes before their own wait returns
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const uint32_t tmem_a = tmem + 2u * BN;
  bool ok = true;

  if (warp == kSkXProd) {
    // ------------------------------ X producer --------------------------------
    if (lane == 0) {
      asm volatile("griddepcontrol.wait;" ::: "memory");  // X prepared by the previous grid
      int tile = (int)(it0 / KS), ks = (int)(it0 % KS);
      for (int i = 0; i < niter; ++i) {
        const int s = i % SX;
        if (i >= SX) ok = mbar_wait_flag(emptyx_bar(s), ((i / SX) + 1) & 1, fault);
        if (!ok) break;
        const uint8_t* src = a.xsw + ((size_t)(tile / a.tiles_n) * KS + ks) * (size_t)C::X_STAGE;
        mbar_expect_tx(fullx_bar(s), (uint32_t)C::X_STAGE);
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
            ::"r"(X_addr(s)), "l"(src), "r"((uint32_t)C::X_STAGE), "r"(fullx_bar(s))
            : "memory");
        if (++ks == KS) { ks = 0; ++tile; }
      }
    }
  } else if (warp < kSkWProd0 + kSkWProds) {
    // ------------------------------ W producers -------------------------------
    // Lane 0 arms the stage and issues the packed-W box; all 32 lanes copy the
    // step's scale bytes (4-byte cp.async) next to it and arrive on the same
    // mbarrier when their copies land.
    {
      const int p = warp - kSkWProd0;
      constexpr int SBY = sk_scale_bytes(FMT);  // scale bytes per row per step
      constexpr int WPR = SBY / 4;
      const size_t srow = (size_t)a.K / kSkBK * SBY;
      int tile = (int)((it0 + p) / KS), ks = (int)((it0 + p) % KS);
      for (int i = p; i < niter; i += kSkWProds) {
        const int s = i % SW;
        if (i >= SW && lane == 0) ok = mbar_wait_flag(emptyw_bar(s), ((i / SW) + 1) & 1, fault);
        ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
        if (!ok) break;
        const int n0 = (tile % a.tiles_n) * kSkRows;
        if (lane == 0) {
          mbar_expect_tx(fullw_bar(s), (uint32_t)C::W_CODES);
          tma_load_2d(base + (uint32_t)W_off(s), &map_w, ks * (kSkBK / 2), n0, fullw_bar(s));
        }
#pragma unroll
        for (int e = lane; e < kSkRows * WPR; e += 32) {
          const int row = e / WPR, wi = e % WPR;
          const int n = (n0 + row < a.N) ? n0 + row : a.N - 1;  // rows past N: their codes are zero-filled
          const uint8_t* src = a.scales + (size_t)n * srow + (size_t)ks * SBY + 4 * wi;
          asm volatile("cp.async.ca.shared.global [%0], [%1], 4;"
                       ::"r"(base + (uint32_t)(W_off(s) + C::W_CODES + row * C::W_SCALE_ROW + 4 * wi)), "l"(src)
                       : "memory");
        }
        asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(fullw_bar(s)) : "memory");
        ks += kSkWProds;
        while (ks >= KS) { ks -= KS; ++tile; }
      }
    }
  } else if (warp == kSkMmaWarp) {
    // ------------------------------ MMA issuer --------------------------------
    // The whole warp runs the loop, so the operand arithmetic stays warp-
    // uniform; one elected lane issues the MMAs and commits.
    {
      constexpr uint32_t idesc = idesc_f16(kSkRows, BN);
      uint32_t leader;
      asm volatile("{ .reg .pred p; elect.sync _|p, 0xFFFFFFFF; selp.u32 %0, 1, 0, p; }" : "=r"(leader));
      int kt = (int)(it0 % KS), seg = 0;
      for (int i = 0; i < niter; ++i) {
        const int sx = i % SX, sa = i % AST;
        const bool first = (i == 0) || (kt == 0);
        const bool last = (i == niter - 1) || (kt == KS - 1);
        if (first && i > 0) ++seg;
        const int b = seg & 1;
        if (first && seg >= 2) ok = mbar_wait_flag(acce_bar(b), ((seg >> 1) + 1) & 1, fault);
        ok = ok && mbar_wait_flag(aready_bar(sa), (i / AST) & 1, fault) &&
             mbar_wait_flag(fullx_bar(sx), (i / SX) & 1, fault);
        ok = __all_sync(0xFFFFFFFFu, ok);
        if (!ok) break;
        tc_fence_after();
        const uint64_t d0 = sw128_desc(X_addr(sx));
        const uint32_t ta = tmem_a + (uint32_t)(sa * 128), td = tmem + (uint32_t)(b * BN);
        const uint32_t acc0 = first ? 0u : 1u;
#pragma unroll
        for (int g4 = 0; g4 < kSkBK / 64; ++g4) {  // sub-tile g4 of X: 4 MMAs of K = 16
          const uint64_t dg = d0 + (uint64_t)(g4 * (C::XBOX >> 4));
          const uint32_t ag = ta + (uint32_t)(g4 * 32);
          asm volatile(
              "{ .reg .pred L, A, T;\n"
              "  setp.ne.b32 L, %0, 0;\n"
              "  setp.ne.b32 A, %1, 0;\n"
              "  setp.eq.b32 T, %0, %0;\n"
              "  @L tcgen05.mma.cta_group::1.kind::f16 [%2], [%3], %4, %5, A;\n"
              "  @L tcgen05.mma.cta_group::1.kind::f16 [%2], [%6], %7, %5, T;\n"
              "  @L tcgen05.mma.cta_group::1.kind::f16 [%2], [%8], %9, %5, T;\n"
              "  @L tcgen05.mma.cta_group::1.kind::f16 [%2], [%10], %11, %5, T; }\n"
              ::"r"(leader), "r"(g4 == 0 ? acc0 : 1u), "r"(td), "r"(ag), "l"(dg), "r"(idesc),
                "r"(ag + 8u), "l"(dg + 2), "r"(ag + 16u), "l"(dg + 4), "r"(ag + 24u), "l"(dg + 6)
              : "memory");
        }
        if (leader) {
          umma_commit(emptyx_bar(sx));
          umma_commit(afree_bar(sa));
          if (last) umma_commit(accf_bar(b));
        }
        __syncwarp();
        if (++kt == KS) kt = 0;
      }
    }
  } else if (warp < kSkEpiWarp0) {
    // ------------------------------ dequant -----------------------------------
    const int q = warp & 3;                  // TMEM lane quadrant
    const int j = (warp - kSkDqWarp0) >> 2;  // 64-k slice of the step
    const int r = 32 * q + lane;             // weight row in the tile = TMEM lane
    const uint32_t t_lane = (uint32_t)(32 * q) << 16;
    // SWIZZLE_128B: 16-byte chunk c of 128-byte row r sits at chunk c ^ (r % 8)
    const uint32_t w_c0 = (uint32_t)(r * 128 + (((2 * j) ^ (r & 7)) << 4));
    const uint32_t w_c1 = (uint32_t)(r * 128 + (((2 * j + 1) ^ (r & 7)) << 4));
    // this thread's scale bits in a W stage: MXFP4 two E8M0 bytes, NVFP4 four
    // E4M3 bytes, INT4 one FP16 group scale (g128: group j / 2, g64: group j)
    const uint32_t sc_off = (uint32_t)(C::W_CODES + r * C::W_SCALE_ROW +
                                       (FMT == 0 ? 2 * j : FMT == 1 ? 4 * j : FMT == 2 ? 2 * (j >> 1) : 2 * j));
    // W ring position of the next step to load, and of the step being widened
    int ld_s = 0, cur_s = 0;
    uint32_t ld_ph = 0;
    auto load_step = [&](uint4& c0, uint4& c1, uint32_t& sc, int& stage) -> bool {
      stage = ld_s;
      bool okw = mbar_wait_flag(fullw_bar(ld_s), ld_ph, fault);
      if (++ld_s == SW) { ld_s = 0; ld_ph ^= 1u; }
      okw = __all_sync(0xFFFFFFFFu, okw);
      if (!okw) return false;
      const uint8_t* st = gbase + W_off(stage);
      c0 = *reinterpret_cast<const uint4*>(st + w_c0);
      c1 = *reinterpret_cast<const uint4*>(st + w_c1);
      sc = (FMT != 1) ? (uint32_t)*reinterpret_cast<const uint16_t*>(st + sc_off)
                      : *reinterpret_cast<const uint32_t*>(st + sc_off);
      return true;
    };
    // 32 codes -> 16 f16x2 words with their block factors applied
    auto widen = [&](uint4 pk4, uint32_t f_lo, uint32_t f_hi, uint32_t* o) {
      if constexpr (FMT >= 2) {
        const uint32_t qw[4] = {pk4.x, pk4.y, pk4.z, pk4.w};
#pragma unroll
        for (int w4 = 0; w4 < 4; ++w4) {
          uint32_t t[4];
          int4x8_to_f16(qw[w4], t);
#pragma unroll
          for (int u = 0; u < 4; ++u) o[4 * w4 + u] = t[u];
        }
      } else {
        e2m1x8_to_f16x2(pk4.x, o);
        e2m1x8_to_f16x2(pk4.y, o + 4);
        e2m1x8_to_f16x2(pk4.z, o + 8);
        e2m1x8_to_f16x2(pk4.w, o + 12);
      }
#pragma unroll
      for (int u = 0; u < 16; ++u) o[u] = hmul2_f16x2(o[u], u < 8 ? f_lo : f_hi);
    };
    // Software pipeline: step i's codes and scales were loaded during step
    // i - 1; step i + 1's are loaded once step i's TMEM store has landed and
    // the step is released (an earlier release feeds the MMA sooner).
    int kt = (int)(it0 % KS), seg = 0, rb = 0;
    int sa = 0;                 // TMEM A stage of step i
    uint32_t afree_ph = 1u;     // parity of afree_bar(sa) to wait for (from the second round on)
    uint4 c0 = make_uint4(0, 0, 0, 0), c1 = c0;
    uint32_t sc = 0;
    if (niter > 0) ok = load_step(c0, c1, sc, cur_s);
    for (int i = 0; i < niter && ok; ++i) {
      const bool first = (i == 0) || (kt == 0);
      if (first && i > 0) ++seg;
      if (FMT != 1 && first) {
        const int b = seg & 1;
        ok = mbar_wait_flag(basef_bar(b), (seg >> 1) & 1, fault);
        ok = __all_sync(0xFFFFFFFFu, ok);
        if (!ok) break;
        rb = sbase[b * kSkRows + r];
        __syncwarp();
        if (lane == 0) mbar_arrive(basee_bar(b));
      }
      uint32_t f0, f1, f2, f3;  // factors of the four 16-code halves of the two chunks
      if (FMT == 0) {
        // 2^(e - 127 - rb) is a normal f16 for e >= rb + 113 (every block
        // within 27 binades of the segment's largest); blocks further down
        // and NaN (0xFF) codes take the exact select chain, warp-uniformly.
        const int b0 = (int)(sc & 0xFFu), b1 = (int)((sc >> 8) & 0xFFu);
        const int e0 = b0 - 127 - rb, e1 = b1 - 127 - rb;
        const bool slow = (e0 < -14) | (e1 < -14) | (b0 == 0xFF) | (b1 == 0xFF);
        const uint32_t h0 = (uint32_t)(e0 + 15) << 10, h1 = (uint32_t)(e1 + 15) << 10;
        f0 = f1 = h0 | (h0 << 16);
        f2 = f3 = h1 | (h1 << 16);
        if (__any_sync(0xFFFFFFFFu, slow)) {
          f0 = f1 = (b0 == 0xFF) ? 0x7E007E00u : f16x2_pow2(e0);
          f2 = f3 = (b1 == 0xFF) ? 0x7E007E00u : f16x2_pow2(e1);
        }
      } else if (FMT >= 2) {
        // FP16 group scale times 2^-rb (rb <= 4: a normal f16)
        f0 = f1 = f2 = f3 = hmul2_f16x2((sc & 0xFFFFu) | (sc << 16), f16x2_pow2(-rb));
      } else {
        // normal E4M3 codes in one step; zero / subnormal / NaN codes exactly
        uint32_t l0, h0, l1, h1;
        const bool ok0 = e4m3x2_to_f16x2_fast(sc & 0xFFFFu, l0, h0);
        const bool ok1 = e4m3x2_to_f16x2_fast(sc >> 16, l1, h1);
        const bool fast = ok0 & ok1;
        f0 = l0; f1 = h0; f2 = l1; f3 = h1;
        if (__any_sync(0xFFFFFFFFu, !fast)) {
          f0 = f16x2_e4m3(sc & 0xFFu); f1 = f16x2_e4m3((sc >> 8) & 0xFFu);
          f2 = f16x2_e4m3((sc >> 16) & 0xFFu); f3 = f16x2_e4m3(sc >> 24);
        }
      }
      uint32_t o[32];
      widen(c0, f0, f1, o);
      widen(c1, f2, f3, o + 16);
      __syncwarp();                                   // every lane's codes are in registers:
      if (lane == 0) mbar_arrive(emptyw_bar(cur_s));  // the W stage may be refilled
      if (i >= AST) ok = mbar_wait_flag(afree_bar(sa), afree_ph, fault);
      ok = __all_sync(0xFFFFFFFFu, ok);
      if (!ok) break;
      tmem_st32(tmem_a + t_lane + (uint32_t)(sa * 128 + 32 * j), o);
      // release the step as soon as its store has landed, then load the next
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(aready_bar(sa));
      int nxt_s = cur_s;
      if (i + 1 < niter) ok = load_step(c0, c1, sc, nxt_s);
      cur_s = nxt_s;
      if (++sa == AST) { sa = 0; afree_ph ^= 1u; }
      if (++kt == KS) kt = 0;
    }
  } else {
    // ------------------------------ epilogue ----------------------------------
    const int q = warp & 3;
    const int r = 32 * q + lane;
    const uint32_t t_lane = (uint32_t)(32 * q) << 16;
    const int first_tile = (int)(it0 / KS);
    // row factor exponent of a segment (MXFP4, INT4), or an L2 prefetch of its scales (NVFP4)
    auto prepare = [&](long long it) -> int {
      const int t = (int)(it / KS), kb = (int)(it % KS);
      const int ke = (int)((kb + (it1 - it)) < KS ? (kb + (it1 - it)) : KS);
      const int n = (t % a.tiles_n) * kSkRows + r;
      if (n >= a.N) return 0;
      if (FMT == 0) {
        const int m = e8m0_row_max(a.scales + (size_t)n * (a.K / 32) + (size_t)kb * (kSkBK / 32),
                                   (ke - kb) * (kSkBK / 32));
        return m - 127 - 13;
      }
      if (FMT >= 2) {
        constexpr int SBY = sk_scale_bytes(FMT);
        const int e = f16_row_emax(a.scales + (size_t)n * (a.K / kSkBK * SBY) + (size_t)kb * SBY, (ke - kb) * SBY);
        return e > 26 ? e - 26 : 0;
      }
      const uint8_t* p = a.scales + (size_t)n * (a.K / 16) + (size_t)kb * (kSkBK / 16);
      for (int off = 0; off < (ke - kb) * (kSkBK / 16); off += 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(p + off));
      return 0;
    };
    auto publish = [&](int b, int v) {
      sbase[b * kSkRows + r] = v;
      __syncwarp();
      if (lane == 0) mbar_arrive(basef_bar(b));
    };
    int rb_cur = 0;
    if (niter > 0) {
      rb_cur = prepare(it0);
      if (FMT != 1) publish(0, rb_cur);
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");  // xs written by the X-preparation grid
    long long it = it0;
    for (int seg = 0; it < it1; ++seg) {
      const int tile = (int)(it / KS), kb = (int)(it % KS);
      const int ke = (int)((kb + (it1 - it)) < KS ? (kb + (it1 - it)) : KS);
      const long long it_next = it + (ke - kb);
      int rb_next = 0;
      if (it_next < it1) {  // next segment's row bases while this one computes
        const int b2 = (seg + 1) & 1;
        if (FMT != 1 && seg + 1 >= 2) ok = ok && mbar_wait_flag(basee_bar(b2), (((seg + 1) >> 1) + 1) & 1, fault);
        rb_next = prepare(it_next);
        if (FMT != 1) publish(b2, rb_next);
      }
      const int b = seg & 1;
      ok = ok && mbar_wait_flag(accf_bar(b), (seg >> 1) & 1, fault);
      ok = __all_sync(0xFFFFFFFFu, ok);
      tc_fence_after();
      const int n = (tile % a.tiles_n) * kSkRows + r, m0 = (tile / a.tiles_n) * BN;
      const bool live = n < a.N;
      const float rowf = (FMT != 1) ? ldexpf(1.0f, rb_cur) : a.ts;
      const bool whole = (kb == 0 && ke == KS);
      const uint32_t tacc = tmem + t_lane + (uint32_t)(b * BN);
      const int slot = 2 * (int)blockIdx.x + (tile == first_tile ? 0 : 1);
      float* part = a.partials + (size_t)slot * (kSkRows * BN) + (size_t)r * BN;
      if (ok) {
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          uint32_t v[16];
          tmem_ld16(tacc + (uint32_t)c0, v);
          if (whole) {
            if (live) {
#pragma unroll
              for (int u = 0; u < 16; ++u) {
                const int m = m0 + c0 + u;
                if (m < a.M) {
                  const float y = u2f(v[u]) * rowf * __ldg(a.xs + m);
                  if (F32OUT) static_cast<float*>(a.Y)[(size_t)m * a.N + n] = y;
                  else if (a.tp.world > 0) tp_store(a.tp, (size_t)m, n, __float2bfloat16_rn(y));
                  else static_cast<__nv_bfloat16*>(a.Y)[(size_t)m * a.N + n] = __float2bfloat16_rn(y);
                }
              }
            }
          } else {
#pragma unroll
            for (int u = 0; u < 16; u += 4)
              __stcg(reinterpret_cast<float4*>(part + c0 + u),
                     make_float4(u2f(v[u]) * rowf, u2f(v[u + 1]) * rowf, u2f(v[u + 2]) * rowf,
                                 u2f(v[u + 3]) * rowf));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce_bar(b));  // accumulator buffer free for segment seg + 2
      if (!whole) {
        // every epilogue warp takes the same named-barrier steps, also after a timeout
        __threadfence();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (warp == kSkEpiWarp0 && lane == 0) *s_ticket = atomicAdd(a.counters + tile, 1u);  // also after a timeout: the tickets still return to zero
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const unsigned ticket = *s_ticket;
        const long long t0 = (long long)tile * KS, t1 = t0 + KS - 1;
        const int c_lo = (int)(((t0 + 1) * a.G - 1) / a.T), c_hi = (int)(((t1 + 1) * a.G - 1) / a.T);
        if (ticket == (unsigned)(c_hi - c_lo)) {  // last contributor: sum in CTA order
          __threadfence();
#pragma unroll 1
          for (int c0 = 0; c0 < BN; c0 += 16) {
            float acc[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) acc[u] = 0.0f;
            // two contributors' loads in flight, added in CTA order
            auto src_of = [&](int cc) {
              const int cs = 2 * cc + (tile == (int)(((long long)cc * a.T / a.G) / KS) ? 0 : 1);
              return reinterpret_cast<const float4*>(a.partials + (size_t)cs * (kSkRows * BN) + (size_t)r * BN + c0);
            };
#pragma unroll 1
            for (int cc = c_lo; cc <= c_hi; cc += 2) {
              const bool two = cc < c_hi;
              const float4* s0 = src_of(cc);
              const float4* s1 = two ? src_of(cc + 1) : s0;
              float4 pv[8];
#pragma unroll
              for (int u = 0; u < 4; ++u) pv[u] = __ldcg(s0 + u);
#pragma unroll
              for (int u = 0; u < 4; ++u) pv[4 + u] = __ldcg(s1 + u);
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                acc[4 * u] += pv[u].x; acc[4 * u + 1] += pv[u].y; acc[4 * u + 2] += pv[u].z; acc[4 * u + 3] += pv[u].w;
              }
              if (two) {
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                  acc[4 * u] += pv[4 + u].x; acc[4 * u + 1] += pv[4 + u].y; acc[4 * u + 2] += pv[4 + u].z;
                  acc[4 * u + 3] += pv[4 + u].w;
                }
              }
            }
            if (live) {
#pragma unroll
              for (int u = 0; u < 16; ++u) {
                const int m = m0 + c0 + u;
                if (m < a.M) {
                  const float y = acc[u] * __ldg(a.xs + m);
                  if (F32OUT) static_cast<float*>(a.Y)[(size_t)m * a.N + n] = y;
                  else if (a.tp.world > 0) tp_store(a.tp, (size_t)m, n, __float2bfloat16_rn(y));
                  else static_cast<__nv_bfloat16*>(a.Y)[(size_t)m * a.N + n] = __float2bfloat16_rn(y);
                }
              }
            }
          }
          if (warp == kSkEpiWarp0 && lane == 0) a.counters[tile] = 0u;  // leave the workspace zeroed
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");  // s_ticket is reused by the next segment
      }
      rb_cur = rb_next;
      it = it_next;
    }
  }

  if (!ok) {
    atomicCAS(fault, 0u, 1u);  // keeps the first site
    if (threadIdx.x == 0) {  // give copies and MMAs in flight a bounded chance to land
      fault_drain();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kSkMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512u));
  }
  if (a.tp.world > 0) tp_finish(a.tp, fault);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

bool make_tma_map_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* ptr, uint64_t inner, uint64_t outer,
                     uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw);

int umma_sk_bn(int M) { return M >= 64 ? 64 : 32; }

// Weights of at least 2^26 codes (32 MiB packed).  Below that the tile
// kernel with K splits was as fast or faster (one B200, NVFP4 / INT4 g128,
// M = 20 / 32 / 64 / 100, CUDA-graph replays of weight-rotated calls):
// 4096 x 4096 18-24 us against 23-51 us here, 14336 x 4096 and 4096 x 14336
// within +-8 % except M = 64 (31-39 us against 39-51 us); from 10240 x 8192
// up this kernel wins (1.1-1.5x; 57344 x 8192 1.5-1.8x), M = 64 at
// 10240 x 8192 excepted (0.86-0.93x).
constexpr size_t kSkMinCodes = (size_t)1 << 26;

bool umma_sk_supported(const qgemm_weights_t* w, int M) {
  return (M >= 32 || (M >= 17 && w->format != QGEMM_FMT_MXFP4)) && M < 128 && w->N * w->K >= kSkMinCodes &&
         (w->format == QGEMM_FMT_MXFP4 || w->format == QGEMM_FMT_NVFP4 || w->format == QGEMM_FMT_INT4_G128 ||
          w->format == QGEMM_FMT_INT4_G64) &&
         w->K % kSkBK == 0 && w->K <= (size_t)INT32_MAX && w->N <= (size_t)INT32_MAX &&
         (reinterpret_cast<uintptr_t>(w->scales) & 3u) == 0;
}

struct SkPlan {
  int bn, tiles_n, tiles, KS, G;
  long long T;
  size_t counter_bytes, partial_bytes;
};

static SkPlan sk_plan(const qgemm_weights_t* w, int M, int sm_count) {
  SkPlan p;
  p.bn = umma_sk_bn(M);
  p.tiles_n = (int)((w->N + kSkRows - 1) / kSkRows);
  p.tiles = p.tiles_n * ((M + p.bn - 1) / p.bn);
  p.KS = (int)(w->K / kSkBK);
  p.T = (long long)p.tiles * p.KS;
  p.G = (int)(p.T < sm_count ? p.T : sm_count);
  p.counter_bytes = (size_t)p.tiles * sizeof(unsigned);  // in the workspace's ticket region
  p.partial_bytes = (size_t)2 * p.G * kSkRows * p.bn * sizeof(float);
  return p;
}

// The partial-sum block; the tickets live in the workspace's ticket region.
size_t umma_sk_workspace(const qgemm_weights_t* w, int M, int sm_count) {
  const SkPlan p = sk_plan(w, M, sm_count);
  return p.partial_bytes;
}

template <int FMT, int BN, bool F32>
static cudaError_t launch_sk_t(const CUtensorMap& mw, const SkArgs& a, cudaStream_t s) {
  constexpr int BYTES = SkCfg<BN>::BYTES;
  static bool attr[64] = {false};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr[dev]) {
    e = cudaFuncSetAttribute(k_umma_sk<FMT, BN, F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, BYTES);
    if (e != cudaSuccess) return e;
    attr[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a.G);
  cfg.blockDim = dim3(kSkThreads);
  cfg.dynamicSmemBytes = BYTES;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_umma_sk<FMT, BN, F32>, mw, a);
}

template <int FMT, bool F32>
static cudaError_t launch_sk_bn(int bn, const CUtensorMap& mw, const SkArgs& a, cudaStream_t s) {
  return bn == 32 ? launch_sk_t<FMT, 32, F32>(mw, a, s) : launch_sk_t<FMT, 64, F32>(mw, a, s);
}

// Xh / xs: the f16 copy of X in the swizzled operand layout and its row
// factors (k_xprep with swz_bn = umma_sk_bn(M)); tickets: the workspace's
// ticket region (zero); partials: umma_sk_workspace bytes.
qgemm_status_t gemm_umma_sk(const qgemm_weights_t* w, const __half* Xh, const float* xs, int M, void* Y, bool f32,
                            unsigned* tickets, void* partials, int sm_count, cudaStream_t s, const TpOut* tp) {
  if (!umma_sk_supported(w, M)) return fail(QGEMM_ERR_UNSUPPORTED_SHAPE, "stream-K tcgen05 path: unsupported shape");
  if (sm_count <= 0) return fail(QGEMM_ERR_CUDA, "stream-K tcgen05 path: no device properties");
  const SkPlan p = sk_plan(w, M, sm_count);
  CUtensorMap mw;
  if (!make_tma_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w->data, w->K / 2, w->N, w->K / 2, kSkBK / 2, kSkRows,
                       CU_TENSOR_MAP_SWIZZLE_128B))
    return fail(QGEMM_ERR_CUDA, "stream-K tcgen05 path: cuTensorMapEncodeTiled failed");
  SkArgs a;
  a.scales = static_cast<const uint8_t*>(w->scales);
  a.xsw = reinterpret_cast<const uint8_t*>(Xh);
  a.Y = Y; a.xs = xs;
  if (p.counter_bytes > ws_ticket_bytes(w->N))
    return fail(QGEMM_ERR_WORKSPACE, "stream-K tcgen05 path: %d tiles exceed the ticket region", p.tiles);
  a.counters = tickets;
  a.partials = static_cast<float*>(partials);
  a.T = p.T; a.M = M; a.N = (int)w->N; a.K = (int)w->K;
  a.tiles_n = p.tiles_n; a.KS = p.KS; a.G = p.G; a.ts = w->tensor_scale;
  a.tp = {};
  if (tp) {
    if (f32) return fail(QGEMM_ERR_INVALID_ARG, "stream-K tcgen05 path: tensor-parallel output is bf16");
    a.tp = *tp;
  }
  cudaError_t e;
  switch (w->format) {
    case QGEMM_FMT_MXFP4:
      e = f32 ? launch_sk_bn<0, true>(p.bn, mw, a, s) : launch_sk_bn<0, false>(p.bn, mw, a, s);
      break;
    case QGEMM_FMT_NVFP4:
      e = f32 ? launch_sk_bn<1, true>(p.bn, mw, a, s) : launch_sk_bn<1, false>(p.bn, mw, a, s);
      break;
    case QGEMM_FMT_INT4_G128:
      e = f32 ? launch_sk_bn<2, true>(p.bn, mw, a, s) : launch_sk_bn<2, false>(p.bn, mw, a, s);
      break;
    default:
      e = f32 ? launch_sk_bn<3, true>(p.bn, mw, a, s) : launch_sk_bn<3, false>(p.bn, mw, a, s);
      break;
  }
  if (e != cudaSuccess) return fail(QGEMM_ERR_CUDA, "stream-K tcgen05 launch: %s", cudaGetErrorString(e));
  return QGEMM_OK;
}

cudaError_t umma_sk_fault_clear() {
  const unsigned z = 0;
  return cudaMemcpyToSymbol(g_sk_fault, &z, sizeof(z));
}

unsigned umma_sk_fault() {
  unsigned f = 0;
  if (cudaMemcpyFromSymbol(&f, g_sk_fault, sizeof(f)) != cudaSuccess) return 0xFFFFFFFFu;
  return f;
}

}  // namespace qg
