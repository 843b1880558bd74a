// gemv_tma.cu -- TMA-fed decode GEMM for M <= 16 (MXFP4, NVFP4, INT4; K % 256 == 0).
//
// Same arithmetic as k_gemv (gemv.cu, through chunk_mma in gemv_core.cuh):
// swap-AB mma.sync m16n8k16 with f16 operands and FP32 accumulation, exact
// E2M1 widening, MXFP4 block scales applied to FP32 per-block partial sums,
// NVFP4 E4M3 scales folded into f16.  What changes is how the weight stream
// reaches the warps.  k_gemv loads W straight into registers, which bounds
// the bytes in flight per SM by the register file; here a persistent CTA per
// SM keeps a deep shared-memory ring full with TMA, so HBM sees enough
// requests in flight to run near its peak.
//
// X is prepared once per call by k_xprep_units, one warp per (activation
// row, 256-k unit): f16 scaled by a power of two 2^-s per row and unit, with
// the row's largest |x| in the unit in [2^14, 2^15), so every bf16 value at or
// above 2^-31 of that largest converts exactly (its 8 significant bits fit
// f16's 11) and smaller ones round to f16's subnormal grid.  The unit's image
// and its row factors 2^s are one contiguous block the producers bulk-copy
// beside the weights.  The consumers sum each unit into a partial and add
// partial * 2^s into the FP32 accumulator (one FMA by an exact power of two),
// so Y differs from the double-accumulated reference (ref_gemm.hpp:15-27)
// only by FP32 summation order.  Per-unit rather than per-row factors make the
// preparation one parallel pass with no row-wide reduction.
//
// Unit of work: a tile of 128 weight rows x 256 k (16 KB of packed codes).
// Schedule: stream-K over (tile, 256-k unit), one contiguous range per CTA;
// tiles split across CTAs are reduced through the workspace by the CTA whose
// ticket shows it arrived last, summing contributors in CTA order.
//
// Warp roles (448 or 320 threads):
//   warps 0, 1   producers, alternate units.  Lane 0 arms the stage's
//                mbarrier and issues the packed-W box (TMA, 128 rows x 128 B,
//                128-byte swizzle) and the unit's X image with its row
//                factors (one bulk copy); all 32 lanes copy the unit's scale
//                bytes, one 8-byte (MXFP4, INT4 g64), 16-byte (NVFP4) or
//                4-byte (INT4 g128) cp.async per weight row, and arrive on
//                the same mbarrier when they land.
//                Weights and scales do not depend on the preparation grid, so
//                the first stages' weights go out before the
//                programmatic-launch wait.  No multicast.
//   warps 2..    consumers, in unit groups (GtCfg): unit i of the CTA's range
//                goes to group i % UG, whose warps each own 16 RPW weight rows
//                and all 256 k of it and run chunk_mma on codes, scales and X
//                fragments read from the stage.  M <= 8: three groups of four
//                warps (32 rows each); M <= 16: two groups of four (32 rows).
//                At each segment end the groups' sums are added in group
//                order and group 0 stores the tile or its stream-K partial.
// Every CTA signals its dependents right after its prologue, so the next
// call's kernels are launched while this one runs and start as its CTAs
// finish; they read nothing this grid writes before their own
// programmatic-launch wait returns.
// Every mbarrier wait is bounded (tc.cuh); on timeout the kernel sets
// g_gemv_tma_fault and returns after letting copies in flight land.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <type_traits>

#include "common.cuh"
#include "gemv_core.cuh"
#include "tc.cuh"
#include "tp.cuh"

namespace qg {

__device__ unsigned g_gemv_tma_fault = 0;

constexpr int kGtUnitK = 256;
constexpr int kGtRows = 128;
constexpr int kGtProd = 2;
constexpr int kGtGroups = 8;   // 16-row groups per 128-row tile

// Consumer layout: UG unit groups of WPG = 8 / RPW warps.  Unit i of a
// CTA's range goes to group i % UG; within the group, warp w owns weight rows
// [16 RPW w, 16 RPW (w + 1)) of the unit and all of its 256 k (RPW 16-row MMA
// tiles, so every X fragment read from shared memory feeds RPW MMAs).  At the
// end of each tile segment the groups' sums are added in group order.
template <int FMT, int NT, int RPW, int UG>
struct GtCfg {
  static constexpr int WPG = kGtGroups / RPW;                          // warps per unit group
  static constexpr int CONS = WPG * UG;
  static constexpr int THREADS = 32 * (kGtProd + CONS);
  static constexpr int MPAD = 8 * NT;
  // scale bytes per row per unit: E8M0 / 32, E4M3 / 16, FP16 / 128, FP16 / 64
  static constexpr int SB = FMT == 0 ? kGtUnitK / 32 : FMT == 1 ? kGtUnitK / 16 : FMT == 2 ? 2 * kGtUnitK / 128
                                                                                           : 2 * kGtUnitK / 64;
  static constexpr int W_BYTES = kGtRows * kGtUnitK / 2;                // 16 KB
  static constexpr int X_BYTES = MPAD * kGtUnitK * 2;
  static constexpr int XF_BYTES = 128;                                  // MPAD row factors 2^s (float)
  static constexpr int S_BYTES = kGtRows * SB;
  static constexpr int STAGE = ((W_BYTES + X_BYTES + XF_BYTES + S_BYTES) + 1023) / 1024 * 1024;
  // the W box lands on a 1024-byte boundary (128-byte swizzle); the unit's X
  // image and its row factors are one bulk copy into [X | XF]
  static_assert(W_BYTES % 1024 == 0 && XF_BYTES >= 4 * MPAD, "stage layout");
  // other groups' sums, two buffers by segment parity (group 0 reads one while
  // the others may already fill the next)
  static constexpr int PART_BYTES = 2 * (UG - 1) * kGtGroups * NT * 32 * 16;
  static constexpr int STAGES = ((200 * 1024 - PART_BYTES) / STAGE) & ~1;  // even: two producers
  static constexpr int BYTES = 1024 + STAGES * STAGE + 3 * STAGES * 8 + 16 + PART_BYTES;
  static_assert(BYTES <= 232448, "shared memory");
  static_assert(STAGES >= 4, "ring depth");
};

struct GtArgs {
  float* partials;       // [2 * G][8 row groups][NT][32 lanes] float4
  unsigned* counters;    // [n_exp * tiles]
  long long T;           // n_exp * tiles * KS
  int N, K, ldy;         // every problem of the launch: W [N, K]; Y rows ldy apart
  int tiles;             // 128-row tiles per problem
  int KS;                // units per tile (K / 256)
  int G;
  TpOut tp;              // world > 0: store into every rank's Y_full, then tp_finish
};

// The problems of one launch: one (MAXE = 1) or up to kGtMaxExperts weight
// matrices of the same format and shape (a mixture-of-experts layer), each
// with its own activations and output.  Global tile gt = e * tiles + t of the
// stream-K iteration space belongs to problem e.  Passed as a grid-constant
// parameter, so the TMA descriptors live in parameter space.
constexpr int kGtMaxExperts = 32;
template <int MAXE>
struct GtGroup {
  CUtensorMap map_w[MAXE];   // packed codes, box 128 rows x 128 B, 128-byte swizzle
  const uint8_t* scales[MAXE];
  const uint8_t* xg[MAXE];   // k_xprep_units image: per 256-k unit, mpad rows x 512 B then mpad row factors
  void* Y[MAXE];
  int M[MAXE];               // activation rows (<= mpad)
  float ts[MAXE];            // NVFP4 tensor scale
};

// ---------------------------------------------------------------------------
// X preparation: one warp per (activation row m < mpad, 256-k unit u).  Lane
// l converts k = 256 u + 8 l .. + 7 of row m; s from the warp's largest |x|
// (bf16 bits without the sign are ordered like the magnitudes; an infinity
// or NaN leaves the row unscaled, so it reaches the output as the
// reference's non-finite sums do).  Image of unit u at u * (mpad 512 + 128):
// row m's 16-byte chunk c at m 512 + 16 xg_pos(c, m), then the mpad factors
// 2^s (rows >= M: zeros and factor 0).
// ---------------------------------------------------------------------------
constexpr int kXuWarps = 8;
template <int MAXE>
struct XuGroup {             // problem e = blockIdx.y: X [M[e]][K] and its image
  const uint16_t* X[MAXE];
  uint8_t* img[MAXE];
  int M[MAXE];
};
template <int MAXE>
__global__ void __launch_bounds__(kXuWarps * 32) k_xprep_units(const __grid_constant__ XuGroup<MAXE> xu, int K, int mpad,
                                                              int fmt) {
  const uint16_t* __restrict__ X = xu.X[MAXE == 1 ? 0 : blockIdx.y];
  uint8_t* __restrict__ img = xu.img[MAXE == 1 ? 0 : blockIdx.y];
  const int M = xu.M[MAXE == 1 ? 0 : blockIdx.y];
  // Dependents (the GEMM) may launch at once and stream their weights; they
  // read the image only after their own wait, which covers this grid.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // X may be the previous grid's output
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * kXuWarps + (threadIdx.x >> 5);
  const int KS = K / kGtUnitK;
  if (gw >= mpad * KS) return;
  const int u = gw / mpad, m = gw % mpad;
  uint8_t* unit = img + (size_t)u * (mpad * (kGtUnitK * 2) + 128);
  uint4 o4 = make_uint4(0u, 0u, 0u, 0u);
  float f = 0.0f;
  if (m < M) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(X + (size_t)m * K + (size_t)u * kGtUnitK + 8 * lane));
    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
    uint32_t mx = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) mx = max(mx, max(w4[q] & 0x7FFFu, (w4[q] >> 16) & 0x7FFFu));
    mx = __reduce_max_sync(0xFFFFFFFFu, mx);
    int sc = 0;  // zero, infinite or NaN: unscaled
    if (mx != 0 && mx < 0x7F80u) {
      const int eb = (int)(mx >> 7);
      const int lg = eb != 0 ? eb - 127 : (31 - __clz((int)mx)) - 133;  // ilogb of the largest |x|
      sc = lg - 14;
      sc = sc < -126 ? -126 : (sc > 114 ? 114 : sc);
    }
    const float inv = u2f((uint32_t)(127 - sc) << 23);  // 2^-s
    float xv[8];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      xv[2 * q] = u2f(w4[q] << 16) * inv;
      xv[2 * q + 1] = u2f(w4[q] & 0xFFFF0000u) * inv;
    }
    __half2 o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q)  // INT4: pairs (q, q + 4), the order int4x8_to_f16 widens codes in
      o[q] = fmt == 2 ? __floats2half2_rn(xv[q], xv[q + 4]) : __floats2half2_rn(xv[2 * q], xv[2 * q + 1]);
    o4 = *reinterpret_cast<const uint4*>(o);
    f = u2f((uint32_t)(127 + sc) << 23);  // 2^s
  }
  *reinterpret_cast<uint4*>(unit + m * (kGtUnitK * 2) + xg_pos(fmt == 0 ? 0 : 1, lane, m) * 16) = o4;
  if (lane == 0) reinterpret_cast<float*>(unit + mpad * (kGtUnitK * 2))[m] = f;
}

// One consumer warp's pass over a unit's two 128-k chunks in the stage
// (codes W, X image, scales SC): its RPW 16-row groups' sums into accu.
template <int FMT, int NT, int RPW, int SB, int SCM>
__device__ __forceinline__ void gt_unit_pass(float (&accu)[RPW][NT][4], const uint8_t* W, const uint8_t* X,
                                             const uint8_t* SC, int wq, int lane) {
  const int g = lane >> 2, j = lane & 3;
  const uint32_t sw = (uint32_t)(g & 7);  // every row this lane touches is g mod 8
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) accu[r][t][e] = 0.0f;
#pragma unroll
  for (int c = 0; c < 2; ++c) {  // the unit's two 128-k chunks
    uint32_t cw[RPW][2][4], cs[RPW][2], cx[NT][16];
#pragma unroll
    for (int r = 0; r < RPW; ++r)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = 16 * (RPW * wq + r) + g + 8 * h;
        const uint8_t* wr = W + row * 128;
        if (FMT == 0) {  // 4 bytes of each of the chunk's 4 blocks
#pragma unroll
          for (int b = 0; b < 4; ++b)
            cw[r][h][b] = *reinterpret_cast<const uint32_t*>(wr + ((((uint32_t)(4 * c + b)) ^ sw) << 4) + 4 * j);
          cs[r][h] = *reinterpret_cast<const uint32_t*>(SC + row * SB + 4 * c);
        } else if (FMT == 3) {  // INT4 g64: 8 bytes of each 64-group, both groups' FP16 scales
          const uint2 lo = *reinterpret_cast<const uint2*>(wr + ((((uint32_t)(4 * c + (j >> 1))) ^ sw) << 4) + 8 * (j & 1));
          const uint2 hi =
              *reinterpret_cast<const uint2*>(wr + ((((uint32_t)(4 * c + 2 + (j >> 1))) ^ sw) << 4) + 8 * (j & 1));
          cw[r][h][0] = lo.x; cw[r][h][1] = lo.y; cw[r][h][2] = hi.x; cw[r][h][3] = hi.y;
          cs[r][h] = *reinterpret_cast<const uint32_t*>(SC + row * SB + 4 * c);
        } else {         // NVFP4 / INT4 g128: 16 contiguous bytes
          const uint4 v = *reinterpret_cast<const uint4*>(wr + ((((uint32_t)(4 * c + j)) ^ sw) << 4));
          cw[r][h][0] = v.x; cw[r][h][1] = v.y; cw[r][h][2] = v.z; cw[r][h][3] = v.w;
          if (FMT == 1) cs[r][h] = *reinterpret_cast<const uint16_t*>(SC + row * SB + 8 * c + 2 * j);
          else cs[r][h] = *reinterpret_cast<const uint16_t*>(SC + row * SB + 2 * c);  // INT4 g128: the chunk's FP16 scale
        }
      }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const int m = 8 * t + g;
      const uint8_t* xr = X + m * (kGtUnitK * 2);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        // 8-f16 chunk of the unit this lane's q-th X word quad comes from
        const int idx = FMT == 0 ? 16 * c + 4 * q + j
                                 : FMT == 3 ? 16 * c + 8 * (q >> 1) + 2 * j + (q & 1) : 16 * c + 4 * j + q;
        const uint4 v = *reinterpret_cast<const uint4*>(xr + xg_pos(FMT == 0 ? 0 : 1, idx, m) * 16);
        cx[t][4 * q] = v.x; cx[t][4 * q + 1] = v.y; cx[t][4 * q + 2] = v.z; cx[t][4 * q + 3] = v.w;
      }
    }
    chunk_mma<FMT, RPW, NT, SCM>(accu, cw, cs, cx);
  }
}

// FAST: every problem's weights are in the scale-checked layout (no scale
// byte needs the exact decoder), so the consumers decode scales without the
// per-chunk search for such bytes.
template <int FMT, int NT, int RPW, int UG, bool F32OUT, int MAXE, bool FAST>
__global__ void __launch_bounds__(GtCfg<FMT, NT, RPW, UG>::THREADS, 1)
k_gemv_tma(const __grid_constant__ GtGroup<MAXE> pg, const GtArgs a) {
  using C = GtCfg<FMT, NT, RPW, UG>;
  constexpr int kGtCons = C::CONS;
  constexpr int S = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = su32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  // stage s: [W 128 x 128 B (swizzled) | X mpad x 512 B | mpad row factors | scales 128 x SB]
  auto W_off = [&](int s) { return s * C::STAGE; };
  auto X_off = [&](int s) { return s * C::STAGE + C::W_BYTES; };
  auto XF_off = [&](int s) { return s * C::STAGE + C::W_BYTES + C::X_BYTES; };
  auto S_off = [&](int s) { return s * C::STAGE + C::W_BYTES + C::X_BYTES + C::XF_BYTES; };
  uint64_t* bars = reinterpret_cast<uint64_t*>(gbase + S * C::STAGE);
  // Two fill barriers per stage, taken by the parity of the use u = i / S
  // of stage s = i % S by unit i.  With S % UG != 0 consecutive uses of a
  // stage go to different consumer groups, so a group may wait for use u
  // while use u - 1 (another group's) is still in flight; on one barrier its
  // parity wait would take that pending phase for the completed one before
  // it.  Uses u - 1 and u are on different barriers here, and use u - 2 (the
  // previous phase of use u's barrier) is complete by then: the group has
  // consumed unit i - lcm(UG, producers), whose producer had issued unit
  // i - S, which needed use u - 2 released.
  auto full_bar = [&](int s, int u) { return su32(&bars[s + S * (u & 1)]); };
  auto empty_bar = [&](int s) { return su32(&bars[2 * S + s]); };
  unsigned* s_ticket = reinterpret_cast<unsigned*>(bars + 3 * S);
  float4* s_part = reinterpret_cast<float4*>(bars + 3 * S + 2);  // [2][UG - 1][8 row groups][NT][32]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long it0 = (long long)blockIdx.x * a.T / a.G;
  const long long it1 = (long long)(blockIdx.x + 1) * a.T / a.G;
  const int niter = (int)(it1 - it0);
  const int KS = a.KS;
  unsigned* fault = &g_gemv_tma_fault;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      for (int u = 0; u < 2; ++u)
        mbar_init(full_bar(s, u), 1 + 32);  // lane 0's expect_tx arrival (W and X) + 32 cp.async arrivals (scales)
      mbar_init(empty_bar(s), C::WPG);  // the unit's group
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  bool ok = true;

  if (warp < kGtProd) {
    // ------------------------------ producers ---------------------------------
    const int p = warp;
    // scale bytes per weight row: E8M0 per 32 k, E4M3 per 16 k, FP16 per 128 / 64 k
    const size_t srow = (size_t)a.K / (FMT == 0 ? 32 : FMT == 1 ? 16 : FMT == 2 ? 64 : 32);
    // (tile, k-unit) of this producer's next unit, advanced by kGtProd units
    // per issue: no 64-bit division in the loop.
    int p_tile = (int)((it0 + p) / KS), p_ks = (int)((it0 + p) % KS);
    auto advance = [&]() {
      p_ks += kGtProd;
      while (p_ks >= KS) { p_ks -= KS; ++p_tile; }
    };
    // problem of global tile gt and its tile within the problem
    auto prob = [&](int gt) { return MAXE == 1 ? 0 : gt / a.tiles; };
    auto ltile = [&](int gt) { return MAXE == 1 ? gt : gt - (gt / a.tiles) * a.tiles; };
    // fb: the fill barrier of the unit's use of stage s
    auto issue_w = [&](int s, uint32_t fb) {  // lane 0: the unit's packed-W box; its X follows on the same barrier
      mbar_expect_tx(fb, (uint32_t)(C::W_BYTES + C::X_BYTES + C::XF_BYTES));
      tma_load_2d(base + (uint32_t)W_off(s), &pg.map_w[prob(p_tile)], p_ks * (kGtUnitK / 2), ltile(p_tile) * kGtRows,
                  fb);
    };
    auto issue_x = [&](int s, uint32_t fb, int gt, int ks) {  // lane 0: the unit's f16 X image and row factors
      const uint8_t* src = pg.xg[prob(gt)] + (size_t)ks * (C::X_BYTES + C::XF_BYTES);
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
          ::"r"(base + (uint32_t)X_off(s)), "l"(src), "r"((uint32_t)(C::X_BYTES + C::XF_BYTES)), "r"(fb)
          : "memory");
    };
    // all lanes: the unit's scale bytes, one 8-byte (MXFP4) or 16-byte (NVFP4)
    // copy per weight row, rows lane + 32 q
    auto issue_scales = [&](int s, uint32_t fb) {
#pragma unroll
      for (int q = 0; q < kGtRows / 32; ++q) {
        const int row = lane + 32 * q;
        int n = ltile(p_tile) * kGtRows + row;
        n = n < a.N ? n : a.N - 1;  // rows past N: TMA zero-fills their codes
        const uint8_t* src = pg.scales[prob(p_tile)] + (size_t)n * srow + (size_t)p_ks * C::SB;
        const uint32_t dst = base + (uint32_t)(S_off(s) + row * C::SB);
        if (C::SB == 16) asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
        else if (C::SB == 8) asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
        else asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
      }
      asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(fb) : "memory");
    };
    if (lane == 0 && MAXE == 1)
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&pg.map_w[0])) : "memory");
    const int pre = niter < S ? niter : S;
    // Weights and scales do not depend on the previous grid: the first stages'
    // go out before the programmatic-launch wait; X follows it.
    for (int i = p; i < pre; i += kGtProd) {  // first uses (u = 0)
      if (lane == 0) issue_w(i, full_bar(i, 0));
      issue_scales(i, full_bar(i, 0));
      advance();
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");  // the X image is the preparation grid's output
    if (lane == 0)
      for (int i = p; i < pre; i += kGtProd) issue_x(i, full_bar(i, 0), (int)((it0 + i) / KS), (int)((it0 + i) % KS));
    for (int i = pre + ((p - pre % kGtProd + kGtProd) % kGtProd); i < niter; i += kGtProd) {
      const int s = i % S;
      const uint32_t fb = full_bar(s, i / S);
      if (lane == 0) ok = mbar_wait_flag(empty_bar(s), ((i / S) + 1) & 1, fault);
      ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
      if (!ok) break;
      if (lane == 0) { issue_w(s, fb); issue_x(s, fb, p_tile, p_ks); }
      issue_scales(s, fb);
      advance();
    }
  } else {
    // ------------------------------ consumers ---------------------------------
    constexpr int WPG = C::WPG;
    static_assert(S % UG == 0 || (UG * kGtProd / (UG % kGtProd == 0 ? kGtProd : 1)) < S,
                  "fill-barrier argument: lcm(UG, producers) < S");
    const int cons = warp - kGtProd;
    const int ug = cons / WPG;                      // unit group: the units i with i % UG == ug
    const int wq = cons % WPG;                      // weight rows [16 RPW wq, 16 RPW (wq + 1)) of a unit
    const int g = lane >> 2, j = lane & 3;
    // (no programmatic-launch wait here: every consumer step depends on a
    // unit whose X the producers copied after theirs)

    float acc[RPW][NT][4];   // FP32 sums in absolute scale
    float accu[RPW][NT][4];  // one unit's sums, in that unit's X scale
    auto zero = [&](float (&v)[RPW][NT][4]) {
#pragma unroll
      for (int r = 0; r < RPW; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
          for (int e = 0; e < 4; ++e) v[r][t][e] = 0.0f;
    };
    zero(acc);
    auto slot_of = [&](int cta, int tile) -> int {
      return 2 * cta + ((int)(((long long)cta * a.T / a.G) / KS) == tile ? 0 : 1);
    };
    auto grp = [&](int r) { return RPW * wq + r; };  // 16-row group of row tile r within the tile
    auto store = [&](int tile, float (&v)[RPW][NT][4]) {
      const int pe = MAXE == 1 ? 0 : tile / a.tiles;        // problem of global tile `tile`
      const int lt = MAXE == 1 ? tile : tile - pe * a.tiles;
      void* Yp = pg.Y[pe];
      const int Mp = pg.M[pe];
      const float ts = pg.ts[pe];
#pragma unroll
      for (int r = 0; r < RPW; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int n = lt * kGtRows + 16 * grp(r) + g + ((e & 2) ? 8 : 0);
            const int m = 8 * t + 2 * j + (e & 1);
            if (n < a.N && m < Mp) {
              float y = v[r][t][e];
              if (FMT == 1) y *= ts;
              if (F32OUT) static_cast<float*>(Yp)[(size_t)m * a.ldy + n] = y;
              else if (a.tp.world > 0) tp_store(a.tp, (size_t)m, n, __float2bfloat16_rn(y));
              else static_cast<__nv_bfloat16*>(Yp)[(size_t)m * a.ldy + n] = __float2bfloat16_rn(y);
            }
          }
        }
    };
    // Group 0 writes a finished segment: the whole tile directly, or its
    // stream-K partial, the last contributor summing all partials in CTA order.
    auto flush = [&](int tile, bool whole) {
      if (whole) {
        store(tile, acc);
        return;
      }
      float4* mine = reinterpret_cast<float4*>(a.partials) + (size_t)slot_of((int)blockIdx.x, tile) * kGtGroups * NT * 32;
#pragma unroll
      for (int r = 0; r < RPW; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t)
          __stcg(mine + (grp(r) * NT + t) * 32 + lane, make_float4(acc[r][t][0], acc[r][t][1], acc[r][t][2], acc[r][t][3]));
      // one acquire-release ticket after the group's barrier orders every
      // thread's partial stores before it and the last contributor's loads
      // after it (the release is cumulative over what the barrier ordered)
      asm volatile("bar.sync 1, %0;" ::"r"(WPG * 32) : "memory");
      if (wq == 0 && lane == 0) *s_ticket = ticket_acq_rel(a.counters + tile);  // also after a timeout: the tickets still return to zero
      asm volatile("bar.sync 1, %0;" ::"r"(WPG * 32) : "memory");
      const unsigned ticket = *s_ticket;
      const long long t0 = (long long)tile * KS, t1 = t0 + KS - 1;
      const int c_lo = (int)(((t0 + 1) * a.G - 1) / a.T), c_hi = (int)(((t1 + 1) * a.G - 1) / a.T);
      if (ticket == (unsigned)(c_hi - c_lo)) {  // last contributor: sum in CTA order
        float sum[RPW][NT][4];
        zero(sum);
        // CB contributors' partials in flight before the first add (they come
        // from L2); the adds stay in CTA order
        constexpr int CB = 2;
#pragma unroll 1
        for (int cb = c_lo; cb <= c_hi; cb += CB) {
          float4 pv[CB][RPW][NT];
#pragma unroll
          for (int u = 0; u < CB; ++u)
            if (cb + u <= c_hi) {
              const float4* src =
                  reinterpret_cast<const float4*>(a.partials) + (size_t)slot_of(cb + u, tile) * kGtGroups * NT * 32;
#pragma unroll
              for (int r = 0; r < RPW; ++r)
#pragma unroll
                for (int t = 0; t < NT; ++t) pv[u][r][t] = __ldcg(src + (grp(r) * NT + t) * 32 + lane);
            }
#pragma unroll
          for (int u = 0; u < CB; ++u)
            if (cb + u <= c_hi) {
#pragma unroll
              for (int r = 0; r < RPW; ++r)
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                  sum[r][t][0] += pv[u][r][t].x; sum[r][t][1] += pv[u][r][t].y;
                  sum[r][t][2] += pv[u][r][t].z; sum[r][t][3] += pv[u][r][t].w;
                }
            }
        }
        store(tile, sum);
        if (wq == 0 && lane == 0) a.counters[tile] = 0u;  // leave the workspace zeroed
      }
      asm volatile("bar.sync 1, %0;" ::"r"(WPG * 32) : "memory");  // s_ticket is reused
    };

    int segp = 0;        // s_part buffer of the current segment
    long long it = it0;  // global index of the segment's first unit
    int ib = 0;          // its index in this CTA's range
    while (ib < niter) {
      const int tile = (int)(it / KS), ks0 = (int)(it % KS);
      const int len = (KS - ks0) < (niter - ib) ? (KS - ks0) : (niter - ib);
      for (int i = ib + (ug - ib % UG + UG) % UG; i < ib + len; i += UG) {
        const int s = i % S;
        // use u = i / S of stage s: fill barrier u % 2, its phase u / 2
        if (ok) ok = mbar_wait_flag(full_bar(s, i / S), ((i / S) >> 1) & 1, fault);
        ok = __all_sync(0xFFFFFFFFu, ok);
        if (ok) {
          const uint8_t* W = gbase + W_off(s);
          const uint8_t* X = gbase + X_off(s);
          const uint8_t* SC = gbase + S_off(s);
          gt_unit_pass<FMT, NT, RPW, C::SB, FAST ? kScalesFast : kScalesCheck>(accu, W, X, SC, wq, lane);
          // acc += unit sums * 2^s of their activation rows (exact scaling)
          const float* XF = reinterpret_cast<const float*>(gbase + XF_off(s));
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            const float2 xf = *reinterpret_cast<const float2*>(XF + 8 * t + 2 * j);
#pragma unroll
            for (int r = 0; r < RPW; ++r) {
              acc[r][t][0] = fmaf(accu[r][t][0], xf.x, acc[r][t][0]);
              acc[r][t][1] = fmaf(accu[r][t][1], xf.y, acc[r][t][1]);
              acc[r][t][2] = fmaf(accu[r][t][2], xf.x, acc[r][t][2]);
              acc[r][t][3] = fmaf(accu[r][t][3], xf.y, acc[r][t][3]);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_bar(s));  // this warp is done with the stage
      }
      // the segment's sums: groups 1.. hand theirs to group 0 (fixed order)
      if (UG > 1) {
        if (ug != 0) {
#pragma unroll
          for (int r = 0; r < RPW; ++r)
#pragma unroll
            for (int t = 0; t < NT; ++t)
              s_part[((((segp * (UG - 1)) + ug - 1) * kGtGroups + grp(r)) * NT + t) * 32 + lane] =
                  make_float4(acc[r][t][0], acc[r][t][1], acc[r][t][2], acc[r][t][3]);
        }
        asm volatile("bar.sync 2, %0;" ::"r"(kGtCons * 32) : "memory");
        if (ug == 0) {
          for (int gg = 1; gg < UG; ++gg)
#pragma unroll
            for (int r = 0; r < RPW; ++r)
#pragma unroll
              for (int t = 0; t < NT; ++t) {
                const float4 h = s_part[((((segp * (UG - 1)) + gg - 1) * kGtGroups + grp(r)) * NT + t) * 32 + lane];
                acc[r][t][0] += h.x; acc[r][t][1] += h.y; acc[r][t][2] += h.z; acc[r][t][3] += h.w;
              }
        }
      }
      if (ug == 0) flush(tile, ks0 == 0 && len == KS);
      // (no barrier here: the next segment's sums go to the other s_part buffer,
      // and group 0 passes the next segment's barrier only after reading this one)
      segp ^= 1;
      zero(acc);
      it += len;
      ib += len;
    }
  }

  if (!ok) {
    atomicCAS(fault, 0u, 1u);  // keeps the first site
    if (threadIdx.x == 0) {  // give copies in flight a bounded chance to land
      fault_drain();
    }
  }
  __syncthreads();
  if (a.tp.world > 0) tp_finish(a.tp, fault);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

bool make_tma_map_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* ptr, uint64_t inner, uint64_t outer,
                     uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw);

// Each weight row's scales of a unit are copied as one piece of 8 (MXFP4),
// 16 (NVFP4), 4 (INT4 g128) or 8 (INT4 g64) bytes: the scale array must start
// on such a boundary (the row pitch is a multiple of it since K % 256 == 0).
bool gemv_tma_supported(const qgemm_weights_t* w, int mb) {
  uintptr_t salign = 0;
  switch (w->format) {
    case QGEMM_FMT_MXFP4: salign = 7u; break;
    case QGEMM_FMT_NVFP4: salign = 15u; break;
    case QGEMM_FMT_INT4_G128: salign = 3u; break;
    case QGEMM_FMT_INT4_G64: salign = 7u; break;
    default: return false;
  }
  return mb >= 1 && mb <= 16 && w->K % kGtUnitK == 0 && w->K <= (size_t)INT32_MAX / 2 &&
         w->N <= (size_t)INT32_MAX / 2 && (reinterpret_cast<uintptr_t>(w->scales) & salign) == 0;
}

struct GtPlan {
  int nt, mpad, tiles, KS, G;
  long long T;
  size_t counter_bytes, partial_bytes, image_bytes;  // image_bytes: one problem's
};
// Plan for n_exp problems of w's shape with at most mb activation rows each.
static GtPlan gt_plan(const qgemm_weights_t* w, int mb, int sm_count, int n_exp = 1) {
  GtPlan p;
  p.nt = mb <= 8 ? 1 : 2;
  p.mpad = 8 * p.nt;
  p.tiles = (int)((w->N + kGtRows - 1) / kGtRows);
  p.KS = (int)(w->K / kGtUnitK);
  p.T = (long long)n_exp * p.tiles * p.KS;
  p.G = (int)(p.T < sm_count ? p.T : sm_count);
  // Narrow problems (fewer than 24 units per SM, e.g. tensor-parallel shards)
  // run fewer CTAs of u = 8 or 16 units each, the smallest u that fits the
  // SMs.  Measured (one B200, M = 1 and 8): 1280 x 8192 12.9 -> 8.5 us
  // (u = 8), 2560 x 8192 12.0 -> 9.0 us (8), 5120 x 8192 13.2 -> 12.1 us
  // (16), 7168 x 8192 14.1 -> 12.6 us (16), 1024 x 28672 17.0 -> 13.6 us (8),
  // 2048 x 28672 17.4 -> 15.2 us (16), 4096 x 14336 15.3 -> 14.1 us (16);
  // with one CTA per SM every tile had up to 19 contributors.
  if (p.T < 24LL * sm_count) {
    for (int u = 8; u <= 16; u *= 2) {
      if (p.T / u <= sm_count) {
        p.G = p.T / u > 0 ? (int)(p.T / u) : 1;  // fewer than u units: one CTA
        break;
      }
    }
  }
  p.counter_bytes = ws_ticket_bytes(w->N);  // holds n_exp * tiles <= 32 * tiles tickets
  p.partial_bytes = (((size_t)2 * p.G * kGtGroups * p.nt * 32 * sizeof(float4)) + 255) & ~(size_t)255;
  p.image_bytes = (((size_t)p.KS * (p.mpad * kGtUnitK * 2 + 128)) + 255) & ~(size_t)255;
  return p;
}
// [tickets | partials | X image], sized for 16 activation rows (two n-tiles)
size_t gemv_tma_workspace(const qgemm_weights_t* w, int sm_count) {
  const GtPlan p = gt_plan(w, 16, sm_count);
  return p.counter_bytes + p.partial_bytes + p.image_bytes;
}

// Consumer layout per activation-tile count: M <= 8, three unit groups of
// four warps with 32 rows each (measured against two and four groups: four
// pushes the register budget to 96 and spills, two leaves too few warps to
// hide the MMA and conversion latencies); 9 <= M <= 16, two groups of four
// warps with 32 rows each (against one group of eight warps with 16 rows:
// NVFP4 14336 x 4096 15.4 -> 14.5 us, 57344 x 8192 77.4 -> 70.2 us, INT4
// 14336 x 4096 15.4 -> 14.1 us; the X fragments feed two row tiles each).
template <int NT>
constexpr int gt_rpw() { return 2; }
template <int NT>
constexpr int gt_ug() { return NT == 1 ? 3 : 2; }

template <int FMT, int NT, bool F32, int MAXE, bool FAST>
static cudaError_t launch_gt_t(const GtGroup<MAXE>& g, const GtArgs& a, cudaStream_t s) {
  constexpr int BYTES = GtCfg<FMT, NT, gt_rpw<NT>(), gt_ug<NT>()>::BYTES;
  static bool attr[64] = {false};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr[dev]) {
    e = cudaFuncSetAttribute(k_gemv_tma<FMT, NT, gt_rpw<NT>(), gt_ug<NT>(), F32, MAXE, FAST>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, BYTES);
    if (e != cudaSuccess) return e;
    attr[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a.G);
  cfg.blockDim = dim3(GtCfg<FMT, NT, gt_rpw<NT>(), gt_ug<NT>()>::THREADS);
  cfg.dynamicSmemBytes = BYTES;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_gemv_tma<FMT, NT, gt_rpw<NT>(), gt_ug<NT>(), F32, MAXE, FAST>, g, a);
}

template <int FMT, int NT, int MAXE, bool FAST>
static cudaError_t launch_gt_f(bool f32, const GtGroup<MAXE>& g, const GtArgs& a, cudaStream_t s) {
  if constexpr (MAXE == 1) {
    if (f32) return launch_gt_t<FMT, NT, true, MAXE, FAST>(g, a, s);
  }
  return launch_gt_t<FMT, NT, false, MAXE, FAST>(g, a, s);  // grouped calls: bf16 output only
}
template <int MAXE, bool FAST>
static cudaError_t launch_gt_l(int fmt, int nt, bool f32, const GtGroup<MAXE>& g, const GtArgs& a, cudaStream_t s) {
  switch (fmt) {
    case QGEMM_FMT_MXFP4:
      return nt == 1 ? launch_gt_f<0, 1, MAXE, FAST>(f32, g, a, s) : launch_gt_f<0, 2, MAXE, FAST>(f32, g, a, s);
    case QGEMM_FMT_NVFP4:
      return nt == 1 ? launch_gt_f<1, 1, MAXE, FAST>(f32, g, a, s) : launch_gt_f<1, 2, MAXE, FAST>(f32, g, a, s);
    case QGEMM_FMT_INT4_G128:  // FP16 group scales: no fast / checked distinction
      return nt == 1 ? launch_gt_f<2, 1, MAXE, false>(f32, g, a, s) : launch_gt_f<2, 2, MAXE, false>(f32, g, a, s);
    default:
      return nt == 1 ? launch_gt_f<3, 1, MAXE, false>(f32, g, a, s) : launch_gt_f<3, 2, MAXE, false>(f32, g, a, s);
  }
}
// fast: every problem of the launch is in the scale-checked layout
template <int MAXE>
static cudaError_t launch_gt(int fmt, int nt, bool f32, bool fast, const GtGroup<MAXE>& g, const GtArgs& a,
                             cudaStream_t s) {
  return fast ? launch_gt_l<MAXE, true>(fmt, nt, f32, g, a, s) : launch_gt_l<MAXE, false>(fmt, nt, f32, g, a, s);
}

template <int MAXE>
static cudaError_t launch_xprep_units(const XuGroup<MAXE>& xu, int n_exp, const GtPlan& p, int K, int fmt,
                                      cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((p.mpad * p.KS + kXuWarps - 1) / kXuWarps), (unsigned)n_exp);
  cfg.blockDim = dim3(kXuWarps * 32);
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  // X image order: 0 MXFP4, 1 NVFP4, 2 INT4 (pair permutation)
  const int xf = fmt == QGEMM_FMT_MXFP4 ? 0 : fmt == QGEMM_FMT_NVFP4 ? 1 : 2;
  return cudaLaunchKernelEx(&cfg, k_xprep_units<MAXE>, xu, K, p.mpad, xf);
}

static bool gt_map(CUtensorMap* m, const qgemm_weights_t* w) {
  return make_tma_map_2d(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, w->data, w->K / 2, w->N, w->K / 2, kGtUnitK / 2, kGtRows,
                         CU_TENSOR_MAP_SWIZZLE_128B);
}

// Two launches over mb <= 16 activation rows X (bf16 [mb][K], 16-byte
// aligned): k_xprep_units, then the GEMM (programmatic dependent launch).
// ws: gemv_tma_workspace bytes, counters zero.
qgemm_status_t gemm_gemv_tma(const qgemm_weights_t* w, const uint16_t* X, int mb, void* Y, int ldy, bool f32,
                             void* ws, int sm_count, cudaStream_t s, const TpOut* tp) {
  if (!gemv_tma_supported(w, mb)) return fail(QGEMM_ERR_UNSUPPORTED_SHAPE, "TMA decode path: unsupported shape");
  if (sm_count <= 0) return fail(QGEMM_ERR_CUDA, "TMA decode path: no device properties");
  if (tp && f32) return fail(QGEMM_ERR_INVALID_ARG, "TMA decode path: tensor-parallel output is bf16");
  const GtPlan p = gt_plan(w, mb, sm_count);
  GtGroup<1> g;
  if (!gt_map(&g.map_w[0], w)) return fail(QGEMM_ERR_CUDA, "TMA decode path: cuTensorMapEncodeTiled failed");
  uint8_t* img = static_cast<uint8_t*>(ws) + p.counter_bytes + p.partial_bytes;
  XuGroup<1> xu;
  xu.X[0] = X; xu.img[0] = img; xu.M[0] = mb;
  cudaError_t e = launch_xprep_units<1>(xu, 1, p, (int)w->K, w->format, s);
  if (e != cudaSuccess) return fail(QGEMM_ERR_CUDA, "TMA decode X preparation: %s", cudaGetErrorString(e));
  g.scales[0] = static_cast<const uint8_t*>(w->scales);
  g.xg[0] = img;
  g.Y[0] = Y;
  g.M[0] = mb;
  g.ts[0] = w->tensor_scale;
  GtArgs a;
  a.counters = static_cast<unsigned*>(ws);
  a.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + p.counter_bytes);
  a.T = p.T; a.N = (int)w->N; a.K = (int)w->K; a.ldy = ldy; a.tiles = p.tiles;
  a.KS = p.KS; a.G = p.G;
  a.tp = {};
  if (tp) a.tp = *tp;
  e = launch_gt<1>(w->format, p.nt, f32, w->layout == QGEMM_LAYOUT_SCALE_CHECKED, g, a, s);
  if (e != cudaSuccess) return fail(QGEMM_ERR_CUDA, "TMA decode launch: %s", cudaGetErrorString(e));
  return QGEMM_OK;
}

// ---------------------------------------------------------------------------
// Grouped decode (mixture of experts): problems e = 0 .. n - 1 of the same
// format and shape, problem e's activations X + row0[e] K ([M[e]][K]) and
// output Y + row0[e] N.  Up to kGtMaxExperts problems per pair of launches;
// all problems' units share one stream-K iteration space, so small experts
// do not each pay a launch and a pipeline fill.
// ---------------------------------------------------------------------------

// Workspace of one launch over up to kGtMaxExperts problems with mpad = 16.
size_t gemv_tma_group_workspace(const qgemm_weights_t* w, int sm_count) {
  const GtPlan p = gt_plan(w, 16, sm_count, kGtMaxExperts);
  return p.counter_bytes + p.partial_bytes + (size_t)kGtMaxExperts * p.image_bytes;
}

// ws: gemv_tma_group_workspace bytes, counters zero.  Every problem needs
// 1 <= M[e] <= 16 and gemv_tma_supported.
qgemm_status_t gemm_gemv_tma_group(const qgemm_weights_t* const* w, const int* M, const size_t* row0, int n,
                                   const uint16_t* X, uint16_t* Y, void* ws, int sm_count, cudaStream_t s) {
  if (n < 1 || n > kGtMaxExperts) return fail(QGEMM_ERR_INVALID_ARG, "grouped decode: 1..%d problems", kGtMaxExperts);
  if (sm_count <= 0) return fail(QGEMM_ERR_CUDA, "grouped decode: no device properties");
  int mmax = 0;
  for (int e = 0; e < n; ++e) mmax = M[e] > mmax ? M[e] : mmax;
  const GtPlan p = gt_plan(w[0], mmax, sm_count, n);
  uint8_t* img = static_cast<uint8_t*>(ws) + p.counter_bytes + p.partial_bytes;
  GtGroup<kGtMaxExperts> g;
  XuGroup<kGtMaxExperts> xu;
  std::memset(&g, 0, sizeof(g));
  std::memset(&xu, 0, sizeof(xu));
  for (int e = 0; e < n; ++e) {
    if (!gt_map(&g.map_w[e], w[e])) return fail(QGEMM_ERR_CUDA, "grouped decode: cuTensorMapEncodeTiled failed");
    g.scales[e] = static_cast<const uint8_t*>(w[e]->scales);
    g.xg[e] = img + (size_t)e * p.image_bytes;
    g.Y[e] = Y + row0[e] * w[0]->N;
    g.M[e] = M[e];
    g.ts[e] = w[e]->tensor_scale;
    xu.X[e] = X + row0[e] * w[0]->K;
    xu.img[e] = img + (size_t)e * p.image_bytes;
    xu.M[e] = M[e];
  }
  cudaError_t e = launch_xprep_units<kGtMaxExperts>(xu, n, p, (int)w[0]->K, w[0]->format, s);
  if (e != cudaSuccess) return fail(QGEMM_ERR_CUDA, "grouped decode X preparation: %s", cudaGetErrorString(e));
  GtArgs a;
  a.counters = static_cast<unsigned*>(ws);
  a.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + p.counter_bytes);
  a.T = p.T; a.N = (int)w[0]->N; a.K = (int)w[0]->K; a.ldy = (int)w[0]->N; a.tiles = p.tiles;
  a.KS = p.KS; a.G = p.G;
  a.tp = {};
  bool fast = true;  // the checked decode only when every problem's scales are checked
  for (int q = 0; q < n; ++q) fast = fast && w[q]->layout == QGEMM_LAYOUT_SCALE_CHECKED;
  e = launch_gt<kGtMaxExperts>(w[0]->format, p.nt, false, fast, g, a, s);
  if (e != cudaSuccess) return fail(QGEMM_ERR_CUDA, "grouped decode launch: %s", cudaGetErrorString(e));
  return QGEMM_OK;
}

cudaError_t gemv_tma_fault_clear() {
  const unsigned z = 0;
  return cudaMemcpyToSymbol(g_gemv_tma_fault, &z, sizeof(z));
}

unsigned gemv_tma_fault() {
  unsigned f = 0;
  if (cudaMemcpyFromSymbol(&f, g_gemv_tma_fault, sizeof(f)) != cudaSuccess) return 0xFFFFFFFFu;
  return f;
}

}  // namespace qg
