// umma_bs.cu -- block-scaled tcgen05 W4A16 GEMM for MXFP4: no dequantisation.
//
// Y[M,N] = X[M,K] . W[N,K]^T with W in the reference's MXFP4 layout
// (titoatwork/qgemm-mx include/qgemm/pack.hpp:14-85: E2M1 codes, two per
// byte, and one E8M0 scale per 32 k in a separate array).
//
// The packed codes go from HBM into shared memory by TMA in the 16U4_ALIGN16B
// form (each 16 codes followed by 8 zero bytes) and straight into
// tcgen05.mma.kind::mxf8f6f4.block_scale as the A operand (E2M1); the E8M0
// scales go into TMEM with tcgen05.cp as A's scale factors.  X enters as two
// E4M3 terms with their own E8M0 scales per 32-block (k_xprep_bs): a bf16
// value has 8 significant bits; with s0 = (block's largest exponent) - 7,
// t0 = e4m3(x / 2^s0) keeps 4 of them and t1 = e4m3((x - 2^s0 t0) / 2^(s0-4))
// the rest exactly, so x = 2^s0 t0 + 2^(s0-4) t1 for every element within 13
// binades of its block's largest; smaller ones keep an absolute error below
// 2^-21 of that largest.  Each MMA multiplies exact E2M1 x E4M3 products by
// power-of-two scales and accumulates in FP32 in TMEM: Y matches the
// double-accumulated reference (ref_gemm.hpp:15-27) up to FP32 summation.
//
// Tile: 128 weight rows (UMMA M) x BN activation rows; the two X terms are
// stacked into one B operand of 2 BN rows (UMMA N = 16 .. 256), so each MMA
// reads the W tile once and writes both terms' sums, which the epilogue adds.
// Sub-step: 128 k = one TMA box of W (8 KB from HBM, 16 KB in shared memory),
// one 512-byte scale-factor atom of W, the 2 BN x 128 B X tile and its atom;
// 4 MMAs of K = 32.  Scale-factor atom byte 16 (r % 32) + 4 (r / 32) + b
// holds row r's scale of block b (X: term 0 in rows r < BN, term 1 in rows
// BN + r); tcgen05.cp .32x128b.warpx4 broadcasts the 32 x 16-byte atom to the
// four TMEM lane quadrants and the MMA's scale-factor id selects the block.
// (Issuing the terms as separate MMAs read the W tile twice per block: the
// MMA is bound by shared-memory reads of A, 4 KB per K = 32.)
//
// Schedule: one CTA per SM, stream-K over (tile, sub-step) as in umma_sk.cu:
// whole tiles are stored directly; split tiles leave FP32 partials, which
// k_bs_fixup, launched next, sums in CTA order.  (Summed inside the GEMM by
// the last contributor of each tile, the partials of a tile went through one
// CTA's four epilogue warps after its main loop: 10 us with 2 contributors
// and 47 us with 19 at BN = 64, measured, against 7 us for the whole main
// loop of a 1024 x 28672 shard.)
//
// Warp roles (320 threads), one ring of S stages [W tile | X image | W atom]:
//   warps 0..3   producers, sub-steps round-robin: lane 0 arms the stage and
//                issues the W box (TMA) and the X image (bulk copy); all lanes
//                copy the sub-step's W scale words into the atom with 4-byte
//                cp.async.  No multicast.
//   warp 4       scale factors: once a stage has landed, two tcgen05.cp put its
//                W and X atoms into the stage's TMEM slot; a commit signals
//                the MMA warp.  (Issued from the MMA warp, the copies and
//                their commits blocked it longer than the MMAs themselves.)
//   warp 5       TMEM allocation and MMA issue (warp-wide loop, elected lane):
//                4 MMAs per sub-step, one commit frees the stage.
//   warps 6..9   epilogue: accumulators (double-buffered) to Y or to the
//                split-tile partials.
// Every mbarrier wait is bounded (tc.cuh); on timeout the kernel sets
// g_bs_fault, lets copies and MMAs in flight land, frees TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "tc.cuh"
#include "tp.cuh"

namespace qg {

__device__ unsigned g_bs_fault = 0;

constexpr int kBsK = 128;                  // k per sub-step (one TMA box, one scale atom)
constexpr int kBsRows = 128;               // weight rows per tile
constexpr int kBsWProds = 4;               // producer warps 0..3
constexpr int kBsSfWarp = 4;
constexpr int kBsMmaWarp = 5;
constexpr int kBsEpiWarp0 = 6;
constexpr int kBsThreads = 32 * (kBsEpiWarp0 + 4);  // 320
constexpr uint32_t kBsWTx = kBsRows * kBsK / 2;     // bytes a W box moves from global memory

template <int BN>
struct BsCfg {
  static constexpr int W_A = kBsRows * kBsK;            // unpacked codes: 128 rows x 128 B
  static constexpr int X_T = BN * kBsK;                 // one E4M3 term: BN rows x 128 B
  static constexpr int X_STAGE = 2 * X_T + 1024;        // both terms (2 BN rows) + their atoms
  static constexpr int X_OFF = W_A;                     // stage: [W tile | X image | W atom]
  static constexpr int SFA_OFF = W_A + X_STAGE;
  static constexpr int STAGE = W_A + X_STAGE + 1024;    // 1024-aligned pieces
  static constexpr int S0 = (232448 - 1024 - 512) / STAGE;
  static constexpr int S = S0 > 16 ? 16 : S0;           // ring depth
  static constexpr int NBAR = 3 * S + 4;
  static constexpr int BYTES = 1024 + S * STAGE + NBAR * 8 + 16;
  static constexpr int NB = 2 * BN;                     // UMMA N: both terms
  static constexpr int SFB_ATOMS = (NB + 127) / 128;    // X scale atoms (128 operand rows each)
  static constexpr int SF_STRIDE = 4 + 4 * SFB_ATOMS;   // TMEM columns per stage's scale factors
  static constexpr int ACC_BUFS = (2 * NB + SF_STRIDE * S <= 512) ? 2 : 1;  // accumulator buffers
  static constexpr int SF_COL = ACC_BUFS * NB;          // TMEM: [accumulators | scale factors per stage]
  static constexpr uint32_t TMEM_COLS = (SF_COL + SF_STRIDE * S) <= 256 ? 256u : 512u;
  static_assert(BYTES <= 232448, "shared memory");
  static_assert(S >= 4, "ring depth");
  static_assert(SF_COL + SF_STRIDE * S <= 512, "TMEM columns");
  static_assert(SFB_ATOMS * 512 <= 1024, "X scale atoms fit the stage");
  static_assert(NB <= 256, "UMMA N");
};

struct BsArgs {
  const uint8_t* scales;
  const uint8_t* xbs;   // X image of k_xprep_bs: [M blocks][K / 128][X_STAGE]
  void* Y;
  float* partials;      // [2 * G slots][BN / 4 column quads][128 rows] float4
  int fixup;            // 1: split tiles exist; k_bs_fixup stores them (and runs tp_finish)
  long long T;          // tiles * KS
  int M, N, K;
  int tiles_n;          // tile t -> rows (t % tiles_n) * 128, activations (t / tiles_n) * BN
  int KS;               // sub-steps per tile (K / 128)
  int G;                // CTAs
  TpOut tp;             // world > 0: store into every rank's Y_full, then tp_finish
};

// Shared-memory matrix descriptor of a 32 x 16-byte scale-factor atom:
// contiguous, no swizzle, 8-row core matrices 128 bytes apart.
__device__ __forceinline__ uint64_t sf_atom_desc(uint32_t addr) {
  return (uint64_t)((addr & 0x3FFFFu) >> 4) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(128 >> 4) << 32) |
         ((uint64_t)1 << 46);
}
// Instruction descriptor, kind::mxf8f6f4 with block scaling: A E2M1, B E4M3,
// FP32 accumulator, both K-major, E8M0 scales, scale-factor ids for A and B.
__host__ __device__ constexpr uint32_t idesc_mxf4f8(int M, int N, int sf_id) {
  return ((uint32_t)sf_id << 4) | (5u << 7) | (0u << 10) | ((uint32_t)(N >> 3) << 17) | (1u << 23) |
         ((uint32_t)(M >> 4) << 24) | ((uint32_t)sf_id << 29);
}

// ---------------------------------------------------------------------------
// X preparation: bf16 -> two E4M3 terms with E8M0 block scales, in the
// shared-memory image the kernel copies per sub-step.
// ---------------------------------------------------------------------------
// One warp per (activation row m, sub-step u); lane l holds k = 128u + 4l ..
// + 3, so a 32-block is 8 lanes.  Image of (row block b, sub-step u), at
// ((b * KS) + u) * X_STAGE: term j's tile at j * BN * 128 (row r at r * 128,
// 16-byte chunk c at c ^ (r % 8)), so the two tiles form one 2 BN-row
// operand, then its scale atoms at 2 BN 128 (one per 128 operand rows; term
// 1 in rows BN + r).
// Rows m >= M are zeros.
__device__ __forceinline__ uint32_t e4m3x2_rn(float hi, float lo) {
  uint16_t v;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(v) : "f"(hi), "f"(lo));
  return v;
}
__device__ __forceinline__ float2 e4m3x2_f32(uint32_t v) {  // low byte -> .x
  uint32_t h;
  asm("{ .reg .b16 t; mov.b16 t, %1; cvt.rn.f16x2.e4m3x2 %0, t; }" : "=r"(h) : "h"((uint16_t)v));
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}
__global__ void __launch_bounds__(256) k_xprep_bs(const uint16_t* __restrict__ X, int M, int K, int BN, int nrows,
                                                  uint8_t* __restrict__ img) {
  // Dependents (the GEMM) may launch at once and stream their weights; they
  // read the image only after their own wait, which covers this grid.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int KS = K / kBsK;
  const long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= (long long)nrows * KS) return;
  const int m = (int)(wid / KS), u = (int)(wid % KS);
  const int b = m / BN, r = m % BN;
  float x[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  uint32_t ebits = 0;  // largest biased bf16 exponent of the lane's finite nonzero values
  uint32_t nonfinite = 0;
  if (m < M) {
    const uint2 v = *reinterpret_cast<const uint2*>(X + (size_t)m * K + (size_t)u * kBsK + 4 * lane);
    const uint32_t w[2] = {v.x, v.y};
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      x[2 * i] = u2f(w[i] << 16);
      x[2 * i + 1] = u2f(w[i] & 0xFFFF0000u);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t e = (f2u(x[i]) >> 23) & 0xFFu;
      ebits = (e != 0xFFu && e > ebits) ? e : ebits;
      nonfinite |= (e == 0xFFu) ? 1u : 0u;
    }
  }
  // block maximum over the 8 lanes of the 32-block
  ebits = max(ebits, __shfl_xor_sync(0xFFFFFFFFu, ebits, 1));
  ebits = max(ebits, __shfl_xor_sync(0xFFFFFFFFu, ebits, 2));
  ebits = max(ebits, __shfl_xor_sync(0xFFFFFFFFu, ebits, 4));
  nonfinite |= __shfl_xor_sync(0xFFFFFFFFu, nonfinite, 1);
  nonfinite |= __shfl_xor_sync(0xFFFFFFFFu, nonfinite, 2);
  nonfinite |= __shfl_xor_sync(0xFFFFFFFFu, nonfinite, 4);
  // s0 = E - 7 as an E8M0 byte (E = ebits - 127): ebits - 7, kept in [4, 254]
  int sb0 = (int)ebits - 7;
  sb0 = sb0 < 4 ? 4 : (sb0 > 254 ? 254 : sb0);
  const int sb1 = sb0 - 4;
  const float inv0 = u2f((uint32_t)(254 - sb0) << 23);  // 2^-(sb0 - 127)
  float v0[4], r1[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v0[i] = x[i] * inv0;
  const uint32_t t0a = e4m3x2_rn(v0[1], v0[0]), t0b = e4m3x2_rn(v0[3], v0[2]);
  const float2 q0 = e4m3x2_f32(t0a), q1 = e4m3x2_f32(t0b);
  r1[0] = (v0[0] - q0.x) * 16.0f;
  r1[1] = (v0[1] - q0.y) * 16.0f;
  r1[2] = (v0[2] - q1.x) * 16.0f;
  r1[3] = (v0[3] - q1.y) * 16.0f;
  const uint32_t t1a = e4m3x2_rn(r1[1], r1[0]), t1b = e4m3x2_rn(r1[3], r1[2]);
  uint8_t* base = img + ((size_t)b * KS + u) * (size_t)(2 * BN * kBsK + 1024);
  const int c = lane >> 2;  // 16-byte chunk of the row's 128 k
  const uint32_t off = (uint32_t)(r * kBsK + ((c ^ (r & 7)) << 4) + 4 * (lane & 3));
  *reinterpret_cast<uint32_t*>(base + off) = t0a | (t0b << 16);
  *reinterpret_cast<uint32_t*>(base + BN * kBsK + off) = t1a | (t1b << 16);
  if ((lane & 7) == 0) {
    const int blk = lane >> 3;
    const uint32_t so = (uint32_t)(16 * (r & 31) + 4 * (r >> 5) + blk);  // term 0: row r
    // a block holding an infinity or NaN gets the NaN scale code: every
    // product with it is NaN, as the reference's are non-finite there
    const int r1 = BN + r;  // term 1 is B-operand row BN + r (atom r1 / 128 for 2 BN = 256)
    const uint32_t so1 = (uint32_t)(512 * (r1 >> 7) + 16 * (r1 & 31) + 4 * ((r1 & 127) >> 5) + blk);
    base[2 * BN * kBsK + so] = nonfinite ? (uint8_t)0xFF : (uint8_t)sb0;
    base[2 * BN * kBsK + so1] = nonfinite ? (uint8_t)0xFF : (uint8_t)sb1;
  }
}

// ---------------------------------------------------------------------------
// The GEMM kernel
// ---------------------------------------------------------------------------
template <int BN, bool F32OUT>
__global__ void __launch_bounds__(kBsThreads, 1)
k_umma_bs(const __grid_constant__ CUtensorMap map_w, const BsArgs a) {
  using C = BsCfg<BN>;
  constexpr int S = C::S;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = su32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;  // swizzled tiles want 1024-byte alignment
  uint8_t* gbase = smem_raw + (base - raw);
  auto ST_addr = [&](int s) { return base + (uint32_t)(s * C::STAGE); };
  uint64_t* bars = reinterpret_cast<uint64_t*>(gbase + S * C::STAGE);
  auto full_bar = [&](int s) { return su32(&bars[s]); };
  auto empty_bar = [&](int s) { return su32(&bars[S + s]); };
  auto sfr_bar = [&](int s) { return su32(&bars[2 * S + s]); };
  auto accf_bar = [&](int b) { return su32(&bars[3 * S + b]); };
  auto acce_bar = [&](int b) { return su32(&bars[3 * S + 2 + b]); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::NBAR);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long it0 = (long long)blockIdx.x * a.T / a.G;
  const long long it1 = (long long)(blockIdx.x + 1) * a.T / a.G;
  const int niter = (int)(it1 - it0);
  const int KS = a.KS;
  unsigned* fault = &g_bs_fault;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar(s), 1 + 32);  // lane 0's expect_tx arrival + 32 cp.async arrivals (scale words)
      mbar_init(empty_bar(s), 1);
      mbar_init(sfr_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) { mbar_init(accf_bar(b), 1); mbar_init(acce_bar(b), 4); }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kBsMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                 "r"(C::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // the next call's kernels may launch now; they take SMs as this grid's
  // CTAs finish and read nothing it writes before their own wait returns
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  bool ok = true;

  if (warp < kBsWProds) {
    // ------------------------------ producers ---------------------------------
    const int p = warp;
    const size_t srow = (size_t)a.K / 32;
    int tile = (int)((it0 + p) / KS), kt = (int)((it0 + p) % KS);
    auto issue_w = [&](int s) {  // the W box and the W scale words of sub-step (tile, kt)
      const int n0 = (tile % a.tiles_n) * kBsRows;
      if (lane == 0) {
        mbar_expect_tx(full_bar(s), kBsWTx + (uint32_t)C::X_STAGE);
        tma_load_2d(ST_addr(s), &map_w, kt * kBsK, n0, full_bar(s));
      }
      // scale words of blocks 4 kt .. 4 kt + 3: row r = lane + 32 q at atom byte 16 lane + 4 q
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int r = lane + 32 * q;
        const int n = (n0 + r < a.N) ? n0 + r : a.N - 1;  // rows past N: zero codes, any scale
        const uint8_t* src = a.scales + (size_t)n * srow + (size_t)kt * 4;
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;"
                     ::"r"(ST_addr(s) + (uint32_t)(C::SFA_OFF + 16 * lane + 4 * q)), "l"(src) : "memory");
      }
      asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(full_bar(s)) : "memory");
    };
    auto issue_x = [&](int s, int xtile, int xkt) {  // the X image of sub-step (xtile, xkt)
      const uint8_t* src = a.xbs + ((size_t)(xtile / a.tiles_n) * KS + xkt) * (size_t)C::X_STAGE;
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
          ::"r"(ST_addr(s) + (uint32_t)C::X_OFF), "l"(src), "r"((uint32_t)C::X_STAGE), "r"(full_bar(s))
          : "memory");
    };
    auto advance = [&]() {
      kt += kBsWProds;
      while (kt >= KS) { kt -= KS; ++tile; }
    };
    // W does not depend on the X-preparation grid: the first stages' W goes out first.
    const int pre = niter < S ? niter : S;
    for (int i = p; i < pre; i += kBsWProds) {
      issue_w(i % S);
      advance();
    }
    if (lane == 0) {
      asm volatile("griddepcontrol.wait;" ::: "memory");  // X image made by the preparation grid
      for (int i = p; i < pre; i += kBsWProds) {
        const long long it = it0 + i;
        issue_x(i % S, (int)(it / KS), (int)(it % KS));
      }
    }
    for (int i = pre + ((p - pre % kBsWProds + kBsWProds) % kBsWProds); i < niter; i += kBsWProds) {
      const int s = i % S;
      if (lane == 0) ok = mbar_wait_flag(empty_bar(s), ((i / S) + 1) & 1, fault);
      ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
      if (!ok) break;
      issue_w(s);
      if (lane == 0) issue_x(s, tile, kt);
      advance();
    }
  } else if (warp == kBsSfWarp) {
    // --------------------------- scale factors to TMEM ------------------------
    uint32_t leader;
    asm volatile("{ .reg .pred p; elect.sync _|p, 0xFFFFFFFF; selp.u32 %0, 1, 0, p; }" : "=r"(leader));
    int s = 0;
    uint32_t ph = 0;
    for (int i = 0; i < niter; ++i) {
      ok = mbar_wait_flag(full_bar(s), ph, fault);
      ok = __all_sync(0xFFFFFFFFu, ok);
      if (!ok) break;
      // the atoms were written by cp.async / bulk copies; tcgen05.cp reads through the async proxy
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      const uint32_t st = ST_addr(s);
      const uint32_t sfa = tmem + (uint32_t)(C::SF_COL + C::SF_STRIDE * s), sfb = sfa + 4u;
      if (leader) {
        asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(sfa),
                     "l"(sf_atom_desc(st + C::SFA_OFF)));
#pragma unroll
        for (int t = 0; t < C::SFB_ATOMS; ++t)
          asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(sfb + 4u * t),
                       "l"(sf_atom_desc(st + C::X_OFF + 2 * C::X_T + 512 * t)));
        umma_commit(sfr_bar(s));
      }
      __syncwarp();
      if (++s == S) { s = 0; ph ^= 1u; }
    }
  } else if (warp == kBsMmaWarp) {
    // ------------------------------ MMA issuer --------------------------------
    uint32_t leader;
    asm volatile("{ .reg .pred p; elect.sync _|p, 0xFFFFFFFF; selp.u32 %0, 1, 0, p; }" : "=r"(leader));
    int kt = (int)(it0 % KS), seg = 0;
    int s = 0;
    uint32_t ph = 0;
    for (int i = 0; i < niter; ++i) {
      const bool first = (i == 0) || (kt == 0);
      const bool last = (i == niter - 1) || (kt == KS - 1);
      if (first && i > 0) ++seg;
      const int b = seg % C::ACC_BUFS;
      if (first && seg >= C::ACC_BUFS)
        ok = mbar_wait_flag(acce_bar(b), ((seg / C::ACC_BUFS) + 1) & 1, fault);
      ok = ok && mbar_wait_flag(sfr_bar(s), ph, fault);  // implies the stage has landed
      ok = __all_sync(0xFFFFFFFFu, ok);
      if (!ok) break;
      tc_fence_after();
      const uint32_t wa = ST_addr(s), xa = wa + (uint32_t)C::X_OFF;
      const uint32_t sfa = tmem + (uint32_t)(C::SF_COL + C::SF_STRIDE * s), sfb = sfa + 4u;
      const uint32_t td = tmem + (uint32_t)(b * C::NB);
      // four K = 32 blocks: two MMAs per asm block
#pragma unroll
      for (int kb = 0; kb < 4; kb += 2) {
        const uint64_t a0 = sw128_desc(wa + 32u * kb), a1 = sw128_desc(wa + 32u * (kb + 1));
        const uint64_t b0 = sw128_desc(xa + 32u * kb), b1 = sw128_desc(xa + 32u * (kb + 1));
        asm volatile(
            "{ .reg .pred L, A, T;\n"
            "  setp.ne.b32 L, %0, 0;\n"
            "  setp.ne.b32 A, %1, 0;\n"
            "  setp.eq.b32 T, %0, %0;\n"
            "  @L tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%2], %3, %4, %5, [%6], [%7], A;\n"
            "  @L tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%2], %8, %9, %10, [%6], [%7], T; }\n"
            ::"r"(leader), "r"((first && kb == 0) ? 0u : 1u), "r"(td), "l"(a0), "l"(b0),
              "r"(idesc_mxf4f8(kBsRows, C::NB, kb)), "r"(sfa), "r"(sfb), "l"(a1), "l"(b1),
              "r"(idesc_mxf4f8(kBsRows, C::NB, kb + 1))
            : "memory");
      }
      if (leader) {
        umma_commit(empty_bar(s));
        if (last) umma_commit(accf_bar(b));
      }
      __syncwarp();
      if (++s == S) { s = 0; ph ^= 1u; }
      if (++kt == KS) kt = 0;
    }
  } else if (warp >= kBsEpiWarp0) {
    // ------------------------------ epilogue ----------------------------------
    // Exactly four warps (their named barrier counts 128 threads).
    static_assert(kBsThreads == 32 * (kBsEpiWarp0 + 4), "four epilogue warps");
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int r = 32 * q + lane;
    const uint32_t t_lane = (uint32_t)(32 * q) << 16;
    const int first_tile = (int)(it0 / KS);
    long long it = it0;
    for (int seg = 0; it < it1; ++seg) {
      const int tile = (int)(it / KS), kb = (int)(it % KS);
      const int ke = (int)((kb + (it1 - it)) < KS ? (kb + (it1 - it)) : KS);
      const int b = seg % C::ACC_BUFS;
      ok = ok && mbar_wait_flag(accf_bar(b), (seg / C::ACC_BUFS) & 1, fault);
      ok = __all_sync(0xFFFFFFFFu, ok);
      tc_fence_after();
      const int n = (tile % a.tiles_n) * kBsRows + r, m0 = (tile / a.tiles_n) * BN;
      const bool live = n < a.N;
      const bool whole = (kb == 0 && ke == KS);
      const uint32_t tacc = tmem + t_lane + (uint32_t)(b * C::NB);
      const int slot = 2 * (int)blockIdx.x + (tile == first_tile ? 0 : 1);
      // a split segment's sums: quad q of row r at float4 (q 128 + r), so a
      // warp's stores (and k_bs_fixup's loads) are contiguous
      float4* part = reinterpret_cast<float4*>(a.partials) + (size_t)slot * (kBsRows * BN / 4) + r;
      if (ok) {
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 8) {
          uint32_t v[8], v1[8];  // term 0 and term 1 sums of activation rows c0 .. c0 + 7
          asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                       : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                         "=r"(v[7])
                       : "r"(tacc + (uint32_t)c0));
          asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                       : "=r"(v1[0]), "=r"(v1[1]), "=r"(v1[2]), "=r"(v1[3]), "=r"(v1[4]), "=r"(v1[5]),
                         "=r"(v1[6]), "=r"(v1[7])
                       : "r"(tacc + (uint32_t)(BN + c0)));
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
          for (int u = 0; u < 8; ++u) v[u] = f2u(u2f(v[u]) + u2f(v1[u]));
          if (whole) {
            if (live) {
#pragma unroll
              for (int u = 0; u < 8; ++u) {
                const int m = m0 + c0 + u;
                if (m < a.M) {
                  const float y = u2f(v[u]);
                  if (F32OUT) static_cast<float*>(a.Y)[(size_t)m * a.N + n] = y;
                  else if (a.tp.world > 0) tp_store(a.tp, (size_t)m, n, __float2bfloat16_rn(y));
                  else static_cast<__nv_bfloat16*>(a.Y)[(size_t)m * a.N + n] = __float2bfloat16_rn(y);
                }
              }
            }
          } else {
            __stcg(part + (size_t)(c0 / 4) * kBsRows, make_float4(u2f(v[0]), u2f(v[1]), u2f(v[2]), u2f(v[3])));
            __stcg(part + (size_t)(c0 / 4 + 1) * kBsRows, make_float4(u2f(v[4]), u2f(v[5]), u2f(v[6]), u2f(v[7])));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce_bar(b));  // accumulator buffer free for segment seg + ACC_BUFS
      it += ke - kb;
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
  if (warp == kBsMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS));
  }
  if (a.tp.world > 0 && !a.fixup) tp_finish(a.tp, fault);
}

// ---------------------------------------------------------------------------
// Split-tile fixup.  A tile whose k range CTAs c_lo .. c_hi of k_umma_bs
// shared (c_hi > c_lo) is summed here: one thread per output quad (one
// weight row, four activation rows), the contributors' partials added in CTA
// order starting from zero, the loads of up to 8 contributors in flight
// before the first add.  Launched right after k_umma_bs with programmatic
// dependent launch; its wait returns once the GEMM grid has completed, so
// every partial (and every whole tile's store) has landed.  With a
// tensor-parallel output this kernel, not the GEMM, ends with tp_finish.
// ---------------------------------------------------------------------------
constexpr int kBsMaxSplit = 512;  // split tiles per call: at most G - 1
struct BsSplitList {
  int n;
  int tile[kBsMaxSplit];
};

template <int BN>
constexpr int bs_fix_ctas_per_tile() { return (kBsRows * BN / 4 + 255) / 256; }

template <int BN, bool F32OUT>
__global__ void __launch_bounds__(256) k_bs_fixup(const __grid_constant__ BsSplitList sl, const BsArgs a) {
  constexpr int PER_TILE = kBsRows * BN / 4;  // float4 outputs of a tile
  constexpr int CPT = bs_fix_ctas_per_tile<BN>();
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the GEMM grid: partials and whole tiles
  const int idx = (int)(blockIdx.x % CPT) * 256 + (int)threadIdx.x;  // q 128 + r
  const int tile = sl.tile[blockIdx.x / CPT];
  if (idx < PER_TILE) {
    const int KS = a.KS;
    const long long t0 = (long long)tile * KS, t1 = t0 + KS - 1;
    const int c_lo = (int)(((t0 + 1) * a.G - 1) / a.T), c_hi = (int)(((t1 + 1) * a.G - 1) / a.T);
    const float4* P = reinterpret_cast<const float4*>(a.partials) + idx;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    constexpr int B = 8;
#pragma unroll 1
    for (int c = c_lo; c <= c_hi; c += B) {
      float4 v[B];
#pragma unroll
      for (int u = 0; u < B; ++u)
        if (c + u <= c_hi) {
          const int cc = c + u;
          const int slot = 2 * cc + (tile == (int)(((long long)cc * a.T / a.G) / KS) ? 0 : 1);
          v[u] = __ldcg(P + (size_t)slot * PER_TILE);
        }
#pragma unroll
      for (int u = 0; u < B; ++u)
        if (c + u <= c_hi) {
          acc.x += v[u].x; acc.y += v[u].y; acc.z += v[u].z; acc.w += v[u].w;
        }
    }
    const int q = idx / kBsRows, r = idx % kBsRows;
    const int n = (tile % a.tiles_n) * kBsRows + r, m0 = (tile / a.tiles_n) * BN + 4 * q;
    if (n < a.N) {
      const float y4[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int m = m0 + u;
        if (m < a.M) {
          if (F32OUT) static_cast<float*>(a.Y)[(size_t)m * a.N + n] = y4[u];
          else if (a.tp.world > 0) tp_store(a.tp, (size_t)m, n, __float2bfloat16_rn(y4[u]));
          else static_cast<__nv_bfloat16*>(a.Y)[(size_t)m * a.N + n] = __float2bfloat16_rn(y4[u]);
        }
      }
    }
  }
  if (a.tp.world > 0) tp_finish(a.tp, &g_bs_fault);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

static PFN_cuTensorMapEncodeTiled_v12000 bs_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// Activation rows per tile: the smallest of 8, 16, 32, 64, 128 covering M
// (one tile column for M <= 128).
int umma_bs_bn(int M) { return M <= 8 ? 8 : M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128; }

// Used for 9 <= M <= 128.  Below that the TMA decode kernel is faster: with
// one 8-row activation tile the MMAs here are bound by shared-memory reads
// of the unpacked codes (16 KB written and 16 KB read per 8 KB of weights),
// while the decode kernel reads each code once (measured, gate-up 57344 x
// 8192 MXFP4, M = 1: 64 us here, 59 us there; M = 16: 66 us here, 82 us
// there).
constexpr int kBsMinM = 9;
bool umma_bs_supported(const qgemm_weights_t* w, int M) {
  return w->format == QGEMM_FMT_MXFP4 && M >= kBsMinM && M <= 128 && w->K % kBsK == 0 &&
         w->K <= (size_t)INT32_MAX && w->N <= (size_t)INT32_MAX &&
         (reinterpret_cast<uintptr_t>(w->data) & 31u) == 0 && (reinterpret_cast<uintptr_t>(w->scales) & 3u) == 0;
}

struct BsPlan {
  int bn, tiles_n, tiles, KS, G;
  long long T;
  size_t x_bytes, counter_bytes, partial_bytes;
};
static BsPlan bs_plan(const qgemm_weights_t* w, int M, int sm_count) {
  BsPlan p;
  p.bn = umma_bs_bn(M);
  p.tiles_n = (int)((w->N + kBsRows - 1) / kBsRows);
  p.tiles = p.tiles_n * ((M + p.bn - 1) / p.bn);
  p.KS = (int)(w->K / kBsK);
  p.T = (long long)p.tiles * p.KS;
  p.G = (int)(p.T < sm_count ? p.T : sm_count);
  const size_t xstage = (size_t)2 * p.bn * kBsK + 1024;
  p.x_bytes = (((size_t)((M + p.bn - 1) / p.bn) * p.KS * xstage) + 255) & ~(size_t)255;
  p.counter_bytes = ws_ticket_bytes(w->N);  // unused here: the fixup kernel needs no tickets
  p.partial_bytes = (((size_t)2 * p.G * kBsRows * p.bn * sizeof(float)) + 255) & ~(size_t)255;
  return p;
}
// The tiles that stream-K splits: every CTA boundary c T / G (0 < c < G)
// strictly inside a tile splits it; boundaries rise, so a tile's repeats are
// adjacent.  Writes up to `cap` tile ids to out (may be null); returns the count.
static int bs_split_tiles(const BsPlan& p, int* out, int cap) {
  int n = 0, last = -1;
  for (int c = 1; c < p.G; ++c) {
    const long long b = (long long)c * p.T / p.G;
    if (b % p.KS == 0) continue;
    const int t = (int)(b / p.KS);
    if (t == last) continue;
    if (out && n < cap) out[n] = t;
    ++n;
    last = t;
  }
  return n;
}

// Launches of one call: k_xprep_bs, k_umma_bs and, with split tiles, k_bs_fixup.
int umma_bs_launches(const qgemm_weights_t* w, int M, int sm_count) {
  if (sm_count <= 0) return 2;
  return bs_split_tiles(bs_plan(w, M, sm_count), nullptr, 0) > 0 ? 3 : 2;
}

// [ticket region | X image | partials]
size_t umma_bs_workspace(const qgemm_weights_t* w, int M, int sm_count) {
  const BsPlan p = bs_plan(w, M, sm_count);
  return p.x_bytes + p.counter_bytes + p.partial_bytes;
}

template <int BN, bool F32>
static cudaError_t launch_bs_t(const CUtensorMap& mw, const BsArgs& a, cudaStream_t s) {
  constexpr int BYTES = BsCfg<BN>::BYTES;
  static bool attr[64] = {false};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr[dev]) {
    e = cudaFuncSetAttribute(k_umma_bs<BN, F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, BYTES);
    if (e != cudaSuccess) return e;
    attr[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a.G);
  cfg.blockDim = dim3(kBsThreads);
  cfg.dynamicSmemBytes = BYTES;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_umma_bs<BN, F32>, mw, a);
}
template <bool F32>
static cudaError_t launch_bs(int bn, const CUtensorMap& mw, const BsArgs& a, cudaStream_t s) {
  switch (bn) {
    case 8: return launch_bs_t<8, F32>(mw, a, s);
    case 16: return launch_bs_t<16, F32>(mw, a, s);
    case 32: return launch_bs_t<32, F32>(mw, a, s);
    case 64: return launch_bs_t<64, F32>(mw, a, s);
    default: return launch_bs_t<128, F32>(mw, a, s);
  }
}

// Two launches: k_xprep_bs then k_umma_bs (programmatic dependent launch).
template <int BN, bool F32>
static cudaError_t launch_fix_t(const BsSplitList& sl, const BsArgs& a, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(sl.n * bs_fix_ctas_per_tile<BN>()));
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_bs_fixup<BN, F32>, sl, a);
}
template <bool F32>
static cudaError_t launch_fix(int bn, const BsSplitList& sl, const BsArgs& a, cudaStream_t s) {
  switch (bn) {
    case 8: return launch_fix_t<8, F32>(sl, a, s);
    case 16: return launch_fix_t<16, F32>(sl, a, s);
    case 32: return launch_fix_t<32, F32>(sl, a, s);
    case 64: return launch_fix_t<64, F32>(sl, a, s);
    default: return launch_fix_t<128, F32>(sl, a, s);
  }
}

// ws: umma_bs_workspace bytes.  A third launch, k_bs_fixup, follows when the
// stream-K ranges split tiles (bs_split_tiles).
qgemm_status_t gemm_umma_bs(const qgemm_weights_t* w, const uint16_t* X, int M, void* Y, bool f32, void* ws,
                            int sm_count, cudaStream_t s, const TpOut* tp) {
  if (!umma_bs_supported(w, M)) return fail(QGEMM_ERR_UNSUPPORTED_SHAPE, "block-scaled path: unsupported shape");
  if (sm_count <= 0) return fail(QGEMM_ERR_CUDA, "block-scaled path: no device properties");
  const BsPlan p = bs_plan(w, M, sm_count);
  auto enc = bs_encode_fn();
  if (!enc) return fail(QGEMM_ERR_CUDA, "block-scaled path: cuTensorMapEncodeTiled unavailable");
  CUtensorMap mw;
  cuuint64_t dims[2] = {(cuuint64_t)w->K, (cuuint64_t)w->N};
  cuuint64_t strides[1] = {(cuuint64_t)(w->K / 2)};
  cuuint32_t box[2] = {(cuuint32_t)kBsK, (cuuint32_t)kBsRows}, estr[2] = {1, 1};
  if (enc(&mw, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 2, const_cast<void*>(static_cast<const void*>(w->data)), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return fail(QGEMM_ERR_CUDA, "block-scaled path: cuTensorMapEncodeTiled failed");
  BsSplitList sl;  // the fixup kernel's parameter block
  sl.n = bs_split_tiles(p, sl.tile, kBsMaxSplit);
  if (sl.n > kBsMaxSplit)
    return fail(QGEMM_ERR_UNSUPPORTED_SHAPE, "block-scaled path: %d split tiles, at most %d", sl.n, kBsMaxSplit);
  uint8_t* img = static_cast<uint8_t*>(ws) + p.counter_bytes;
  const int nrows = (M + p.bn - 1) / p.bn * p.bn;
  {
    cudaLaunchConfig_t cfg = {};
    const long long warps = (long long)nrows * p.KS;
    cfg.gridDim = dim3((unsigned)((warps * 32 + 255) / 256));
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, k_xprep_bs, X, M, (int)w->K, p.bn, nrows, img);
    if (e != cudaSuccess) return fail(QGEMM_ERR_CUDA, "block-scaled X preparation: %s", cudaGetErrorString(e));
  }
  BsArgs a;
  a.scales = static_cast<const uint8_t*>(w->scales);
  a.xbs = img;
  a.Y = Y;
  a.partials = reinterpret_cast<float*>(img + p.x_bytes);
  a.T = p.T; a.M = M; a.N = (int)w->N; a.K = (int)w->K;
  a.tiles_n = p.tiles_n; a.KS = p.KS; a.G = p.G;
  a.fixup = sl.n > 0 ? 1 : 0;
  a.tp = {};
  if (tp) {
    if (f32) return fail(QGEMM_ERR_INVALID_ARG, "block-scaled path: tensor-parallel output is bf16");
    a.tp = *tp;
  }
  cudaError_t e = f32 ? launch_bs<true>(p.bn, mw, a, s) : launch_bs<false>(p.bn, mw, a, s);
  if (e != cudaSuccess) return fail(QGEMM_ERR_CUDA, "block-scaled launch: %s", cudaGetErrorString(e));
  if (sl.n > 0) {
    e = f32 ? launch_fix<true>(p.bn, sl, a, s) : launch_fix<false>(p.bn, sl, a, s);
    if (e != cudaSuccess) return fail(QGEMM_ERR_CUDA, "block-scaled fixup launch: %s", cudaGetErrorString(e));
  }
  return QGEMM_OK;
}

cudaError_t umma_bs_fault_clear() {
  const unsigned z = 0;
  return cudaMemcpyToSymbol(g_bs_fault, &z, sizeof(z));
}

unsigned umma_bs_fault() {
  unsigned f = 0;
  if (cudaMemcpyFromSymbol(&f, g_bs_fault, sizeof(f)) != cudaSuccess) return 0xFFFFFFFFu;
  return f;
}

}  // namespace qg
