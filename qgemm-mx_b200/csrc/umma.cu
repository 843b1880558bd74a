// umma.cu -- tile-per-CTA tcgen05 (5th-generation tensor core) W4A16 GEMM
// for M >= 128, and below that where the stream-K kernel (umma_sk.cu) does
// not apply: K % 256 != 0, or weights of fewer than 2^26 codes (NVFP4 and
// INT4 from M = 17, X padded to 32 rows below M = 32).
//
// Y[M,N] = X[M,K] . W[N,K]^T, W packed in the reference layouts
// (titoatwork/qgemm-mx include/qgemm/pack.hpp:14-85); X arrives as the f16
// copy with per-row power-of-two factors made by k_xprep (gemv.cu).
//
// Swap-AB tile: 128 weight rows form the UMMA M side, BN activation rows
// (32..256) the UMMA N side, so one tcgen05.mma.kind::f16 instruction computes
// a [128 x BN x 16] slab and the FP32 accumulator D = Y^T tile lives in TMEM
// (128 lanes x BN columns).  The dequantised operand is written straight into
// TMEM (TS form, below); K is split across CTAs when the tile count alone
// does not fill the SMs, with a deterministic last-arriver reduction.
//
// Every mbarrier wait is bounded by SM cycles; on timeout the kernel sets
// g_umma_fault, gives its in-flight copies a bounded chance to land, frees its
// TMEM and returns (qgemm_umma_status reports it).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "gemv_core.cuh"
#include "tc.cuh"

namespace qg {

__device__ unsigned g_umma_fault = 0;

constexpr int kUBM = 128;  // weight rows per tile (UMMA M)
constexpr int kUBK = 64;   // K per stage (one 128-byte swizzle row of bf16)

struct UmmaArgs {
  const void* scales;
  void* Y;
  int M, N, K;
  float ts;
  int splits;           // K splits per tile (grid z); 1 = no split
  float* partials;      // [tiles][splits][BN][128] FP32 partial accumulators
  unsigned* counters;   // [tiles] arrival tickets (start and end at zero)
};

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------

// Bounded wait; false (and the fault flag set) when the phase never completes.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  return mbar_wait_flag(bar, parity, &g_umma_fault);
}
// ---------------------------------------------------------------------------
// TS variant: dequantised W in TMEM, f16 operands
// ---------------------------------------------------------------------------
//
// For 32 <= M the W stream must stay near HBM speed, so the dequantised
// operand skips shared memory: each dequant thread widens its row's codes
// with cvt.rn.f16x2.e2m1x2, folds the block scale with one f16x2 multiply and
// writes the row into TMEM with tcgen05.st (lane = weight row, 32-bit column
// = two consecutive k); tcgen05.mma takes A from TMEM and B (the f16 copy of
// X made by k_xprep) from shared memory.
//   NVFP4  e2m1 * e4m3 is exact in f16 (<= 6 significant bits, [2^-10, 2688]).
//   MXFP4  2^(e8m0-127) is folded relative to a per-row base exponent
//          b_n = max_blocks(e8m0) - 127 - 13, so every factor 2^(t-b_n) <= 2^13
//          and e2m1 * 2^(t-b_n) <= 49152 fits f16.  Products are exact while
//          t - b_n >= -23 (a 37-binade window below the row's largest block);
//          the next binade rounds to f16's smallest subnormals and blocks
//          below it are flushed to zero.  The epilogue multiplies
//          row n by 2^b_n and column m by the X prescale 2^s_m.
//   INT4   q (exact in f16) times the FP16 group scale, rounded to f16
//          (exact while q s needs <= 11 significant bits, e.g. scales of up
//          to 8 bits; otherwise within 2^-11 relative); rows whose scales
//          could overflow f16 are folded by a power of two the epilogue
//          multiplies back.  Codes widen in (c_i, c_i+4) pairs, so X comes
//          with k_xprep's INT4 pair permutation.
// Warps: 0 TMA producer, 1 MMA issuer, 2..9 dequant (two per TMEM lane
// quadrant, each covering 32 of the 64 k of a stage) and epilogue.

constexpr int kTsThreads = 320;
constexpr int kTsAStages = 4;            // TMEM A stages of 32 columns each
// TMEM columns: accumulator (BN) + A stages; 256 lets two CTAs share an SM.
__host__ __device__ constexpr uint32_t ts_tmem_cols(int bn) { return bn + 32 * kTsAStages <= 256 ? 256u : 512u; }

template <int FMT, int BN, int STAGES, bool F32OUT>
__global__ void __launch_bounds__(kTsThreads, 2)
k_umma_ts(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x, const UmmaArgs a,
          const float* __restrict__ xs) {
  constexpr int B_BYTES = BN * kUBK * 2;
  constexpr int P_BYTES = kUBM * kUBK / 2;
  constexpr int STAGE = B_BYTES + P_BYTES;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = su32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  auto B_addr = [&](int s) { return base + (uint32_t)(s * STAGE); };
  auto P_ptr = [&](int s) { return gbase + s * STAGE + B_BYTES; };
  uint64_t* bars = reinterpret_cast<uint64_t*>(gbase + STAGES * STAGE);
  // full[STAGES] (TMA) | empty[STAGES] (MMA done with smem stage) |
  // aready[kTsAStages] (A stage written) | afree[kTsAStages] (MMA done with A stage) | acc
  auto full_bar = [&](int s) { return su32(&bars[s]); };
  auto empty_bar = [&](int s) { return su32(&bars[STAGES + s]); };
  auto aready_bar = [&](int s) { return su32(&bars[2 * STAGES + s]); };
  auto afree_bar = [&](int s) { return su32(&bars[2 * STAGES + kTsAStages + s]); };
  const uint32_t acc_bar = su32(&bars[2 * STAGES + 2 * kTsAStages]);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 2 * kTsAStages + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kUBM, m0 = blockIdx.y * BN;
  const int ktotal = a.K / kUBK;
  const int kbeg = (int)((long long)blockIdx.z * ktotal / a.splits);
  const int ksteps = (int)((long long)(blockIdx.z + 1) * ktotal / a.splits) - kbeg;  // local steps 0..ksteps-1

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(full_bar(s), 1); mbar_init(empty_bar(s), 1); }
    for (int s = 0; s < kTsAStages; ++s) { mbar_init(aready_bar(s), 256); mbar_init(afree_bar(s), 1); }
    mbar_init(acc_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // accumulator (BN columns) + A stages (kTsAStages x 32)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                 "r"(ts_tmem_cols(BN)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // the next call's kernels may launch now; they take SMs as this grid's
  // CTAs finish and read nothing it writes before their own wait returns
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const uint32_t tmem_a = tmem + (uint32_t)BN;
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {
      asm volatile("griddepcontrol.wait;" ::: "memory");  // X prepared by the previous grid
      const uint32_t tx = (uint32_t)(B_BYTES + P_BYTES);
      for (int ks = 0; ks < ksteps && ok; ++ks) {
        const int s = ks % STAGES;
        if (ks >= STAGES) ok = mbar_wait(empty_bar(s), ((ks / STAGES) + 1) & 1);
        if (!ok) break;
        mbar_expect_tx(full_bar(s), tx);
        tma_load_2d(B_addr(s), &map_x, (kbeg + ks) * kUBK, m0, full_bar(s));
        tma_load_2d(su32(P_ptr(s)), &map_w, (kbeg + ks) * (kUBK / 2), n0, full_bar(s));
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(kUBM, BN);
      for (int ks = 0; ks < ksteps && ok; ++ks) {
        const int s = ks % STAGES, sa = ks % kTsAStages;
        ok = mbar_wait(full_bar(s), (ks / STAGES) & 1) && mbar_wait(aready_bar(sa), (ks / kTsAStages) & 1);
        if (!ok) break;
        tc_fence_after();
        const uint64_t bd = sw128_desc(B_addr(s));
#pragma unroll
        for (int kk = 0; kk < kUBK / 16; ++kk)  // A: 8 TMEM columns per K=16, B: +32 bytes
          umma_f16_ts(tmem, tmem_a + (uint32_t)(sa * 32 + kk * 8), bd + 2 * kk, idesc, (ks | kk) != 0);
        umma_commit(empty_bar(s));
        umma_commit(afree_bar(sa));
      }
      umma_commit(acc_bar);
    }
  } else {
    // dequant: warp w (2..9) covers TMEM lane quadrant q = w % 4 and half
    // h = (w - 2) / 4 of each stage's 64 k (columns 16h .. 16h+15)
    const int q = warp & 3, h = (warp - 2) >> 2;
    const int r = 32 * q + lane;  // weight row within the tile = TMEM lane
    const int n = n0 + r;
    const bool live = n < a.N;
    const uint8_t* sc8 = static_cast<const uint8_t*>(a.scales);
    // Scale bytes come 16 at a time: a group covers SPG K-steps (MXFP4: 8
    // steps x 2 blocks, NVFP4: 4 steps x 4 blocks, INT4 g128: 16 steps x 1/2
    // group, INT4 g64: 8 steps x 1 group).  vec needs the row's scale run to
    // start on a 16-byte boundary; otherwise one load per step.
    constexpr int SPG = (FMT == 0) ? 8 : (FMT == 1) ? 4 : (FMT == 2) ? 16 : 8;
    const size_t srow_bytes = (size_t)a.K / (FMT == 0 ? 32 : FMT == 1 ? 16 : FMT == 2 ? 64 : 32);
    const uint8_t* srow = sc8 + (size_t)n * srow_bytes;
    const bool vec = (srow_bytes % 16 == 0) && ((reinterpret_cast<uintptr_t>(sc8) & 15u) == 0);
    int rbase = 0;  // MXFP4: per-row base exponent
    if (FMT == 0 && live) {
      int tmax = -1000;
      auto fold_max = [&](uint32_t v, int nb) {
#pragma unroll
        for (int t = 0; t < 4; ++t)
          if (t < nb) {
            const int b = (int)((v >> (8 * t)) & 0xFFu);
            if (b != 0xFF && b > tmax) tmax = b;
          }
      };
      if (vec) {
        for (size_t i = 0; i < srow_bytes; i += 16) {
          const uint4 v = *reinterpret_cast<const uint4*>(srow + i);
          fold_max(v.x, 4); fold_max(v.y, 4); fold_max(v.z, 4); fold_max(v.w, 4);
        }
      } else {
        for (size_t i = 0; i < srow_bytes; i += 2) fold_max(*reinterpret_cast<const uint16_t*>(srow + i), 2);
      }
      rbase = (tmax < 0) ? 0 : tmax - 127 - 13;
    }
    // INT4: q * s is formed in f16 (exact while it needs at most 11
    // significant bits, as for scales of up to 8 bits); rows whose largest
    // FP16 scale field e would overflow f16 (|q s| < 2^(e - 11)) are folded
    // by 2^-rbase, rbase = max(0, e - 26), and multiplied back in the epilogue.
    if (FMT >= 2 && live) {
      int emax = 0;
      auto fold16 = [&](uint32_t v) {
        const int e0 = (int)((v >> 10) & 0x1Fu), e1 = (int)((v >> 26) & 0x1Fu);
        emax = max(emax, e0 == 31 ? 0 : e0);
        emax = max(emax, e1 == 31 ? 0 : e1);
      };
      if (vec) {
        for (size_t i = 0; i < srow_bytes; i += 16) {
          const uint4 v = *reinterpret_cast<const uint4*>(srow + i);
          fold16(v.x); fold16(v.y); fold16(v.z); fold16(v.w);
        }
      } else {
        for (size_t i = 0; i < srow_bytes; i += 2) fold16(*reinterpret_cast<const uint16_t*>(srow + i));
      }
      rbase = emax > 26 ? emax - 26 : 0;
    }
    uint4 grp_cur = make_uint4(0, 0, 0, 0), grp_nxt = make_uint4(0, 0, 0, 0);
    int grp_id = -1;
    auto load_group = [&](int g) -> uint4 {
      if (!live || (size_t)g * 16 >= srow_bytes) return make_uint4(0, 0, 0, 0);
      return *reinterpret_cast<const uint4*>(srow + (size_t)g * 16);
    };
    // scale bits of (absolute) step gk for this thread's half h
    auto load_scale = [&](int gk) -> uint32_t {
      if (!live) return 0u;
      if (!vec) {
        if (FMT == 0) return srow[gk * 2 + h];
        if (FMT == 2) return *reinterpret_cast<const uint16_t*>(srow + (gk >> 1) * 2);
        if (FMT == 3) return *reinterpret_cast<const uint16_t*>(srow + gk * 2);
        return *reinterpret_cast<const uint16_t*>(srow + gk * 4 + 2 * h);
      }
      const int g = gk / SPG;
      if (g != grp_id) {  // entering a new group: the next one starts loading now
        grp_cur = (grp_id >= 0 && g == grp_id + 1) ? grp_nxt : load_group(g);
        grp_nxt = load_group(g + 1);
        grp_id = g;
      }
      const int byte = (FMT == 0) ? (gk % SPG) * 2 + h
                     : (FMT == 1) ? (gk % SPG) * 4 + 2 * h
                     : (FMT == 2) ? ((gk % SPG) >> 1) * 2 : (gk % SPG) * 2;
      const int wi = byte >> 2;
      const uint32_t wv = wi == 0 ? grp_cur.x : wi == 1 ? grp_cur.y : wi == 2 ? grp_cur.z : grp_cur.w;
      return (FMT == 0) ? ((wv >> (8 * (byte & 3))) & 0xFFu) : ((wv >> (8 * (byte & 3))) & 0xFFFFu);
    };
    // Produce step ks into registers: wait for its packed tile and for its
    // TMEM A stage to be free, widen, fold the block scale.
    auto produce = [&](int ks, uint32_t sc, uint32_t (&o)[16]) -> bool {
      const int s = ks % STAGES, sa = ks % kTsAStages;
      if (!mbar_wait(full_bar(s), (ks / STAGES) & 1)) return false;
      if (ks >= kTsAStages && !mbar_wait(afree_bar(sa), ((ks / kTsAStages) + 1) & 1)) return false;
      const uint4 pk = *reinterpret_cast<const uint4*>(P_ptr(s) + r * 32 + 16 * h);  // 32 codes
      const uint32_t qw[4] = {pk.x, pk.y, pk.z, pk.w};
      if constexpr (FMT >= 2) {
        // INT4: pairs (c_i, c_i+4) of each 8 codes, the order the X copy of
        // k_xprep (INT4 pair permutation) holds; times the FP16 group scale,
        // folded by 2^-rbase
#pragma unroll
        for (int w4 = 0; w4 < 4; ++w4) {
          uint32_t t[4];
          int4x8_to_f16(qw[w4], t);
#pragma unroll
          for (int i = 0; i < 4; ++i) o[4 * w4 + i] = t[i];
        }
        const uint32_t f = hmul2_f16x2((sc & 0xFFFFu) | (sc << 16), f16x2_pow2(-rbase));
#pragma unroll
        for (int i = 0; i < 16; ++i) o[i] = hmul2_f16x2(o[i], f);
      } else {
#pragma unroll
        for (int w4 = 0; w4 < 4; ++w4) e2m1x8_to_f16x2(qw[w4], o + 4 * w4);
        if constexpr (FMT == 0) {
          const uint32_t b = sc & 0xFFu;
          const uint32_t f = (b == 0xFFu) ? 0x7E007E00u : f16x2_pow2((int)b - 127 - rbase);
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = hmul2_f16x2(o[i], f);
        } else {
          // normal E4M3 codes by bit placement; zero, subnormal or NaN codes
          // anywhere in the warp through the exact decoder (one uniform branch)
          uint32_t f0, f1;
          const bool fast = e4m3x2_to_f16x2_fast(sc & 0xFFFFu, f0, f1);
          if (__any_sync(0xFFFFFFFFu, !fast)) {
            f0 = f16x2_e4m3(sc & 0xFFu);
            f1 = f16x2_e4m3((sc >> 8) & 0xFFu);
          }
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = hmul2_f16x2(o[i], i < 8 ? f0 : f1);
        }
      }
      return true;
    };
    // Each step is released to the MMA as soon as its TMEM store has
    // landed; the next step is widened after that.
    uint32_t cur[16];
    if (ksteps > 0) ok = produce(0, load_scale(kbeg), cur);
    for (int ks = 0; ks < ksteps && ok; ++ks) {
      const int sa = ks % kTsAStages;
      tmem_st16(tmem_a + ((uint32_t)(32 * q) << 16) + (uint32_t)(sa * 32 + 16 * h), cur);
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      mbar_arrive(aready_bar(sa));
      if (ks + 1 < ksteps) ok = produce(ks + 1, load_scale(kbeg + ks + 1), cur);
    }

    // epilogue: the warps of half 0 (one per TMEM lane quadrant) drain the
    // accumulator.  With split K every split parks its FP32 tile in the
    // workspace and the split that arrives last sums them in split order.
    if (h == 0) {
      if (ok) ok = mbar_wait(acc_bar, 0);
      tc_fence_after();
      asm volatile("griddepcontrol.wait;" ::: "memory");  // xs written by the X-preparation grid
      const float rowf = (FMT != 1) ? ((rbase >= -126) ? u2f((uint32_t)(127 + rbase) << 23) : ldexpf(1.0f, rbase))
                                    : a.ts;
      auto store = [&](int m, float acc) {
        if (live && m < a.M) {
          const float y = acc * rowf * xs[m];
          if (F32OUT) static_cast<float*>(a.Y)[(size_t)m * a.N + n] = y;
          else static_cast<__nv_bfloat16*>(a.Y)[(size_t)m * a.N + n] = __float2bfloat16_rn(y);
        }
      };
      const size_t tile_lin = (size_t)blockIdx.y * gridDim.x + blockIdx.x;
      float* part = a.partials + (tile_lin * a.splits + blockIdx.z) * (size_t)(BN * kUBM);
      if (ok) {
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          uint32_t v[16];
          tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, v);
          if (a.splits == 1) {
#pragma unroll
            for (int i = 0; i < 16; ++i) store(m0 + c0 + i, u2f(v[i]));
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) __stcg(part + (size_t)(c0 + i) * kUBM + r, u2f(v[i]));
          }
        }
      }
      if (a.splits > 1) {
        __shared__ unsigned s_ticket;
        __threadfence();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (warp == 2 && lane == 0) s_ticket = atomicAdd(a.counters + tile_lin, 1u);  // also after a timeout: the tickets still return to zero
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (s_ticket == (unsigned)(a.splits - 1)) {
          __threadfence();
          const float* base = a.partials + tile_lin * a.splits * (size_t)(BN * kUBM);
          // 16 columns at a time with up to two splits' loads in flight
          // before the first add (they come from L2; one load and add per
          // column and split made this a chain of BN x splits round trips);
          // the adds stay in split order
#pragma unroll 1
          for (int c0 = 0; c0 < BN; c0 += 16) {
            float acc[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) acc[i] = 0.0f;
#pragma unroll 1
            for (int z0 = 0; z0 < a.splits; z0 += 2) {
              float pv[2][16];
#pragma unroll
              for (int j = 0; j < 2; ++j)
                if (z0 + j < a.splits) {
#pragma unroll
                  for (int i = 0; i < 16; ++i)
                    pv[j][i] = __ldcg(base + (size_t)(z0 + j) * (BN * kUBM) + (size_t)(c0 + i) * kUBM + r);
                }
#pragma unroll
              for (int j = 0; j < 2; ++j)
                if (z0 + j < a.splits) {
#pragma unroll
                  for (int i = 0; i < 16; ++i) acc[i] += pv[j][i];
                }
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) store(m0 + c0 + i, acc[i]);
          }
          if (warp == 2 && lane == 0) a.counters[tile_lin] = 0u;  // leave the workspace zeroed
        }
      }
    }
  }

  if (!ok && threadIdx.x == 0) {
    fault_drain();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ts_tmem_cols(BN)));
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

bool make_tma_map_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* ptr, uint64_t inner, uint64_t outer,
                        uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Largest supported tile width not above M, so a TMA box never exceeds the
// X tensor's row count.
template <int FMT, int BN, int STAGES, bool F32>
static cudaError_t launch_ts_t(const CUtensorMap& mw, const CUtensorMap& mx, const UmmaArgs& a, const float* xs,
                               cudaStream_t s) {
  constexpr int BYTES = STAGES * (BN * kUBK * 2 + kUBM * kUBK / 2) + 1024 + 512;
  static bool attr[64] = {false};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    e = cudaFuncSetAttribute(k_umma_ts<FMT, BN, STAGES, F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, BYTES);
    if (e != cudaSuccess) return e;
    attr[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((a.N + kUBM - 1) / kUBM), (unsigned)((a.M + BN - 1) / BN), (unsigned)a.splits);
  cfg.blockDim = dim3(kTsThreads);
  cfg.dynamicSmemBytes = BYTES;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_umma_ts<FMT, BN, STAGES, F32>, mw, mx, a, xs);
}

template <int FMT, bool F32>
static cudaError_t launch_ts_bn(int bn, const CUtensorMap& mw, const CUtensorMap& mx, const UmmaArgs& a,
                                const float* xs, cudaStream_t s) {
  switch (bn) {
    case 32: return launch_ts_t<FMT, 32, 10, F32>(mw, mx, a, xs, s);   //  80 KB: 2 CTAs/SM
    case 64: return launch_ts_t<FMT, 64, 8, F32>(mw, mx, a, xs, s);    //  96 KB: 2 CTAs/SM
    case 128: return launch_ts_t<FMT, 128, 5, F32>(mw, mx, a, xs, s);  // 100 KB: 2 CTAs/SM
    default: return launch_ts_t<FMT, 256, 4, F32>(mw, mx, a, xs, s);   // 144 KB, 512 TMEM columns
  }
}

int umma_bn_for(int M) { return M >= 256 ? 256 : M >= 128 ? 128 : M >= 64 ? 64 : 32; }

// TS path: Xh / xs are the f16 copy of X and its row factors (k_xprep); for
// M < 32 Xh holds 32 rows, the ones past M zero.
// K splits for a launch: enough CTAs to fill every SM slot when the tile
// count alone does not, each split keeping >= 8 K-steps.
int umma_splits(const qgemm_weights_t* w, int M, int sm_count) {
  const int bn = umma_bn_for(M);
  const long long tiles = (long long)((w->N + kUBM - 1) / kUBM) * ((M + bn - 1) / bn);
  const long long slots = (long long)sm_count * (bn <= 128 ? 2 : 1);
  long long s = slots / (tiles > 0 ? tiles : 1);
  const long long kmax = (long long)(w->K / kUBK) / 8;
  if (s > kmax) s = kmax;
  // split tiles take one ticket each in the workspace's ticket region (fewer
  // than sm_count tiles whenever s >= 2)
  if ((size_t)tiles * sizeof(unsigned) > ws_ticket_bytes(w->N)) s = 1;
  return s < 1 ? 1 : (int)s;
}
size_t umma_split_workspace(const qgemm_weights_t* w, int M, int splits) {
  if (splits <= 1) return 0;
  const int bn = umma_bn_for(M);
  const size_t tiles = ((w->N + kUBM - 1) / kUBM) * (size_t)((M + bn - 1) / bn);
  return tiles * (size_t)splits * bn * kUBM * sizeof(float);
}

qgemm_status_t gemm_umma_ts(const qgemm_weights_t* w, const __half* Xh, const float* xs, int M, void* Y, bool f32,
                            int splits, unsigned* tickets, void* partials, cudaStream_t s) {
  if (w->format != QGEMM_FMT_MXFP4 && w->format != QGEMM_FMT_NVFP4 && w->format != QGEMM_FMT_INT4_G128 &&
      w->format != QGEMM_FMT_INT4_G64)
    return fail(QGEMM_ERR_UNSUPPORTED_SHAPE, "umma path: unknown format");
  if (w->K % kUBK != 0 || w->K > (size_t)INT32_MAX || w->N > (size_t)INT32_MAX)
    return fail(QGEMM_ERR_UNSUPPORTED_SHAPE, "umma path: K must be a multiple of %d", kUBK);
  const int bn = umma_bn_for(M);
  CUtensorMap mw, mx;
  if (!make_tma_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w->data, w->K / 2, w->N, w->K / 2, kUBK / 2, kUBM,
                   CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_tma_map_2d(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, Xh, w->K, (uint64_t)(M < 32 ? 32 : M), w->K * 2, kUBK,
                   (uint32_t)bn, CU_TENSOR_MAP_SWIZZLE_128B))
    return fail(QGEMM_ERR_CUDA, "umma path: cuTensorMapEncodeTiled failed");
  UmmaArgs a;
  a.scales = w->scales; a.Y = Y; a.M = M; a.N = (int)w->N; a.K = (int)w->K; a.ts = w->tensor_scale;
  a.splits = splits < 1 ? 1 : splits;
  a.counters = nullptr; a.partials = nullptr;
  if (a.splits > 1) {
    const size_t tiles = ((w->N + kUBM - 1) / kUBM) * (size_t)((M + bn - 1) / bn);
    if (tiles * sizeof(unsigned) > ws_ticket_bytes(w->N))
      return fail(QGEMM_ERR_WORKSPACE, "umma path: %zu split tiles exceed the ticket region", tiles);
    a.counters = tickets;
    a.partials = static_cast<float*>(partials);
  }
  cudaError_t e;
  switch (w->format) {
    case QGEMM_FMT_MXFP4:
      e = f32 ? launch_ts_bn<0, true>(bn, mw, mx, a, xs, s) : launch_ts_bn<0, false>(bn, mw, mx, a, xs, s);
      break;
    case QGEMM_FMT_NVFP4:
      e = f32 ? launch_ts_bn<1, true>(bn, mw, mx, a, xs, s) : launch_ts_bn<1, false>(bn, mw, mx, a, xs, s);
      break;
    case QGEMM_FMT_INT4_G128:
      e = f32 ? launch_ts_bn<2, true>(bn, mw, mx, a, xs, s) : launch_ts_bn<2, false>(bn, mw, mx, a, xs, s);
      break;
    default:
      e = f32 ? launch_ts_bn<3, true>(bn, mw, mx, a, xs, s) : launch_ts_bn<3, false>(bn, mw, mx, a, xs, s);
      break;
  }
  if (e != cudaSuccess) return fail(QGEMM_ERR_CUDA, "umma launch: %s", cudaGetErrorString(e));
  return QGEMM_OK;
}

unsigned umma_sk_fault();
unsigned gemv_tma_fault();
unsigned umma_bs_fault();
cudaError_t umma_sk_fault_clear();
cudaError_t gemv_tma_fault_clear();
cudaError_t umma_bs_fault_clear();
cudaError_t tp_fault_clear();
cudaError_t probe_fault_clear();

}  // namespace qg

using namespace qg;

extern "C" {

qgemm_status_t qgemm_umma_status(int32_t* faulted) {
  unsigned f = 0;
  QG_CUDA_RET(cudaMemcpyFromSymbol(&f, g_umma_fault, sizeof(f)));
  const unsigned g = umma_sk_fault(), h = gemv_tma_fault(), b = umma_bs_fault();
  if (g == 0xFFFFFFFFu || h == 0xFFFFFFFFu || b == 0xFFFFFFFFu)
    return fail(QGEMM_ERR_CUDA, "umma: reading a fault flag failed");
  if (faulted) *faulted = (int32_t)(f | g | h | b);
  if (!(f | g | h | b)) return QGEMM_OK;
  // each flag holds where its kernel's first wait gave up (0x8wwcccbb: warp,
  // CTA, barrier index) or 1
  return fail(QGEMM_ERR_TIMEOUT,
              "umma: a bounded barrier wait gave up (sites: tile %08x, stream-K %08x, decode %08x, block-scaled %08x)",
              f, g, h, b);
}

qgemm_status_t qgemm_clear_faults(void) {
  QG_CUDA_RET(cudaDeviceSynchronize());  // no kernel may still be setting a flag
  const unsigned z = 0;
  QG_CUDA_RET(cudaMemcpyToSymbol(g_umma_fault, &z, sizeof(z)));
  QG_CUDA_RET(umma_sk_fault_clear());
  QG_CUDA_RET(gemv_tma_fault_clear());
  QG_CUDA_RET(umma_bs_fault_clear());
  QG_CUDA_RET(tp_fault_clear());
  QG_CUDA_RET(probe_fault_clear());
  return QGEMM_OK;
}

}  // extern "C"
