// tp.cuh -- output side of the tensor-parallel GEMM, shared by the kernels
// that write their Y slice straight into every rank's Y_full.
//
// A kernel given a TpOut with world > 0 stores each bf16 result at
// y[d][m * ldy + col0 + n] for every rank d (the peer mappings; NVLink P2P
// stores) and ends with tp_finish, called by every thread of every CTA:
//   * after a CTA barrier, one thread per destination rank d adds the CTA's
//     share to arrival slot [rank] of rank d's sync block with a
//     system-scope release reduction.  The release is cumulative over the
//     whole CTA's stores (they precede it through the barrier), so a rank
//     that has seen a sender's shares has seen the stores behind them.
//     The shares of a call's CTAs sum to exactly kTpCallUnits whatever the
//     grid size: share(b) = floor((b + 1) U / G) - floor(b U / G);
//   * CTA 0 raises this rank's expected count by kTpCallUnits and waits
//     (bounded, acquire loads of its own sync block) until every rank's slot
//     has reached it.
// Counters wrap modulo 2^32 and are compared by signed difference, which is
// exact while ranks are fewer than 2^15 calls apart (a rank is at most one
// call ahead: it waits for the others at the end of every call).
//
// Sync block of a rank (uint32 words, qgemm_tp_sync_bytes): [0, kTpMaxWorld)
// arrival slots, then the expected count, then one reserved word.  Zero it
// once before the first call; every rank must make the same sequence of calls.
#pragma once

#include <cuda_bf16.h>

#include "common.cuh"

namespace qg {

constexpr int kTpMaxWorld = 8;
// The completion wait's bound in SM cycles (clock64 moves only forward on an
// SM; the driver may step %globaltimer): ~2 s at 2 GHz, longer at lower clocks.
constexpr unsigned long long kTpWaitCycles = 4000000000ull;
constexpr uint32_t kTpCallUnits = 1u << 16;              // arrival units per call and sender

struct TpOut {
  int world;   // 0: not a tensor-parallel launch
  int rank;
  int col0;    // this rank's first column in Y_full
  int ldy;     // Y_full row pitch (N of the full matrix)
  uint16_t* y[kTpMaxWorld];
  uint32_t* sync[kTpMaxWorld];
};

__device__ __forceinline__ void tp_store(const TpOut& t, size_t m, int n, __nv_bfloat16 v) {
  const uint16_t b = __bfloat16_as_ushort(v);
  const size_t off = m * (size_t)t.ldy + (size_t)(t.col0 + n);
  for (int d = 0; d < t.world; ++d) t.y[d][off] = b;
}

__device__ __forceinline__ unsigned long long tp_cycles() { return (unsigned long long)clock64(); }

// Called by every thread of every CTA after its last Y store; a wait that
// gives up sets *fault (the calling kernel's own flag).
__device__ __forceinline__ void tp_finish(const TpOut& t, unsigned* fault) {
  __syncthreads();  // every store of this CTA precedes the releases below
  const int tid = threadIdx.x;
  if (tid < t.world) {
    const uint32_t G = gridDim.x, b = blockIdx.x;
    const uint32_t share = (uint32_t)((((unsigned long long)(b + 1)) * kTpCallUnits) / G -
                                      (((unsigned long long)b) * kTpCallUnits) / G);
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(t.sync[tid] + t.rank), "r"(share) : "memory");
  }
  if (blockIdx.x != 0 || tid >= 32) return;
  uint32_t* mine = t.sync[t.rank];
  uint32_t expect = 0;
  if (tid == 0) {  // only CTA 0 of this rank's launches touches the expected count; launches are stream-ordered
    expect = mine[kTpMaxWorld] + kTpCallUnits;
    mine[kTpMaxWorld] = expect;
  }
  expect = __shfl_sync(0xFFFFFFFFu, expect, 0);
  bool ok = true;
  if (tid < t.world) {
    const unsigned long long c0 = tp_cycles();
    for (;;) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine + tid) : "memory");
      if ((int32_t)(v - expect) >= 0) break;
      if (tp_cycles() - c0 > kTpWaitCycles) { ok = false; break; }
    }
  }
  if (!ok) atomicCAS(fault, 0u, 1u);
}

}  // namespace qg
