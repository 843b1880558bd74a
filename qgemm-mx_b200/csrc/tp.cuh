// tp.cuh -- output side of the tensor-parallel GEMM, shared by the kernels
// that write their Y slice straight into every rank's Y_full.
//
// A kernel given a TpOut with world > 0 stores each bf16 result at
// y[d][m * ldy + col0 + n] for every rank d (the peer mappings; NVLink P2P
// stores), and finishes with tp_finish: every thread fences its stores at
// system scope, the CTA takes a ticket, and the CTA that finishes last
// announces the call's epoch in every rank's sync block and waits (bounded)
// until every rank has announced it in this rank's block.
//
// Sync block of a rank: uint32 [kTpMaxWorld] arrival slots, the local call
// counter, the CTA ticket counter (qgemm_tp_sync_bytes).
#pragma once

#include <cuda_bf16.h>

#include "common.cuh"

namespace qg {

constexpr int kTpMaxWorld = 8;
constexpr unsigned long long kTpWaitNs = 2000000000ull;  // 2 s

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

__device__ __forceinline__ unsigned long long tp_gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Called by every thread of every CTA after its last Y store; a wait that
// gives up sets *fault (the calling kernel's own flag).
__device__ __forceinline__ void tp_finish(const TpOut& t, unsigned* fault) {
  __threadfence_system();  // this thread's peer stores are performed
  __syncthreads();
  uint32_t* mine = t.sync[t.rank];
  __shared__ unsigned s_tp_last;
  __shared__ uint32_t s_tp_epoch;
  if (threadIdx.x == 0) s_tp_last = (atomicAdd(mine + kTpMaxWorld + 1, 1u) == gridDim.x - 1) ? 1u : 0u;
  __syncthreads();
  if (!s_tp_last || threadIdx.x >= 32) return;
  // the last CTA: every CTA's stores were fenced before its ticket
  const int lane = threadIdx.x;
  if (lane == 0) {
    mine[kTpMaxWorld + 1] = 0u;                 // ticket counter back to zero for the next launch
    const uint32_t e = mine[kTpMaxWorld] + 1u;  // call counter: same sequence on every rank
    mine[kTpMaxWorld] = e;
    s_tp_epoch = e;
  }
  __syncwarp();
  const uint32_t epoch = s_tp_epoch;
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  if (lane < t.world)
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(t.sync[lane] + t.rank), "r"(epoch) : "memory");
  bool ok = true;
  if (lane < t.world) {
    const unsigned long long t0 = tp_gtimer();
    for (;;) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine + lane) : "memory");
      if ((int32_t)(v - epoch) >= 0) break;
      if (tp_gtimer() - t0 > kTpWaitNs) { ok = false; break; }
    }
  }
  if (!ok) atomicExch(fault, 1u);
}

}  // namespace qg
