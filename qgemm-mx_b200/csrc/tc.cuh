// tc.cuh -- PTX wrappers shared by the tcgen05 kernels: mbarriers, TMA tile
// loads, tcgen05 fences / commits / TMEM loads and stores, shared-memory
// matrix and instruction descriptors for kind::f16.
//
// Every wait is bounded by SM cycles: mbar_wait returns false and sets the
// caller's fault flag once the phase has not completed within kWaitCycles.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace qg {

// Bounds of the device-side waits.  They count SM cycles (clock64, which
// only moves forward on an SM) and polls, not %globaltimer: the driver may
// step the global timer, and one step backwards wrapped the unsigned
// difference and ended a healthy wait at once (intermittent "a bounded
// barrier wait gave up" on an otherwise normal run, and a teardown whose
// drain, timed the same way, freed TMEM under copies still in flight).
constexpr unsigned long long kWaitCycles = 4000000000ull;  // ~2 s at 2 GHz, longer at lower clocks
constexpr int kWaitMinPolls = 1000;                          // a poll sleeps up to ~1 ms
constexpr unsigned long long kDrainCycles = 100000000ull;  // ~50 ms at 2 GHz

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ unsigned long long sm_cycles() { return (unsigned long long)clock64(); }
// After a wait gave up: let the CTA's copies and MMAs in flight land before
// it frees TMEM and exits.
__device__ __forceinline__ void fault_drain() {
  const unsigned long long c0 = sm_cycles();
  while (sm_cycles() - c0 < kDrainCycles) { }
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// try_wait with a suspend-time hint: a waiting thread sleeps until the phase
// completes (or about 1 ms passes) instead of spinning, so warps that wait
// for long stretches do not take issue slots from the warps doing the work.
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok) : "r"(bar), "r"(parity), "r"(1000000u) : "memory");
  return ok != 0;
}
// Where a wait gave up, as the first value a fault flag takes: bit 31 set,
// warp in bits 24..30, CTA in bits 8..23, and the barrier's index in its
// 1024-byte-aligned barrier block (the kernels keep their mbarriers at the
// start of such a block) in bits 0..7.
__device__ __forceinline__ unsigned fault_site(uint32_t bar) {
  return 0x80000000u | (((threadIdx.x >> 5) & 0x7Fu) << 24) | ((blockIdx.x & 0xFFFFu) << 8) | ((bar & 0x3FFu) >> 3);
}
// Bounded wait; false (and *fault set to the wait's site unless already
// set) when the phase never completes.
__device__ __forceinline__ bool mbar_wait_flag(uint32_t bar, uint32_t parity, unsigned* fault) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long c0 = sm_cycles();
  int polls = 1;
  for (;;) {
    if (mbar_try(bar, parity)) return true;
    if (polls < kWaitMinPolls) ++polls;  // saturates
    else if (sm_cycles() - c0 > kWaitCycles) {
      atomicCAS(fault, 0u, fault_site(bar));
      return false;
    }
  }
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// K-major, SWIZZLE_128B shared-memory matrix descriptor: 8-row atoms of
// 128-byte rows, 1024 bytes apart (stride byte offset), version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  return (uint64_t)((addr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor: kind::f16, A = B = bf16, D = f32, both K-major.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// Instruction descriptor: kind::f16, A = B = f16 (format code 0), D = f32.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// D(tmem) (+)= A(tmem) . B(smem descriptor)
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc,
                                            uint32_t acc) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p; }"
      ::"r"(tmem_d), "r"(tmem_a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// 32 lanes x 16 columns of 32 bits; waits for completion.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

// 32 lanes x 32 columns of 32 bits, one instruction.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
        "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]),
        "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

// byte t of q (codes 2t, 2t+1) -> f16x2 (low half = even code), sign included
__device__ __forceinline__ void e2m1x8_to_f16x2(uint32_t q, uint32_t* o) {
  asm("{ .reg .b8 b0, b1, b2, b3;\n"
      "  mov.b32 {b0, b1, b2, b3}, %4;\n"
      "  cvt.rn.f16x2.e2m1x2 %0, b0;\n"
      "  cvt.rn.f16x2.e2m1x2 %1, b1;\n"
      "  cvt.rn.f16x2.e2m1x2 %2, b2;\n"
      "  cvt.rn.f16x2.e2m1x2 %3, b3; }\n"
      : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
      : "r"(q));
}
__device__ __forceinline__ uint32_t hmul2_f16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// f16x2 broadcast of 2^e: normal for e >= -14, subnormal down to 2^-24,
// zero below.  (Callers keep e <= 15.)
__device__ __forceinline__ uint32_t f16x2_pow2(int e) {
  const uint32_t nrm = (uint32_t)(e + 15) << 10;               // e >= -14
  const uint32_t sub = 1u << ((e + 24) & 31);                  // -24 <= e < -14
  const uint32_t h = e >= -14 ? nrm : (e >= -24 ? sub : 0u);   // selects, no branches
  return h | (h << 16);
}
// f16x2 broadcast of an E4M3 value (exact; NaN code -> f16 NaN).
__device__ __forceinline__ uint32_t f16x2_e4m3(uint32_t b) {
  const uint32_t h = (uint32_t)__half_as_ushort(__float2half_rn(e4m3_decode(b & 0xFFu)));
  return h | (h << 16);
}

}  // namespace qg
