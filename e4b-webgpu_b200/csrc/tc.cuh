// 5th-generation tensor-core (tcgen05) and TMA building blocks shared by the
// warp-specialised GEMMs (tcgemm.cu: batched-prefill q4_0; q6tc.cu: batched
// q6_K LM head):
//   - bounded mbarrier waits that give up with E4B_ST_TIMEOUT (or as soon as
//     another CTA has recorded one),
//   - 2-D TMA tile loads, cp.async with a source size (zero fill),
//   - tcgen05.mma kind::f16 (cta_group::1), commit, TMEM loads, and the
//     shared-memory / instruction descriptors for K-major 128-byte-swizzled
//     operands.
#pragma once

#include "stream.cuh"

namespace e4b {

E4B_DEV bool tc_aborted(const uint32_t* status) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(status) : "memory");
  return (v & E4B_ST_TIMEOUT) != 0;
}
// try_wait that lets the hardware suspend the thread until the phase completes
// or about `hint_ns` pass (instead of the short default), so waiting warps do
// not take issue slots from the working ones.
E4B_DEV bool mbar_try_wait_sleep(uint64_t* b, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
// Bounded mbarrier wait; false after limit_ns (recording E4B_ST_TIMEOUT) or once
// any CTA has recorded a time-out.
E4B_DEV bool wait_bar(uint64_t* b, uint32_t parity, uint32_t* status, uint64_t limit_ns) {
  if (mbar_try_wait(b, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0;; i++) {
    if (mbar_try_wait_sleep(b, parity, 20000u)) return true;
    if ((i & 63u) == 63u) {
      if (tc_aborted(status)) return false;
      if (globaltimer_ns() - t0 > limit_ns) {
        set_status(status, E4B_ST_TIMEOUT);
        return false;
      }
    }
  }
}
// Wait (bounded, no status) for a barrier phase: used while draining copies
// still in flight before a CTA ends.
E4B_DEV void drain_bar(uint64_t* b, uint32_t parity, uint64_t limit_ns) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(b, parity) && globaltimer_ns() - t0 < limit_ns) {
  }
}
E4B_DEV void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}
// 16-byte cp.async reading src_bytes (<= 16) and zero-filling the rest.
E4B_DEV void cp_async16z(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
E4B_DEV void cp_async_commit_group() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
E4B_DEV void cp_async_wait_group() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

E4B_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
E4B_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
E4B_DEV void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
E4B_DEV void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// 32 consecutive accumulator columns of this thread's TMEM lane (no wait).
E4B_DEV void tc_ld32_nowait(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
E4B_DEV void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// store 32 consecutive accumulator columns of this thread's TMEM lane
E4B_DEV void tc_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
E4B_DEV void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
E4B_DEV void tc_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  tc_ld32_nowait(taddr, r);
  tc_wait_ld();
#pragma unroll
  for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}
E4B_DEV void tc_alloc(uint32_t* dst_smem, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
E4B_DEV void tc_dealloc(uint32_t tmem, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(cols) : "memory");
}

// Shared-memory matrix descriptor: K-major operand in the 128-byte swizzle
// layout (8-row x 128-byte atoms, 1024 bytes apart), version 1 (sm_100).
E4B_DEV uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor: f16 x f16 -> f32, both operands K-major, M = 128,
// N = n (a multiple of 16, <= 256), optionally negating A.
E4B_DEV uint32_t idesc_m128(uint32_t n, bool neg_a) {
  return (1u << 4) | ((n >> 3) << 17) | ((128u >> 4) << 24) | (neg_a ? (1u << 13) : 0u);
}

E4B_DEV uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

}  // namespace e4b
