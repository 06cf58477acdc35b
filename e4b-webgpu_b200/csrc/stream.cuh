// Building blocks of the streaming quantised GEMVs (sm_100a):
//   - mbarrier + cp.async.bulk (TMA bulk copy) helpers with bounded waits,
//   - warp-level tensor-core MMA (m16n8k16, f16 x f16 -> f32),
//   - the balanced persistent partition of work units over CTAs and the
//     deterministic split-K merge ("last arriving CTA sums the partials in
//     chunk order") used when a row tile is split across CTAs.
#pragma once

#include "common.cuh"

namespace e4b {

E4B_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

E4B_DEV void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
// Make barrier initialisation visible to the async (TMA) proxy.
E4B_DEV void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
E4B_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

E4B_DEV void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
E4B_DEV void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
E4B_DEV bool mbar_try_wait(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
E4B_DEV uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait: gives up after ~1 s, records E4B_ST_TIMEOUT and returns false.
E4B_DEV bool mbar_wait(uint64_t* b, uint32_t parity, uint32_t* status) {
  if (mbar_try_wait(b, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0;; i++) {
    if (mbar_try_wait(b, parity)) return true;
    if ((i & 255u) == 255u && globaltimer_ns() - t0 > 1000000000ull) {
      set_status(status, E4B_ST_TIMEOUT);
      return false;
    }
  }
}

// TMA bulk copy global -> this CTA's shared memory, completing on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
E4B_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// GPU-scope atomics with explicit ordering (split-K merge protocol): a
// contributor publishes its partial and then release-adds its coverage; the
// contributor whose add completes the tile acquires everyone's partials.
E4B_DEV unsigned long long atom_or_release(unsigned long long* a, unsigned long long v) {
  unsigned long long old;
  asm volatile("atom.release.gpu.global.or.b64 %0, [%1], %2;" : "=l"(old) : "l"(a), "l"(v) : "memory");
  return old;
}
E4B_DEV unsigned long long atom_or_acquire(unsigned long long* a, unsigned long long v) {
  unsigned long long old;
  asm volatile("atom.acquire.gpu.global.or.b64 %0, [%1], %2;" : "=l"(old) : "l"(a), "l"(v) : "memory");
  return old;
}
E4B_DEV uint32_t atom_add_acq_rel(uint32_t* a, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(a), "r"(v) : "memory");
  return old;
}

// Named barrier among the consumer warps (the producer warp does not take part).
E4B_DEV void consumer_sync(int nthreads) { asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory"); }

// D += A * B, m16n8k16, A row-major f16 (4 regs), B col-major f16 (2 regs), f32 accumulate.
E4B_DEV void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

E4B_DEV uint32_t hsub2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
E4B_DEV uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}
E4B_DEV uint32_t pack_h2(uint16_t lo, uint16_t hi) { return (uint32_t)lo | ((uint32_t)hi << 16); }

// ---- persistent partition: CTA i of G owns units [U*i/G, U*(i+1)/G)
E4B_DEV int64_t part_begin(int64_t U, int G, int i) { return U * (int64_t)i / G; }

// Is `u` the first unit of some CTA's range?
E4B_DEV bool is_range_start(int64_t u, int64_t U, int G) {
  if (u == 0) return true;
  const int64_t i = (u * G + U - 1) / U;  // smallest i with U*i/G >= u (up to rounding)
  for (int64_t j = i > 0 ? i - 1 : 0; j <= i + 1 && j < G; j++)
    if (part_begin(U, G, (int)j) == u) return true;
  return false;
}

}  // namespace e4b
