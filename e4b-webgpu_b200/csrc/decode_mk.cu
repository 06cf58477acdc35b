// Fused dense decode token: the whole per-token operator sequence of the dense
// (E4B) graph -- embedding, per-layer-embedding projection, and per layer
// q|k|v GEMV, head prep + split-KV attention, o GEMV, gate|up GEMV + GeGLU,
// down GEMV, PLE gate GEMV, PLE projection GEMV, with the residual / RMSNorm
// steps between them -- as ONE persistent cooperative kernel (one CTA per SM).
//
// Why: a decode token is ~250 dependent steps.  As separate kernels each step
// costs a launch-to-launch gap of several microseconds on B200 even inside a
// CUDA graph with programmatic dependent launch; here consecutive steps are
// separated by a grid barrier and the weight stream never stops.
//
// Weight stream.  Every GEMV's work is cut into quanta (32 rows x 8 q4_0 blocks,
// two 2304-byte pieces of the plan's tile-packed copy of the weights, one bulk
// copy each).  Each warp owns a fixed,
// host-precomputed schedule of quanta spanning ALL GEMV phases of the token and
// a private ring of mbarrier-tracked shared-memory stages.  A stage is refilled
// with the warp's next quantum as soon as it has been consumed, whatever phase
// that quantum belongs to, so weights of the following phases are in flight
// while a phase waits at a barrier or runs its prologue (weights never depend
// on activations).
//
// Partition.  A GEMV of T row tiles (32 rows; gate|up: 16 gate + 16 up rows)
// and qpr quanta per tile is split into T*s (tile, k-range) pieces, s = 1 or a
// small split factor; with s = 1 a CTA owns whole tiles (balanced), with s > 1
// CTA v owns k-range v % s of tile v / s.  A per-phase rotation places the
// pieces on the CTAs with the least cumulative weight traffic so far.  Inside a
// CTA quantum i goes to warp i % 8; warps flush one partial per (tile, warp)
// into shared memory and the CTA sums them in warp order.  Outputs are stored
// as [tile][s][32] partials and consumers add the s partials in order, so every
// result is deterministic.
//
// Residual stream.  Every CTA keeps the hidden state in shared memory and
// applies the same residual / RMSNorm updates in its phase prologues (same
// code, same data, same order: bit-identical copies), so no phase exists only
// to normalise a vector.  Phase descriptors are double-buffered in shared
// memory (the next one is fetched during the current phase).
//
// Arithmetic per operator follows the multi-kernel path (q40mv.wgsl /
// q40gu.wgsl / headprep.wgsl / attsplit.wgsl / attcomb.wgsl / rmsacc.wgsl /
// pleprep.wgsl semantics, see the kernels in q40_stream.cu, attn.cu, norm.cu,
// q6k.cu); only f32 summation orders differ.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <string.h>

#include <algorithm>

#include "q40_frag.cuh"

namespace e4b {
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();
}

namespace {
using namespace e4b;

constexpr int kWarps = 8;
constexpr int kThreads = 32 * kWarps;
constexpr int kStages = 4;
constexpr int kPrefetch = 6;          // quanta per warp prefetched into L2 beyond the ring
constexpr int kMaxPer = 8;            // hidden and PLE width <= 8 * kThreads

enum : int { PH_GEMV = 0, PH_ATTN = 1, PH_FINAL = 2 };
enum : int { XB_NONE = 0, XB_NORM = 1, XB_RAW = 2, XB_F32 = 3, XB_ATTN = 4, XB_PLE = 5 };
enum : int { XK_SMEM_F16 = 0, XK_STAGED_F16 = 1, XK_SMEM_F32 = 2 };
constexpr int kMaxRope = 4;           // distinct (theta, rotated pairs) layer kinds
enum : int { EPI_SLOTS = 0, EPI_GEGLU = 1 };

// A GEMV output as partials: buf[row / 32][s][row % 32]; the value of a row is
// the in-order sum of its s partials.  Every partial is published as one 64-bit
// word (epoch << 32 | f32 bits), epoch = token counter * 256 + tag, tag = the
// producing layer (255: the per-token PLE projection), so a consumer polls
// exactly the words it needs instead of waiting at a grid barrier.
struct SlotSrc {
  const uint64_t* buf;
  int s, tag;
};

struct MkGemv {
  int T, qpr, s, rot;   // tiles, quanta per tile, k-splits, CTA rotation
  int gu, ff;           // gate|up row layout: subtile 1 rows start at ff
  int xk;               // XK_*
  const uint32_t* xg;   // XK_STAGED_F16: global f16 x as (epoch16 << 16 | f16) words; the CTA's k-range is staged
  int xtag;             // producing layer of xg
  int epi, tag;         // tag: this layer (epoch of the outputs)
  uint64_t* out;        // EPI_SLOTS: [T][s][32] epoch words
  uint32_t* outh;       // EPI_GEGLU: [ff] (epoch16 << 16 | f16) words
};

struct MkAttn {
  SlotSrc qkv;
  const float* qn;
  const float* kn;
  uint16_t* kc;
  uint16_t* vc;
  float* part_o;        // [QH][nct][HD] chunk partials (unnormalised)
  float* part_ml;       // [QH][nct][2] chunk max and sum
  unsigned* cnt;        // [QH] finished chunks per head (zero at rest)
  uint32_t* out;        // [QH * HD] combined head outputs, (epoch16 << 16 | f16) words
  int cachemode, ring, window, slots, angles, keqv, nct, tag;
  int rope;             // index into the per-token RoPE table
  float theta, scale;
};

struct alignas(16) MkPhase {
  int kind;
  int kvpf;             // prefetch this layer's KV cache into L2 (q|k|v phase)
  int sync_after;       // grid barrier at the end of the phase (last phase of a layer)
  int res;              // residual first: h = (h + rms(t) * rw) * rmul, t from rt
  SlotSrc rt;
  const float* rw;
  float rmul;
  float* dump;          // h after the residual (CTA 0 writes; may be null)
  int xb;               // XB_*
  const float* xw;
  int layer;
  SlotSrc ple_gate;     // XB_PLE: the gate GEMV's output
  MkGemv g;
  MkAttn a;             // PH_ATTN, and the layer's attention for XB_ATTN
};
static_assert(sizeof(MkPhase) % 16 == 0, "phase descriptors are copied in 16-byte pieces");

// One entry of a warp's weight schedule: its quanta of one GEMV phase.
struct SchedEnt {
  const uint8_t* wt;    // the GEMV's tile-packed weights (2304-byte pieces of 16 rows x 256 k)
  int t0, k0, kq, nw, gu, ff, nq;
};

struct MkArgs {
  const MkPhase* ph;
  const SchedEnt* sched;
  const int2* sched_rng;  // [G * kWarps]: first entry, count
  int nph, G, H, QH, KVH, HD, PD, L, V, qdim;
  float eps, emb_mult, ple_mult, proj_scale;
  const uint8_t* emb;
  const uint8_t* ple_table;
  const float* ple_norm;
  SlotSrc pleproj;
  const float* out_norm;
  const uint32_t* params;
  uint32_t* status;
  unsigned* bar;        // [0] arrivals, [1] finished CTAs (zero at rest), [2] token counter, [3] abort flag
  float* xf;
  float* hout;
  unsigned long long* trace;   // optional [nph][8] globaltimer stamps (see e4b_dense_plan_trace)
  int xs_bytes, scr_bytes;
  int nrope;                   // RoPE kinds: theta and rotated pairs
  float rope_theta[kMaxRope];
  int rope_angles[kMaxRope];
};

// ------------------------------------------------------------------ CTA reductions
// Sum / max over the CTA: warp shuffles, one barrier, then every thread reads
// the 8 warp results as two 16-byte words (no serial chain); a trailing
// barrier frees `sh` (16-byte aligned, >= 8 floats) for the next reduction.
E4B_DEV float cta_sum(float v, float* sh) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  const float4 a = reinterpret_cast<const float4*>(sh)[0], b = reinterpret_cast<const float4*>(sh)[1];
  const float t = ((a.x + a.y) + (a.z + a.w)) + ((b.x + b.y) + (b.z + b.w));
  __syncthreads();
  return t;
}
E4B_DEV float cta_max(float v, float* sh) {
  v = warp_max(v);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  const float4 a = reinterpret_cast<const float4*>(sh)[0], b = reinterpret_cast<const float4*>(sh)[1];
  const float t = fmaxf(fmaxf(fmaxf(a.x, a.y), fmaxf(a.z, a.w)), fmaxf(fmaxf(b.x, b.y), fmaxf(b.z, b.w)));
  __syncthreads();
  return t;
}
static_assert(kWarps == 8, "cta_sum / cta_max read exactly 8 warp results");

// ------------------------------------------------------------------ partition
struct Work {
  int t0, nt, k0, kq, sp;   // tiles [t0, t0+nt), quanta [k0, k0+kq) of each, split index
};
__host__ __device__ inline Work cta_work(int T, int qpr, int s, int rot, int G, int c) {
  Work w{0, 0, 0, 0, 0};
  int v = c - rot;
  if (v < 0) v += G;
  if (s == 1) {
    w.t0 = (int)((long long)T * v / G);
    w.nt = (int)((long long)T * (v + 1) / G) - w.t0;
    w.k0 = 0;
    w.kq = qpr;
  } else if (v < T * s) {
    w.t0 = v / s;
    w.nt = 1;
    w.sp = v % s;
    w.k0 = qpr * w.sp / s;
    w.kq = qpr * (w.sp + 1) / s - w.k0;
  }
  return w;
}
__host__ __device__ inline int warp_items(const Work& w, int warp) {
  const int n = w.nt * w.kq;
  return n > warp ? (n - warp + kWarps - 1) / kWarps : 0;
}

E4B_DEV Work cta_work(const MkGemv& g, int G, int c) { return cta_work(g.T, g.qpr, g.s, g.rot, G, c); }

// ---- epoch-tagged publication (flag-in-data)
E4B_DEV void st_ll64(uint64_t* p, float v, uint32_t e) {
  const uint64_t w = ((uint64_t)e << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
E4B_DEV void st_ll32(uint32_t* p, uint16_t h, uint32_t e) {
  const uint32_t w = (e << 16) | h;
  asm volatile("st.relaxed.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(w) : "memory");
}
E4B_DEV uint64_t ld_ll64(const uint64_t* p) {
  uint64_t w;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
// Two epoch words (each loaded as one 64-bit element: value and epoch never tear).
E4B_DEV void ld_ll64x2(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
// Four 32-bit (epoch16 << 16 | f16) words.
E4B_DEV uint4 ld_ll32x4(const uint32_t* p) {
  uint4 w;
  asm volatile("ld.relaxed.gpu.global.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(w.x), "=r"(w.y), "=r"(w.z), "=r"(w.w)
               : "l"(p)
               : "memory");
  return w;
}
E4B_DEV uint32_t ep_of(uint64_t w) { return (uint32_t)(w >> 32); }
E4B_DEV float val_of(uint64_t w) { return __uint_as_float((uint32_t)w); }

// Bounded polling: gives up after ~1 s (status TIMEOUT) or when another CTA
// has given up (abort flag), returning false.
struct Spin {
  uint32_t it = 0;
  uint64_t t0 = 0;
};
E4B_DEV bool spin_more(Spin& sp, const MkArgs& A) {
  ++sp.it;
  if (sp.it == 8) sp.t0 = globaltimer_ns();
  if (sp.it > 8 && (sp.it & 7u) == 0) {
    unsigned ab;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(ab) : "l"(A.bar + 3) : "memory");
    if (ab) return false;
    if (globaltimer_ns() - sp.t0 > 1000000000ull) {
      set_status(A.status, E4B_ST_TIMEOUT);
      atomicExch(A.bar + 3, 1u);
      return false;
    }
  }
  return true;
}

// One output row (sum of its s partials), polled until published.
E4B_DEV float ll_row(const MkArgs& A, const SlotSrc& S, int row, uint32_t ebase, bool& dead) {
  const uint64_t* b = S.buf + (size_t)(row >> 5) * S.s * 32 + (row & 31);
  const uint32_t e = ebase + (uint32_t)S.tag;
  float v = 0.f;
  for (int k = 0; k < S.s; k++) {
    uint64_t w = ld_ll64(b + 32 * k);
    Spin sp;
    while (ep_of(w) != e && !dead) {
      if (!spin_more(sp, A)) dead = true;
      w = ld_ll64(b + 32 * k);
    }
    v = k == 0 ? val_of(w) : v + val_of(w);
  }
  return v;
}

// B fragments from shared memory: f16 x, or f32 x split into f16 hi + lo.
E4B_DEV void xget(const void* x, bool xf32, int blk, const XLane& X, uint4& hi, uint4& lo) {
  if (xf32) {
    xfrag_f32_any(reinterpret_cast<const float*>(x), blk, X, hi, lo);
  } else {
    hi = xfrag_f16_any(reinterpret_cast<const uint16_t*>(x), blk, X);
    lo = make_uint4(0, 0, 0, 0);
  }
}

// ---- memory-system helpers
// Weights are read exactly once per token: mark their L2 lines first to evict,
// so activations, norm vectors and the KV cache stay resident in L2.
E4B_DEV uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
E4B_DEV void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}
// Bulk L2 prefetch of [p, p + bytes): p 16-byte aligned, bytes a multiple of 16.
E4B_DEV void bulk_prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
E4B_DEV void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
E4B_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
E4B_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// Asynchronous copy of n floats (n % 4 == 0, both ends 16-byte aligned) by the CTA.
E4B_DEV void stage_floats(float* dst, const float* src, int n) {
  for (int i = threadIdx.x; i < n / 4; i += kThreads) cp_async16(dst + 4 * i, src + 4 * i);
}

E4B_DEV float rope_angle(uint32_t pos, int p, int HD, float theta) {
  const float ex = (-2.0f * (float)p) / (float)HD;
  return (float)pos * powf(theta, ex);
}

// Slot rule of the decode attention (kernels/attnf32.wgsl:28-53).
struct Rule {
  int cachemode, ring, window;
  uint32_t qp, len;
  E4B_DEV uint32_t nslots() const { return cachemode == 1 ? min(qp + 1, (uint32_t)ring) : len; }
  E4B_DEV bool valid(uint32_t t) const {
    if (cachemode == 1) {
      const uint32_t ps = qp - ((qp + (uint32_t)ring - t) % (uint32_t)ring);
      return ps <= qp && ps + (uint32_t)window > qp;
    }
    if (t >= len) return false;
    if (cachemode == 0 && window > 0 && len > (uint32_t)window) return t >= len - (uint32_t)window;
    return true;
  }
};
E4B_DEV Rule make_rule(const MkAttn& a, const uint32_t* params) {
  Rule r{a.cachemode, a.ring, a.window, 0u, 0u};
  r.qp = __ldcg(params + 0);
  r.len = a.cachemode == 2 ? __ldcg(params + 5) : __ldcg(params + 1);
  return r;
}
// Chunk length (a multiple of 32) so that QH x chunks fits the grid in one round.
__host__ __device__ inline void chunking(uint32_t nslots, int nct, int& CH, int& nch) {
  uint32_t ch = (nslots + (uint32_t)nct - 1) / (uint32_t)nct;
  ch = (ch + 31u) & ~31u;
  if (ch < 32u) ch = 32u;
  CH = (int)ch;
  nch = (int)((nslots + ch - 1) / ch);
}

// ------------------------------------------------------------------ grid barrier
// Arrivals only ever increase within a launch: barrier b completes when all G
// CTAs have arrived b times.  Bounded: gives up after ~1 s (status TIMEOUT).
E4B_DEV bool grid_sync(unsigned* ctr, unsigned target, uint32_t* status, volatile int* flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
    unsigned v = 0;
    uint64_t t0 = 0;
    int ok = 1;
    for (uint32_t i = 0;; i++) {
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
      if (v >= target) break;
      if (i == 32) t0 = globaltimer_ns();
      if (i > 32 && (i & 63u) == 0 && globaltimer_ns() - t0 > 1000000000ull) {
        set_status(status, E4B_ST_TIMEOUT);
        ok = 0;
        break;
      }
    }
    *flag = ok;
  }
  __syncthreads();
  return *flag != 0;
}

// ------------------------------------------------------------------ weight producer
// The warp's position in its schedule; the entry after the current one is
// loaded ahead so a phase change costs no dependent global load.
struct Prod {
  SchedEnt e, nx;
  int idx, end, j;
  int tl, kk;           // local tile and quantum of item j (warp + 8 j = tl * kq + kk)
};

E4B_DEV void prod_seek(Prod& u, int warp) {
  u.j = 0;
  u.tl = warp / u.e.kq;
  u.kk = warp - u.tl * u.e.kq;
}

E4B_DEV void prod_init(const MkArgs& A, Prod& u, int c, int warp) {
  const int2 r = A.sched_rng[c * kWarps + warp];
  u.idx = r.x;
  u.end = r.x + r.y;
  if (u.idx < u.end) {
    u.e = A.sched[u.idx];
    prod_seek(u, warp);
  }
  if (u.idx + 1 < u.end) u.nx = A.sched[u.idx + 1];
}

// The cursor's quantum: its two 16-row pieces in the packed copy (gate|up:
// gate rows 16 tile and up rows ff + 16 tile; else rows 32 tile and 32 tile + 16).
E4B_DEV void prod_src(const Prod& u, const uint8_t*& a, const uint8_t*& b) {
  const int tile = u.e.t0 + u.tl, kq = u.e.k0 + u.kk;
  const int r0 = u.e.gu ? tile : 2 * tile, r1 = u.e.gu ? u.e.ff / 16 + tile : 2 * tile + 1;
  a = u.e.wt + ((size_t)r0 * u.e.nq + kq) * kPkSub;
  b = u.e.wt + ((size_t)r1 * u.e.nq + kq) * kPkSub;
}
E4B_DEV void prod_advance(const MkArgs& A, Prod& u, int warp) {
  u.kk += kWarps;
  while (u.kk >= u.e.kq) {
    u.kk -= u.e.kq;
    u.tl++;
  }
  if (++u.j == u.e.nw) {
    if (++u.idx < u.end) {
      u.e = u.nx;
      prod_seek(u, warp);
      if (u.idx + 1 < u.end) u.nx = A.sched[u.idx + 1];
    }
  }
}
// Issue the cursor's quantum into `stage` (lane 0), then advance the cursor.
E4B_DEV void prod_issue(const MkArgs& A, Prod& u, uint8_t* stage, uint64_t* bar, int warp, int lane, uint64_t pol) {
  if (lane == 0) {
    const uint8_t *a, *b;
    prod_src(u, a, b);
    mbar_expect_tx(bar, 2u * kPkSub);
    bulk_g2s_hint(stage, a, kPkSub, bar, pol);
    bulk_g2s_hint(stage + kPkSub, b, kPkSub, bar, pol);
  }
  prod_advance(A, u, warp);
}
// L2 prefetch of the prefetch cursor's quantum, then advance it.
E4B_DEV void prod_prefetch(const MkArgs& A, Prod& u, int warp, int lane) {
  if (lane == 0) {
    const uint8_t *a, *b;
    prod_src(u, a, b);
    bulk_prefetch_l2(a, kPkSub);
    bulk_prefetch_l2(b, kPkSub);
  }
  prod_advance(A, u, warp);
}

struct Ring {
  uint8_t* base;        // this warp's stages
  uint64_t* full;       // this warp's barriers
  uint32_t cnt;         // quanta consumed
  uint32_t issued;      // quanta issued
  bool ok;
  unsigned long long wait_ns;   // time spent waiting for weights (traced runs)
};

// One quantum (8 blocks x 32 rows) of a packed stage (pieces: subtile 0 then
// 1): quantum_mma's A registers, scales and MMAs, from one 16-byte load per
// row and 4 blocks and one 4-byte scale load per row; the f32-activation
// (hi + lo) MMAs chosen at run time, one copy of the code for both kinds.
E4B_DEV void quantum_mma_pk(const uint8_t* st, const uint4 xh, const uint4 xl, int g, int t, float (&acc)[4],
                            bool xf32) {
  float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};   // subtile 0: low / high k-half
  float c2[4] = {0.f, 0.f, 0.f, 0.f}, c3[4] = {0.f, 0.f, 0.f, 0.f};   // subtile 1
#pragma unroll
  for (int kh = 0; kh < 2; kh++) {
    const uint8_t* nb = st + 256 + ((kh * 16 + g) * 4 + t) * 16;
    const uint4 N0 = *reinterpret_cast<const uint4*>(nb);                  // subtile 0, row g
    const uint4 N1 = *reinterpret_cast<const uint4*>(nb + 8 * 64);         // subtile 0, row g + 8
    const uint4 N2 = *reinterpret_cast<const uint4*>(nb + kPkSub);        // subtile 1, row g
    const uint4 N3 = *reinterpret_cast<const uint4*>(nb + kPkSub + 8 * 64);
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int k = 4 * kh + j;
      uint32_t A[16];
      dq_row(u32w(N0, j), A[0], A[1], A[2], A[3]);
      dq_row(u32w(N1, j), A[4], A[5], A[6], A[7]);
      dq_row(u32w(N2, j), A[8], A[9], A[10], A[11]);
      dq_row(u32w(N3, j), A[12], A[13], A[14], A[15]);
      const bool mine = g == k;
      const uint32_t b0 = mine ? xh.x : 0u, b1 = mine ? xh.y : 0u, b2 = mine ? xh.z : 0u, b3 = mine ? xh.w : 0u;
      mma16816(c0, A[0], A[4], A[1], A[5], b0, b1);
      mma16816(c2, A[8], A[12], A[9], A[13], b0, b1);
      mma16816(c1, A[2], A[6], A[3], A[7], b2, b3);
      mma16816(c3, A[10], A[14], A[11], A[15], b2, b3);
      if (xf32) {
        const uint32_t l0 = mine ? xl.x : 0u, l1 = mine ? xl.y : 0u, l2 = mine ? xl.z : 0u, l3 = mine ? xl.w : 0u;
        mma16816(c0, A[0], A[4], A[1], A[5], l0, l1);
        mma16816(c2, A[8], A[12], A[9], A[13], l0, l1);
        mma16816(c1, A[2], A[6], A[3], A[7], l2, l3);
        mma16816(c3, A[10], A[14], A[11], A[15], l2, l3);
      }
    }
  }
  // C cols 2t, 2t+1 = blocks 2t, 2t+1: word t of each row's 8 scales
  float d[8];
  const int so[4] = {16 * g, 16 * (g + 8), kPkSub + 16 * g, kPkSub + 16 * (g + 8)};
#pragma unroll
  for (int r = 0; r < 4; r++) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(st + so[r] + 4 * t);
    d[2 * r] = h2f((uint16_t)(w & 0xFFFFu));
    d[2 * r + 1] = h2f((uint16_t)(w >> 16));
  }
  acc[0] = fmaf(d[0], c0[0] + c1[0], fmaf(d[1], c0[1] + c1[1], acc[0]));
  acc[1] = fmaf(d[2], c0[2] + c1[2], fmaf(d[3], c0[3] + c1[3], acc[1]));
  acc[2] = fmaf(d[4], c2[0] + c3[0], fmaf(d[5], c2[1] + c3[1], acc[2]));
  acc[3] = fmaf(d[6], c2[2] + c3[2], fmaf(d[7], c2[3] + c3[3], acc[3]));
}

// ------------------------------------------------------------------ GEMV phase
// x: activations in shared memory indexed by absolute block (8 k + g); XF32:
// f32 x split into f16 hi + lo (twice the MMAs; one GEMV per token uses it).
template <bool XF32>
E4B_DEV void gemv_phase(const MkArgs& A, const Work& W, int warp, int lane, Ring& R, Prod& u, Prod& pf,
                        uint64_t pol, const void* x, float* P) {
  constexpr bool xf32 = XF32;
  const int nw = warp_items(W, warp);
  if (nw == 0) return;
  const int gg = lane >> 2, t = lane & 3;
  const XLane X = xlane(gg, t);
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  int tl = warp / W.kq, kk = warp - tl * W.kq;      // item j: warp + 8 j = tl * kq + kk
  uint4 xh, xl;
  xget(x, xf32, (W.k0 + kk) * 8 + gg, X, xh, xl);
  for (int j = 0; j < nw; j++) {
    int ntl = tl, nkk = kk + kWarps;
    while (nkk >= W.kq) {
      nkk -= W.kq;
      ntl++;
    }
    uint4 nh = make_uint4(0, 0, 0, 0), nl = make_uint4(0, 0, 0, 0);
    if (j + 1 < nw) xget(x, xf32, (W.k0 + nkk) * 8 + gg, X, nh, nl);
    const uint32_t s = R.cnt % kStages;
    const bool tw = A.trace && blockIdx.x == 0 && warp == 0 && lane == 0;
    const unsigned long long tw0 = tw ? globaltimer_ns() : 0ull;
    if (R.ok) R.ok = mbar_wait(&R.full[s], (R.cnt / kStages) & 1u, A.status);
    if (tw) R.wait_ns += globaltimer_ns() - tw0;
    if (R.ok) quantum_mma_pk(R.base + s * kQuantumBytes, xh, xl, gg, t, acc, xf32);
    R.cnt++;
    // every lane's shared-memory reads of the stage are complete (their values
    // fed the MMAs) before the TMA unit overwrites it
    __syncwarp();
    if (R.ok && u.idx < u.end) {
      prod_issue(A, u, R.base + s * kQuantumBytes, &R.full[s], warp, lane, pol);
      R.issued++;
      if (pf.idx < pf.end) prod_prefetch(A, pf, warp, lane);
    }
    xh = nh;
    xl = nl;
    if (j + 1 == nw || ntl != tl) {
      float v[4];
#pragma unroll
      for (int r = 0; r < 4; r++) {
        v[r] = acc[r];
        v[r] += __shfl_xor_sync(0xffffffffu, v[r], 1);
        v[r] += __shfl_xor_sync(0xffffffffu, v[r], 2);
        acc[r] = 0.f;
      }
      if (t == 0) {
        float* pp = P + ((size_t)tl * kWarps + warp) * 32;
        pp[gg] = v[0];
        pp[8 + gg] = v[1];
        pp[16 + gg] = v[2];
        pp[24 + gg] = v[3];
      }
    }
    tl = ntl;
    kk = nkk;
  }
}

// Warps that flushed a partial for local tile tl (its quanta are the CTA-local
// indices [tl*kq, (tl+1)*kq), quantum i belongs to warp i % kWarps).
E4B_DEV uint32_t warps_of_tile(const Work& W, int tl) {
  if (W.kq >= kWarps) return (1u << kWarps) - 1u;
  uint32_t m = 0;
  for (int i = tl * W.kq; i < (tl + 1) * W.kq; i++) m |= 1u << (i % kWarps);
  return m;
}

// CTA-wide: sum the warps' partials per tile (in warp order) and publish.
E4B_DEV void gemv_epilogue(const MkGemv& g, const Work& W, const float* P, uint32_t ebase) {
  const uint32_t ep = ebase + (uint32_t)g.tag;
  if (g.epi == EPI_GEGLU) {
    for (int idx = threadIdx.x; idx < W.nt * 16; idx += kThreads) {
      const int tl = idx >> 4, r = idx & 15;
      const float* pp = P + (size_t)tl * kWarps * 32;
      const uint32_t wm = warps_of_tile(W, tl);
      float gv = 0.f, uv = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; w++) {
        if (!(wm >> w & 1u)) continue;
        gv += pp[w * 32 + r];
        uv += pp[w * 32 + 16 + r];
      }
      const int o = 16 * (W.t0 + tl) + r;
      if (o < g.ff) st_ll32(g.outh + o, f2h(gelu_tanh(gv) * uv), ep);
    }
  } else {
    for (int idx = threadIdx.x; idx < W.nt * 32; idx += kThreads) {
      const int tl = idx >> 5, r = idx & 31;
      const float* pp = P + (size_t)tl * kWarps * 32;
      const uint32_t wm = warps_of_tile(W, tl);
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; w++)
        if (wm >> w & 1u) v += pp[w * 32 + r];
      st_ll64(g.out + ((size_t)(W.t0 + tl) * g.s + W.sp) * 32 + r, v, ep);
    }
  }
}

// ------------------------------------------------------------------ prologues
// v[k] = row tid + 256 k of a GEMV output (sum of its s <= 2 partials), for the
// rows below n; every load is issued before any is checked, stale words
// (older epoch) are re-read until published.
E4B_DEV void slot_rows(const MkArgs& A, const SlotSrc& S, int n, uint32_t ebase, float (&v)[kMaxPer], bool& dead) {
  uint64_t a[kMaxPer], b[kMaxPer];
  const uint32_t e = ebase + (uint32_t)S.tag;
  const bool two = S.s > 1;
#pragma unroll
  for (int k = 0; k < kMaxPer; k++) {
    const int i = threadIdx.x + k * kThreads;
    a[k] = b[k] = (uint64_t)e << 32;
    if (i < n) {
      const uint64_t* p = S.buf + (size_t)(i >> 5) * S.s * 32 + (i & 31);
      a[k] = ld_ll64(p);
      if (two) b[k] = ld_ll64(p + 32);
    }
  }
  Spin sp;
  for (;;) {
    bool ok = true;
#pragma unroll
    for (int k = 0; k < kMaxPer; k++) ok = ok && ep_of(a[k]) == e && ep_of(b[k]) == e;
    if (ok || dead) break;
    if (!spin_more(sp, A)) {
      dead = true;
      break;
    }
#pragma unroll
    for (int k = 0; k < kMaxPer; k++) {
      const int i = threadIdx.x + k * kThreads;
      if (i >= n) continue;
      const uint64_t* p = S.buf + (size_t)(i >> 5) * S.s * 32 + (i & 31);
      if (ep_of(a[k]) != e) a[k] = ld_ll64(p);
      if (two && ep_of(b[k]) != e) b[k] = ld_ll64(p + 32);
    }
  }
#pragma unroll
  for (int k = 0; k < kMaxPer; k++) v[k] = two ? val_of(a[k]) + val_of(b[k]) : val_of(a[k]);
}

// h = (h + t * rms(t) * w) * mul (kernels/rmsacc.wgsl).
E4B_DEV void residual(const MkArgs& A, const MkPhase& P, float* hs, const float* rw, float* red, uint32_t ebase,
                      bool& dead) {
  float tv[kMaxPer];
  slot_rows(A, P.rt, A.H, ebase, tv, dead);
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < kMaxPer; k++)
    if (threadIdx.x + k * kThreads < A.H) s = fmaf(tv[k], tv[k], s);
  const float inv = rms_scale(cta_sum(s, red), A.H, A.eps);
  const bool dump = P.dump && blockIdx.x == 0;
#pragma unroll
  for (int k = 0; k < kMaxPer; k++) {
    const int i = threadIdx.x + k * kThreads;
    if (i < A.H) {
      const float h = (hs[i] + tv[k] * inv * rw[i]) * P.rmul;
      hs[i] = h;
      if (dump) P.dump[i] = h;
    }
  }
}

// x = f16(h * rms(h) * w)  or  f16(h).
E4B_DEV void build_x_norm(const MkArgs& A, const float* hs, const float* w, uint16_t* xs, float* red, int norm) {
  float inv = 1.f;
  if (norm) {
    float s = 0.f;
    for (int i = threadIdx.x; i < A.H; i += kThreads) s = fmaf(hs[i], hs[i], s);
    inv = rms_scale(cta_sum(s, red), A.H, A.eps);
  }
  for (int i = threadIdx.x; i < A.H; i += kThreads) {
    float v = hs[i];
    if (norm) v = v * inv * w[i];
    xs[i] = f2h(v);
  }
}

// The o-GEMV input: the combined attention outputs of the columns the CTA's
// quanta read, polled until the attention phase published them.
E4B_DEV void build_x_attn(const MkArgs& A, const MkPhase& P, const Work& W, uint16_t* xs, uint32_t ebase,
                          bool& dead) {
  if (W.nt == 0) return;
  const uint32_t e16 = (ebase + (uint32_t)P.a.tag) & 0xFFFFu;
  const uint32_t* src = P.a.out + 256 * W.k0;
  for (int i = threadIdx.x; i < W.kq * 64; i += kThreads) {
    if (256 * W.k0 + 4 * i >= A.qdim) break;
    uint4 w = ld_ll32x4(src + 4 * i);
    Spin sp;
    while (((w.x >> 16) != e16 || (w.y >> 16) != e16 || (w.z >> 16) != e16 || (w.w >> 16) != e16) && !dead) {
      if (!spin_more(sp, A)) dead = true;
      w = ld_ll32x4(src + 4 * i);
    }
    reinterpret_cast<uint2*>(xs + 256 * W.k0)[i] = make_uint2(__byte_perm(w.x, w.y, 0x5410), __byte_perm(w.z, w.w, 0x5410));
  }
}

// PLE input of layer l (kernels/pleprep.wgsl) times GeGLU of the gate GEMV:
// x[o] = f16(gelu(gate[o]) * ((p_o rms(p) nw[o] + table[tok][l PD + o] sqrt(PD)) / sqrt 2)), p = Wp h / sqrt(H).
E4B_DEV void build_x_ple(const MkArgs& A, const MkPhase& P, const float* nw, uint16_t* xs, float* red, uint32_t ebase,
                         bool& dead) {
  float pv[kMaxPer], gv[kMaxPer], idv[kMaxPer];
  const int base = P.layer * A.PD;
  const uint32_t row = __ldcg(A.params + 2);
  const bool tok_ok = row < (uint32_t)A.V;
  const uint8_t* r = A.ple_table + (size_t)(tok_ok ? row : 0) * ((size_t)A.L * A.PD / 256) * 210;
  // issue every load first: projection and gate partials, table weights
  const SlotSrc pp{A.pleproj.buf + (size_t)(base >> 5) * A.pleproj.s * 32, A.pleproj.s, A.pleproj.tag};
  slot_rows(A, pp, A.PD, ebase, pv, dead);
  slot_rows(A, P.ple_gate, A.PD, ebase, gv, dead);
#pragma unroll
  for (int k = 0; k < kMaxPer; k++) {
    const int o = threadIdx.x + k * kThreads;
    idv[k] = 0.f;
    if (o < A.PD && tok_ok) {
      const int gi = base + o;
      idv[k] = q6k_elem(r + (size_t)(gi >> 8) * 210, gi & 255);
    }
  }
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < kMaxPer; k++) {
    pv[k] *= A.proj_scale;
    if (threadIdx.x + k * kThreads < A.PD) s = fmaf(pv[k], pv[k], s);
  }
  const float inv = rms_scale(cta_sum(s, red), A.PD, A.eps);
#pragma unroll
  for (int k = 0; k < kMaxPer; k++) {
    const int o = threadIdx.x + k * kThreads;
    if (o < A.PD) {
      const float ple = (pv[k] * inv * nw[o] + idv[k] * A.ple_mult) * 0.70710678118654752f;
      xs[o] = f2h(gelu_tanh(gv[k]) * ple);
    }
  }
}

// ------------------------------------------------------------------ attention phase
// Items (q head, chunk of slots): q RMSNorm + RoPE, the current token's k / v
// (RMSNorm, RoPE, f16 cache write by the group's first head), scores, local
// softmax and p.V over the chunk (kernels/headprep.wgsl + attsplit.wgsl).
// Scores: 4 threads per slot, 16-byte K loads; p.V: each thread 8 dims of a
// slot subset, 16-byte V loads, then a shared-memory reduction over subsets.
E4B_DEV void attention_phase(const MkArgs& A, const MkAttn& a, int c, const float* qn, const float* kn,
                             const float* rope_tab, float* scr, float* red, unsigned long long* tr, uint32_t ebase,
                             bool& dead) {
  const uint32_t ep = ebase + (uint32_t)a.tag;
  const Rule rule = make_rule(a, A.params);
  const uint32_t nslots = rule.nslots();
  int CH, nch;
  chunking(nslots, a.nct, CH, nch);
  const uint32_t qp = rule.qp;
  const uint32_t cur = a.cachemode == 1 ? qp % (uint32_t)a.ring : (a.cachemode == 2 ? __ldcg(A.params + 4) : qp);
  const bool cur_ok = cur < (uint32_t)a.slots;
  if (!cur_ok && c == 0 && threadIdx.x == 0) set_status(A.status, E4B_ST_BADINDEX);
  const int HD = A.HD, half = HD / 2, grp = A.QH / A.KVH;
  const int tid = threadIdx.x;
  // qs: q in 4 quarters of HD/4 floats with 4 floats of padding between them,
  // so the 4 threads of a slot read conflict-free 16-byte words
  const int qpad = HD / 4 + 4;
  float* qs = scr;                            // [4 * qpad]
  float* kcur = scr + 4 * qpad;
  float* vcur = kcur + HD;
  float* red2 = vcur + HD;                    // [kThreads * 8]
  float* sc = red2 + kThreads * 8;            // [CH]
  auto qix = [&](int d) { return (d / (HD / 4)) * qpad + d % (HD / 4); };
  const int items = A.QH * nch;
  const int part = tid & 3, q4 = HD / 4, nv = q4 / 8;          // scores: 4 threads per slot
  const int ndg = HD / 8, nsg = kThreads / ndg;                // p.V: dim group of 8 x slot subset
  const int dg = tid % ndg, sg = tid / ndg;
  for (int item = c; item < items; item += A.G) {
    const int h = item / nch, ch = item - h * nch, kvh = h / grp;
    const uint32_t t0 = (uint32_t)ch * CH;
    const uint32_t hi = min(t0 + (uint32_t)CH, nslots);
    const bool has_cur = cur_ok && cur >= t0 && cur < t0 + (uint32_t)CH && cur < nslots;
    const int krow = A.QH * HD + kvh * HD;
    const int vrow = a.keqv ? krow : A.QH * HD + A.KVH * HD + kvh * HD;
    // K and V of the chunk's first slots do not depend on this token's q: load
    // them first, so their latency overlaps the q preparation
    uint4 kw[8], vw[4];
    const uint32_t tk = t0 + (uint32_t)(tid >> 2);
    const bool kpre = nv <= 8 && (tid >> 2) < CH && tk < hi && !(has_cur && tk == cur);
    if (kpre) {
      const uint4* kr = reinterpret_cast<const uint4*>(a.kc + ((size_t)tk * A.KVH + kvh) * HD + part * q4);
#pragma unroll
      for (int u = 0; u < 8; u++)
        if (u < nv) kw[u] = kr[u];
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const uint32_t ts = t0 + (uint32_t)(sg + u * nsg);
      vw[u] = make_uint4(0, 0, 0, 0);
      if (ts < hi && !(has_cur && ts == cur))
        vw[u] = *reinterpret_cast<const uint4*>(a.vc + ((size_t)ts * A.KVH + kvh) * HD + 8 * dg);
    }
    // raw q (and the current k / v)
    float sq = 0.f, sk = 0.f, sv = 0.f;
    for (int d = tid; d < HD; d += kThreads) {
      const float qv = ll_row(A, a.qkv, h * HD + d, ebase, dead);
      qs[qix(d)] = qv;
      sq = fmaf(qv, qv, sq);
      if (has_cur) {
        const float kv = ll_row(A, a.qkv, krow + d, ebase, dead), vv = ll_row(A, a.qkv, vrow + d, ebase, dead);
        kcur[d] = kv;
        vcur[d] = vv;
        sk = fmaf(kv, kv, sk);
        sv = fmaf(vv, vv, sv);
      }
    }
    const float qinv = rms_scale(cta_sum(sq, red), HD, A.eps);
    float kinv = 0.f, vinv = 0.f;
    if (has_cur) {
      kinv = rms_scale(cta_sum(sk, red), HD, A.eps);
      vinv = rms_scale(cta_sum(sv, red), HD, A.eps);
    }
    const bool writer = has_cur && (h % grp) == 0;
    uint16_t* kcw = a.kc + ((size_t)cur * A.KVH + kvh) * HD;
    uint16_t* vcw = a.vc + ((size_t)cur * A.KVH + kvh) * HD;
    for (int p = tid; p < half; p += kThreads) {
      const bool rot = p < a.angles;
      const float cs = rot ? rope_tab[(2 * a.rope) * half + p] : 1.f;
      const float sn = rot ? rope_tab[(2 * a.rope + 1) * half + p] : 0.f;
      const int i0 = qix(p), i1 = qix(p + half);
      const float x0 = qs[i0] * qinv * qn[p];
      const float x1 = qs[i1] * qinv * qn[p + half];
      qs[i0] = rot ? x0 * cs - x1 * sn : x0;
      qs[i1] = rot ? x0 * sn + x1 * cs : x1;
      if (has_cur) {
        const float y0 = kcur[p] * kinv * kn[p];
        const float y1 = kcur[p + half] * kinv * kn[p + half];
        const uint16_t k0 = f2h(rot ? y0 * cs - y1 * sn : y0), k1 = f2h(rot ? y0 * sn + y1 * cs : y1);
        kcur[p] = h2f(k0);
        kcur[p + half] = h2f(k1);
        if (writer) {
          kcw[p] = k0;
          kcw[p + half] = k1;
        }
      }
    }
    if (has_cur) {
      for (int d = tid; d < HD; d += kThreads) {
        const uint16_t v16 = f2h(vcur[d] * vinv);
        vcur[d] = h2f(v16);
        if (writer) vcw[d] = v16;
      }
    }
    __syncthreads();
    if (tr && item == c) tr[2] = globaltimer_ns();
    // scores: 4 threads per slot, each a quarter of the dims in 16-byte vectors
    for (int sb = 0; sb < CH; sb += kThreads / 4) {
      const int tt = sb + (tid >> 2);
      const uint32_t ts = t0 + (uint32_t)tt;
      const bool ok = tt < CH && ts < nslots && rule.valid(ts);
      float acc = 0.f;
      if (ok) {
        if (has_cur && ts == cur) {
          for (int d = 0; d < q4; d++) acc = fmaf(qs[part * qpad + d], kcur[part * q4 + d], acc);
        } else {
          const uint4* kr = reinterpret_cast<const uint4*>(a.kc + ((size_t)ts * A.KVH + kvh) * HD + part * q4);
          for (int v0 = 0; v0 < nv; v0 += 8) {
            uint4 kk[8];
            const bool pre = sb == 0 && v0 == 0 && kpre;
#pragma unroll
            for (int u = 0; u < 8; u++)
              if (v0 + u < nv) kk[u] = pre ? kw[u] : kr[v0 + u];
#pragma unroll
            for (int u = 0; u < 8; u++) {
              if (v0 + u >= nv) break;
              const float4* qd = reinterpret_cast<const float4*>(qs + part * qpad + 8 * (v0 + u));
              const float4 qa = qd[0], qb = qd[1];
              const __half2* k2 = reinterpret_cast<const __half2*>(&kk[u]);
              const float2 k0 = __half22float2(k2[0]), k1 = __half22float2(k2[1]);
              const float2 k2f = __half22float2(k2[2]), k3 = __half22float2(k2[3]);
              acc = fmaf(qa.x, k0.x, acc);
              acc = fmaf(qa.y, k0.y, acc);
              acc = fmaf(qa.z, k1.x, acc);
              acc = fmaf(qa.w, k1.y, acc);
              acc = fmaf(qb.x, k2f.x, acc);
              acc = fmaf(qb.y, k2f.y, acc);
              acc = fmaf(qb.z, k3.x, acc);
              acc = fmaf(qb.w, k3.y, acc);
            }
          }
        }
      }
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      if (part == 0 && tt < CH) sc[tt] = ok ? acc * a.scale : -INFINITY;
    }
    __syncthreads();
    float m = -INFINITY;
    for (int tt = tid; tt < CH; tt += kThreads) m = fmaxf(m, sc[tt]);
    m = cta_max(m, red);
    float l = 0.f;
    for (int tt = tid; tt < CH; tt += kThreads) {
      const float sv2 = sc[tt];
      const float p = sv2 == -INFINITY ? 0.f : expf(sv2 - m);
      sc[tt] = p;
      l += p;
    }
    l = cta_sum(l, red);   // also orders the p writes before the reads below
    if (tr && item == c) tr[3] = globaltimer_ns();
    // p.V: four slots per step, V vectors loaded before use (the first four early)
    {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (uint32_t ts0 = t0 + (uint32_t)sg; ts0 < hi; ts0 += 4u * (uint32_t)nsg) {
        float pu[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
          const uint32_t ts = ts0 + (uint32_t)(u * nsg);
          pu[u] = ts < hi ? sc[ts - t0] : 0.f;
          if (ts0 != t0 + (uint32_t)sg) {
            vw[u] = make_uint4(0, 0, 0, 0);
            if (pu[u] != 0.f && !(has_cur && ts == cur))
              vw[u] = *reinterpret_cast<const uint4*>(a.vc + ((size_t)ts * A.KVH + kvh) * HD + 8 * dg);
          }
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
          const uint32_t ts = ts0 + (uint32_t)(u * nsg);
          const float p = pu[u];
          if (p == 0.f) continue;
          if (has_cur && ts == cur) {
#pragma unroll
            for (int e = 0; e < 8; e++) acc[e] = fmaf(p, vcur[8 * dg + e], acc[e]);
          } else {
            const __half2* v2 = reinterpret_cast<const __half2*>(&vw[u]);
#pragma unroll
            for (int e = 0; e < 4; e++) {
              const float2 vf = __half22float2(v2[e]);
              acc[2 * e] = fmaf(p, vf.x, acc[2 * e]);
              acc[2 * e + 1] = fmaf(p, vf.y, acc[2 * e + 1]);
            }
          }
        }
      }
#pragma unroll
      for (int e = 0; e < 8; e++) red2[sg * HD + 8 * dg + e] = acc[e];
      __syncthreads();
      const size_t pi = (size_t)h * a.nct + ch;
      for (int d = tid; d < HD; d += kThreads) {
        float o = 0.f;
        for (int k = 0; k < nsg; k++) o += red2[k * HD + d];
        a.part_o[pi * HD + d] = o;
      }
      if (tid == 0) {
        a.part_ml[2 * pi] = l > 0.f ? m : -INFINITY;
        a.part_ml[2 * pi + 1] = l;
      }
    }
    // the head's last finishing chunk merges all its chunks (kernels/attcomb.wgsl):
    // out[d] = sum_c o_c[d] e^(m_c - M) / sum_c l_c e^(m_c - M)
    __syncthreads();
    volatile int* lastp = reinterpret_cast<volatile int*>(red + 16);
    if (tid == 0) {
      unsigned old;
      asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(a.cnt + h) : "memory");
      *lastp = old == (unsigned)nch - 1u;
    }
    __syncthreads();
    if (*lastp) {
      float* ew = red2;                       // [nch] weights e^(m_c - M), then den at [nch]
      if (tid < nch) {
        ew[tid] = __ldcg(a.part_ml + 2 * ((size_t)h * a.nct + tid));
        ew[64 + tid] = __ldcg(a.part_ml + 2 * ((size_t)h * a.nct + tid) + 1);
      }
      __syncthreads();
      if (tid == 0) {
        float M = -INFINITY;
        for (int k = 0; k < nch; k++)
          if (ew[64 + k] > 0.f) M = fmaxf(M, ew[k]);
        float den = 0.f;
        for (int k = 0; k < nch; k++) {
          const float lk = ew[64 + k];
          const float wk = lk > 0.f ? expf(ew[k] - M) : 0.f;
          den += lk > 0.f ? lk * wk : 0.f;
          ew[k] = wk;
        }
        ew[128] = den;
        a.cnt[h] = 0u;                        // next use is after the layer's grid barrier
      }
      __syncthreads();
      const float den = ew[128];
      for (int d = tid; d < HD; d += kThreads) {
        const float* po = a.part_o + (size_t)h * a.nct * HD + d;
        float acc = 0.f;
        for (int k = 0; k < nch; k++) acc = fmaf(__ldcg(po + (size_t)k * HD), ew[k], acc);
        st_ll32(a.out + (size_t)h * HD + d, f2h(den > 0.f ? acc / den : 0.f), ep);
      }
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------ the kernel
// Stage phase P's norm vectors into wbuf ([0,H) residual weight, [H,2H) input
// norm / PLE norm / output norm, [2H,2H+HD) q norm, [2H+HD,2H+2HD) k norm).
E4B_DEV void stage_vectors(const MkArgs& A, const MkPhase& P, float* wbuf) {
  if (P.kind == PH_ATTN) {
    stage_floats(wbuf + 2 * A.H, P.a.qn, A.HD);
    stage_floats(wbuf + 2 * A.H + A.HD, P.a.kn, A.HD);
  } else {
    if (P.res) stage_floats(wbuf, P.rw, A.H);
    if (P.xw) stage_floats(wbuf + A.H, P.xw, P.xb == XB_PLE ? A.PD : A.H);
  }
  cp_async_commit();
}

// This CTA's share of layer l's attended K and V bytes, into L2.
E4B_DEV void prefetch_kv(const MkArgs& A, const MkAttn& a, int c) {
  const Rule rule = make_rule(a, A.params);
  const uint32_t total = rule.nslots() * (uint32_t)(A.KVH * A.HD * 2);
  const uint32_t chunk = ((total + (uint32_t)A.G - 1) / (uint32_t)A.G + 15u) & ~15u;
  const uint32_t off = (uint32_t)c * chunk;
  if (off >= total) return;
  const uint32_t len = min(chunk, total - off);
  bulk_prefetch_l2(reinterpret_cast<const uint8_t*>(a.kc) + off, len);
  bulk_prefetch_l2(reinterpret_cast<const uint8_t*>(a.vc) + off, len);
}

__global__ void __launch_bounds__(kThreads, 1) k_decode_dense(const MkArgs A) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x;
  uint8_t* ring = smem;
  float* hs = reinterpret_cast<float*>(smem + (size_t)kWarps * kStages * kQuantumBytes);
  uint8_t* xs = reinterpret_cast<uint8_t*>(hs + A.H);
  float* scr = reinterpret_cast<float*>(xs + A.xs_bytes);
  float* wbuf = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(scr) + A.scr_bytes);
  MkPhase* phs = reinterpret_cast<MkPhase*>(wbuf + 2 * A.H + 2 * A.HD);
  uint64_t* bars = reinterpret_cast<uint64_t*>(phs + 3);
  float* red = reinterpret_cast<float*>(bars + kWarps * kStages);
  volatile int* flag = reinterpret_cast<volatile int*>(red + 32);
  float* rope_tab = red + 36;   // [nrope][cos, sin][HD / 2]
  constexpr int kPh16 = (int)(sizeof(MkPhase) / 16);
  auto fetch_desc = [&](int p) {   // descriptor p -> phs[p % 3], asynchronously
    const uint8_t* src = reinterpret_cast<const uint8_t*>(A.ph + p);
    uint8_t* dst = reinterpret_cast<uint8_t*>(phs + p % 3);
    for (int i = threadIdx.x; i < kPh16; i += kThreads) cp_async16(dst + 16 * i, src + 16 * i);
  };

  Ring R;
  R.base = ring + (size_t)warp * kStages * kQuantumBytes;
  R.full = bars + warp * kStages;
  R.cnt = 0;
  R.issued = 0;
  R.ok = true;
  R.wait_ns = 0;
  if (lane == 0) {
    for (int s = 0; s < kStages; s++) mbar_init(&R.full[s], 1);
    fence_barrier_init();
  }
  __syncwarp();
  const uint64_t pol = policy_evict_first();
  Prod u, pf;
  prod_init(A, u, c, warp);
  pf = u;
  for (int s = 0; s < kStages && u.idx < u.end; s++) {
    prod_issue(A, u, R.base + s * kQuantumBytes, &R.full[s], warp, lane, pol);
    R.issued++;
    prod_advance(A, pf, warp);
  }
  for (int s = 0; s < kPrefetch && pf.idx < pf.end; s++) prod_prefetch(A, pf, warp, lane);

  fetch_desc(0);
  if (A.nph > 1) fetch_desc(1);
  cp_async_commit();
  cp_async_wait_all();
  __syncthreads();
  stage_vectors(A, phs[0], wbuf);
  if (A.PD && c == 0) {
    // the token's PLE table row (used by every layer's PLE step) into L2
    const uint32_t row = __ldcg(A.params + 2);
    if (row < (uint32_t)A.V) {
      const size_t rb = (size_t)A.L * A.PD / 256 * 210;
      const uint8_t* r = A.ple_table + (size_t)row * rb;
      for (size_t o = (size_t)threadIdx.x * 128; o < rb + 128; o += (size_t)kThreads * 128)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(r + (o < rb ? o : rb - 1)));
    }
  }

  // RoPE cos / sin of this token's position for every layer kind
  // (kernels/headprep.wgsl:55: theta_p = pos * THETA^(-2p/HD))
  {
    const uint32_t pos = __ldcg(A.params + 0);
    const int half = A.HD / 2;
    for (int i = threadIdx.x; i < A.nrope * half; i += kThreads) {
      const int r = i / half, p = i - r * half;
      float sn = 0.f, cs = 1.f;
      if (p < A.rope_angles[r]) sincosf(rope_angle(pos, p, A.HD, A.rope_theta[r]), &sn, &cs);
      rope_tab[2 * r * half + p] = cs;
      rope_tab[(2 * r + 1) * half + p] = sn;
    }
  }

  // token embedding (kernels/q6k.wgsl MODE 0), computed by every CTA
  {
    const uint32_t row = __ldcg(A.params + 2);
    const bool ok = row < (uint32_t)A.V;
    if (!ok && c == 0 && threadIdx.x == 0) set_status(A.status, E4B_ST_BADINDEX);
    const uint8_t* r = A.emb + (size_t)(ok ? row : 0) * (A.H / 256) * 210;
    for (int i = threadIdx.x; i < A.H; i += kThreads)
      hs[i] = ok ? q6k_elem(r + (size_t)(i >> 8) * 210, i & 255) * A.emb_mult : 0.f;
  }

  // epochs of this launch: token counter * 256 + producing layer
  const uint32_t ebase = __ldcg(A.bar + 2) << 8;
  bool dead = false;          // this thread gave up polling (status TIMEOUT / abort)
  unsigned nbar = 0;
  bool alive = true;
  for (int p = 0; p < A.nph && alive; p++) {
    cp_async_wait_all();      // this phase's vectors and the next descriptor have landed
    __syncthreads();
    const MkPhase& P = phs[p % 3];
    if (p + 2 < A.nph) {
      fetch_desc(p + 2);
      cp_async_commit();
    }
    const bool tr = A.trace && c == 0 && threadIdx.x == 0;
    if (tr) A.trace[8 * p] = globaltimer_ns();
    if (P.kvpf && threadIdx.x == 0) prefetch_kv(A, P.a, c);
    if (P.res) residual(A, P, hs, wbuf, red, ebase, dead);
    if (tr) A.trace[8 * p + 1] = globaltimer_ns();
    if (P.kind == PH_FINAL) {
      float s = 0.f;
      for (int i = threadIdx.x; i < A.H; i += kThreads) s = fmaf(hs[i], hs[i], s);
      const float inv = rms_scale(cta_sum(s, red), A.H, A.eps);
      if (c == 0) {
        for (int i = threadIdx.x; i < A.H; i += kThreads) {
          A.hout[i] = hs[i];
          A.xf[i] = hs[i] * inv * wbuf[A.H + i];
        }
      }
      break;
    }
    if (P.kind == PH_ATTN) {
      attention_phase(A, P.a, c, wbuf + 2 * A.H, wbuf + 2 * A.H + A.HD, rope_tab, scr, red,
                      tr ? A.trace + 8 * p : nullptr, ebase, dead);
      if (tr) A.trace[8 * p + 4] = globaltimer_ns();
      __syncthreads();
      if (p + 1 < A.nph) stage_vectors(A, phs[(p + 1) % 3], wbuf);
    } else {
      const Work W = cta_work(P.g, A.G, c);
      // prologue: activations of this GEMV (only CTAs with work in it)
      if (W.nt > 0) {
        if (P.g.xk == XK_STAGED_F16) {   // the CTA's k-range of a global f16 input, polled
          const uint32_t* src = P.g.xg + 256 * W.k0;
          const uint32_t e16 = (ebase + (uint32_t)P.g.xtag) & 0xFFFFu;
          for (int i = threadIdx.x; i < W.kq * 64; i += kThreads) {
            uint4 w = ld_ll32x4(src + 4 * i);
            Spin sp;
            while (((w.x >> 16) != e16 || (w.y >> 16) != e16 || (w.z >> 16) != e16 || (w.w >> 16) != e16) && !dead) {
              if (!spin_more(sp, A)) dead = true;
              w = ld_ll32x4(src + 4 * i);
            }
            reinterpret_cast<uint2*>(xs)[i] = make_uint2(__byte_perm(w.x, w.y, 0x5410), __byte_perm(w.z, w.w, 0x5410));
          }
        }
        if (P.xb == XB_NORM || P.xb == XB_RAW)
          build_x_norm(A, hs, wbuf + A.H, reinterpret_cast<uint16_t*>(xs), red, P.xb == XB_NORM);
        else if (P.xb == XB_ATTN)
          build_x_attn(A, P, W, reinterpret_cast<uint16_t*>(xs), ebase, dead);
        else if (P.xb == XB_PLE)
          build_x_ple(A, P, wbuf + A.H, reinterpret_cast<uint16_t*>(xs), red, ebase, dead);
      }
      __syncthreads();
      if (p + 1 < A.nph) stage_vectors(A, phs[(p + 1) % 3], wbuf);
      if (tr) A.trace[8 * p + 2] = globaltimer_ns();
      {
        const bool xf32 = P.g.xk == XK_SMEM_F32;
        const void* xp = xf32 ? static_cast<const void*>(hs)
                              : (P.g.xk == XK_STAGED_F16   // staged block k0 sits at xs[0]
                                     ? static_cast<const void*>(reinterpret_cast<uint16_t*>(xs) - 256 * W.k0)
                                     : static_cast<const void*>(xs));
        if (xf32) gemv_phase<true>(A, W, warp, lane, R, u, pf, pol, xp, scr);
        else gemv_phase<false>(A, W, warp, lane, R, u, pf, pol, xp, scr);
      }
      if (!R.ok) dead = true;
      __syncthreads();
      if (tr) {
        A.trace[8 * p + 3] = globaltimer_ns();
        A.trace[8 * p + 7] = R.wait_ns;
        R.wait_ns = 0;
      }
      gemv_epilogue(P.g, W, scr, ebase);
    }
    if (A.trace) {
      __syncthreads();
      if (threadIdx.x == 0) {
        const unsigned long long t = globaltimer_ns();
        if (c == 0) A.trace[8 * p + 4] = t;
        atomicMax(A.trace + 8 * p + 5, t);
      }
    }
    // end of phase: the CTA's shared scratch is free again; a thread that gave
    // up stops the CTA (the others give up through the abort flag)
    if (__syncthreads_or(dead ? 1 : 0)) {
      alive = false;
      break;
    }
    if (P.sync_after) {
      nbar++;
      alive = grid_sync(A.bar, nbar * (unsigned)A.G, A.status, flag);
    }
    if (tr) A.trace[8 * p + 6] = globaltimer_ns();
  }

  cp_async_wait_all();
  // drain this warp's copies still in flight (only after a failure)
  for (uint32_t k = R.cnt; k < R.issued; k++) {
    const uint32_t s = k % kStages;
    if (!mbar_wait(&R.full[s], (k / kStages) & 1u, A.status)) break;
  }
  if (alive) {
    __syncthreads();
    if (threadIdx.x == 0) {
      // last CTA out resets the barrier counters for the next launch
      const unsigned done = atomicAdd(A.bar + 1, 1u);
      if (done == (unsigned)A.G - 1u) {
        A.bar[0] = 0u;
        A.bar[1] = 0u;
        A.bar[2] = A.bar[2] + 1u;   // next launch's epochs
        __threadfence();
      }
    }
  }
}

// ------------------------------------------------------------------ host side
struct DensePlan {
  MkArgs args{};
  int G = 0;
  size_t smem = 0;
  std::vector<void*> allocs;
  std::vector<int> kinds;   // per phase: 0 Wp, 1 qkv, 2 attention, 3 o, 4 gate|up, 5 down, 6 PLE gate, 7 PLE proj, 8 final
};

std::vector<DensePlan*>& registry(e4b_ctx* c) {
  static std::vector<std::pair<e4b_ctx*, std::vector<DensePlan*>>> all;
  for (auto& e : all)
    if (e.first == c) return e.second;
  all.push_back({c, {}});
  return all.back().second;
}

void plan_free(DensePlan* p) {
  for (void* a : p->allocs) cudaFree(a);
  delete p;
}

// k-split of a GEMV: 1 for the gate|up GEMV (GeGLU needs whole sums) and
// whenever there are at least G/2 tiles; else as many splits (at most 2, the
// consumers' load pattern) as fit the grid while every split keeps >= 8 quanta.
int split_for(int T, int qpr, int gu, int G) {
  if (gu) return 1;
  return std::max(1, std::min(std::min(G / T, qpr / 8), 2));
}

struct Builder {
  e4b_ctx* c;
  DensePlan* plan;
  int G;
  std::vector<MkPhase> ph;
  std::vector<const uint8_t*> wt_of_phase;   // the GEMV's tile-packed weights, null: none
  std::vector<long long> load;     // cumulative weight bytes per CTA (rotation choice)

  int alloc(size_t bytes, void** out) {
    *out = nullptr;
    cudaError_t e = cudaMalloc(out, bytes ? bytes : 16);
    if (e != cudaSuccess) return e4b_fail(c, E4B_ENOMEM, "dense plan: cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    plan->allocs.push_back(*out);
    cudaMemsetAsync(*out, 0, bytes ? bytes : 16, c->stream);
    return E4B_OK;
  }

  MkPhase& add(int kind) {
    MkPhase p;
    memset(&p, 0, sizeof(p));
    p.kind = kind;
    p.rmul = 1.f;
    ph.push_back(p);
    wt_of_phase.push_back(nullptr);
    return ph.back();
  }

  // One q4_0 GEMV [rows][IN] in phase P (the last added).
  int gemv(MkPhase& P, const uint8_t* w, int IN, int OUT, int gu, int ff, int xk, const uint32_t* xg, int xtag,
           uint64_t* out, uint32_t* outh, int tag, SlotSrc* src) {
    E4B_REQUIRE(c, w && IN > 0 && IN % 256 == 0 && IN <= 65536, "dense plan: GEMV IN=%d must be a multiple of 256", IN);
    E4B_REQUIRE(c, reinterpret_cast<uintptr_t>(w) % 16 == 0, "dense plan: weight not 16-byte aligned");
    MkGemv& g = P.g;
    g.qpr = IN / 256;
    g.gu = gu;
    g.ff = ff;
    g.T = gu ? (ff + 15) / 16 : (OUT + 31) / 32;
    g.s = split_for(g.T, g.qpr, gu, G);
    g.xk = xk;
    g.xg = xg;
    g.xtag = xtag;
    g.tag = tag;
    g.epi = gu ? EPI_GEGLU : EPI_SLOTS;
    g.out = out;
    g.outh = outh;
    // rotation: place the pieces where the cumulative weight traffic is lowest
    std::vector<long long> b(G);
    for (int v = 0; v < G; v++) {
      const Work W = cta_work(g.T, g.qpr, g.s, 0, G, v);
      b[v] = (long long)W.nt * W.kq * kQuantumBytes;
    }
    long long best = -1;
    int best_rot = 0;
    for (int rot = 0; rot < G; rot++) {
      long long mx = 0;
      for (int cc = 0; cc < G; cc++) {
        int v = cc - rot;
        if (v < 0) v += G;
        mx = std::max(mx, load[cc] + b[v]);
      }
      if (best < 0 || mx < best) {
        best = mx;
        best_rot = rot;
      }
    }
    g.rot = best_rot;
    for (int cc = 0; cc < G; cc++) {
      int v = cc - best_rot;
      if (v < 0) v += G;
      load[cc] += b[v];
    }
    if (src) *src = SlotSrc{out, g.s, tag};
    // a tile-packed copy of the weights (2304-byte pieces of 16 rows x 256 k),
    // owned by the plan: every quantum is two contiguous bulk copies
    const int rows_total = gu ? 2 * ff : OUT;
    E4B_REQUIRE(c, gu ? ff % 16 == 0 : OUT % 32 == 0, "dense plan: GEMV rows %d (ff %d) not in 32-row tiles", OUT, ff);
    uint8_t* wt = nullptr;
    if (int rc = alloc((size_t)rows_total * (IN / 32) * 18, (void**)&wt)) return rc;
    if (int rc = e4b_q40_pack_tiles(c, w, wt, rows_total, IN)) return rc;
    wt_of_phase.back() = wt;
    return E4B_OK;
  }
};

int plan_create(e4b_ctx* c, const e4b_dense_model* m, int* handle) {
  E4B_REQUIRE(c, m && handle, "dense plan: null argument");
  const int H = m->hidden, QH = m->q_heads, KVH = m->kv_heads, HD = m->head_dim, FF = m->ff, PD = m->ple_dim;
  const int L = m->layers, qdim = QH * HD;
  E4B_REQUIRE(c, L > 0 && m->layer, "dense plan: no layers");
  E4B_REQUIRE(c, H % 256 == 0 && H <= kMaxPer * kThreads, "dense plan: hidden %d must be a multiple of 256, <= %d", H,
              kMaxPer * kThreads);
  E4B_REQUIRE(c, QH > 0 && KVH > 0 && QH % KVH == 0 && HD % 64 == 0 && HD <= 1024 && qdim % 256 == 0,
              "dense plan: bad head geometry QH=%d KVH=%d HD=%d", QH, KVH, HD);
  E4B_REQUIRE(c, FF % 256 == 0, "dense plan: ff %d must be a multiple of 256", FF);
  E4B_REQUIRE(c, PD == 0 || (PD % 256 == 0 && PD <= kMaxPer * kThreads && m->ple_table && m->ple_proj_w && m->ple_norm),
              "dense plan: ple_dim %d must be a multiple of 256 with table, projection and norm", PD);
  E4B_REQUIRE(c, m->token_embd && m->params && m->xf && m->hidden_out && m->out_norm, "dense plan: missing buffers");
  E4B_REQUIRE(c, m->vocab > 0 && m->eps > 0.f, "dense plan: bad vocab / eps");
  const int G = c->sm_count;
  E4B_REQUIRE(c, G > 0, "dense plan: no SMs");

  DensePlan* plan = new DensePlan();
  Builder b{c, plan, G, {}, {}, std::vector<long long>(G, 0)};
  auto fail = [&](int rc) {
    plan_free(plan);
    return rc;
  };

  int max_qkv = 0, max_slots = 0;
  for (int l = 0; l < L; l++) {
    const e4b_dense_layer& ly = m->layer[l];
    max_qkv = std::max(max_qkv, ly.qkv_rows);
    max_slots = std::max(max_slots, ly.slots);
    const bool ok = ly.qkv && ly.o && ly.gu && ly.down && ly.attn_norm && ly.q_norm && ly.k_norm && ly.post_attn &&
                    ly.ffn_norm && ly.post_ffw && ly.kcache && ly.vcache && ly.slots > 0 &&
                    ly.rope_angles >= 0 && ly.rope_angles <= HD / 2 &&
                    ly.qkv_rows == qdim + KVH * HD * (ly.keqv ? 1 : 2) &&
                    (!ly.sliding || (ly.ring > 0 && ly.ring <= ly.slots)) &&
                    (!PD || (ly.ple_gate && ly.ple_proj && ly.post_norm));
    if (!ok) return fail(e4b_fail(c, E4B_EINVAL, "dense plan: layer %d incomplete or inconsistent", l));
  }
  const int nct = std::max(1, G / QH);

  // activations owned by the plan: every channel a layer writes is double
  // buffered by layer parity (a buffer is rewritten two layers later, after a
  // grid barrier), published as epoch words
  E4B_REQUIRE(c, L < 255, "dense plan: at most 254 layers");
  auto out_bytes = [&](int rows, int IN) {
    const int T = (rows + 31) / 32;
    return (size_t)T * split_for(T, IN / 256, 0, G) * 32 * 8;
  };
  uint64_t *qkv_s[2], *to_s[2], *td_s[2], *pg_s[2] = {nullptr, nullptr}, *tp_s[2] = {nullptr, nullptr};
  uint64_t* wp_s = nullptr;
  float *part_o[2], *part_ml[2];
  uint32_t* att_out[2];
  unsigned* att_cnt;
  uint32_t* geglu[2];
  unsigned* bar;
  int rc;
  size_t qkv_bytes = 0;
  for (int l = 0; l < L; l++) qkv_bytes = std::max(qkv_bytes, out_bytes(m->layer[l].qkv_rows, H));
  for (int k = 0; k < 2; k++) {
    if ((rc = b.alloc(qkv_bytes, (void**)&qkv_s[k]))) return fail(rc);
    if ((rc = b.alloc(out_bytes(H, qdim), (void**)&to_s[k]))) return fail(rc);
    if ((rc = b.alloc(out_bytes(H, FF), (void**)&td_s[k]))) return fail(rc);
    if ((rc = b.alloc((size_t)FF * 4, (void**)&geglu[k]))) return fail(rc);
    if (PD) {
      if ((rc = b.alloc(out_bytes(PD, H), (void**)&pg_s[k]))) return fail(rc);
      if ((rc = b.alloc(out_bytes(H, PD), (void**)&tp_s[k]))) return fail(rc);
    }
    if ((rc = b.alloc((size_t)QH * nct * HD * 4, (void**)&part_o[k]))) return fail(rc);
    if ((rc = b.alloc((size_t)QH * nct * 2 * 4, (void**)&part_ml[k]))) return fail(rc);
    if ((rc = b.alloc((size_t)QH * HD * 4, (void**)&att_out[k]))) return fail(rc);
  }
  if (PD && (rc = b.alloc(out_bytes(L * PD, H), (void**)&wp_s))) return fail(rc);
  if ((rc = b.alloc(64, (void**)&bar))) return fail(rc);
  if ((rc = b.alloc((size_t)QH * 4, (void**)&att_cnt))) return fail(rc);
  E4B_REQUIRE(c, nct <= 64, "dense plan: at most 64 attention chunks per head");
  {
    // token counter starts at 1: zero-initialised words carry epoch 0, never current
    const unsigned one = 1u;
    cudaError_t e = cudaMemcpyAsync(bar + 2, &one, 4, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) return fail(e4b_fail(c, E4B_ECUDA, "dense plan: %s", cudaGetErrorString(e)));
  }

  MkArgs& A = plan->args;
  A.G = G;
  A.H = H;
  A.QH = QH;
  A.KVH = KVH;
  A.HD = HD;
  A.PD = PD;
  A.L = L;
  A.V = m->vocab;
  A.qdim = qdim;
  A.eps = m->eps;
  A.emb_mult = sqrtf((float)H);
  A.ple_mult = PD ? sqrtf((float)PD) : 0.f;
  A.proj_scale = 1.0f / sqrtf((float)H);
  A.emb = m->token_embd;
  A.ple_table = m->ple_table;
  A.ple_norm = m->ple_norm;
  A.out_norm = m->out_norm;
  A.params = m->params;
  A.status = c->status;
  A.bar = bar;
  A.xf = m->xf;
  A.hout = m->hidden_out;

  // ---- phase list
  if (PD) {
    MkPhase& P = b.add(PH_GEMV);
    P.xb = XB_F32;
    if ((rc = b.gemv(P, m->ple_proj_w, H, L * PD, 0, 0, XK_SMEM_F32, nullptr, 0, wp_s, nullptr, 255, &A.pleproj)))
      return fail(rc);
  }
  SlotSrc prev_t{};
  const float* prev_w = nullptr;
  float prev_mul = 1.f;
  for (int l = 0; l < L; l++) {
    const e4b_dense_layer& ly = m->layer[l];
    const int pb = l & 1;   // buffer parity of this layer
    SlotSrc qkv_src, to_src, td_src, pg_src, tp_src;
    {   // q|k|v (and the L2 prefetch of this layer's KV cache)
      MkPhase& P = b.add(PH_GEMV);
      P.kvpf = 1;
      if (l > 0) {
        P.res = 1;
        P.rt = prev_t;
        P.rw = prev_w;
        P.rmul = prev_mul;
        P.dump = m->dump ? m->dump + (size_t)(l - 1) * H : nullptr;
      }
      P.xb = XB_NORM;
      P.xw = ly.attn_norm;
      if ((rc = b.gemv(P, ly.qkv, H, ly.qkv_rows, 0, 0, XK_SMEM_F16, nullptr, 0, qkv_s[pb], nullptr, l, &qkv_src)))
        return fail(rc);
    }
    MkAttn at{};
    at.qkv = qkv_src;
    at.qn = ly.q_norm;
    at.kn = ly.k_norm;
    at.kc = ly.kcache;
    at.vc = ly.vcache;
    at.part_o = part_o[pb];
    at.part_ml = part_ml[pb];
    at.cnt = att_cnt;
    at.out = att_out[pb];
    at.tag = l;
    at.cachemode = ly.sliding ? 1 : 2;
    at.ring = ly.sliding ? ly.ring : 1;
    at.window = ly.sliding ? m->window : 0;
    at.slots = ly.slots;
    at.angles = ly.rope_angles;
    at.keqv = ly.keqv ? 1 : 0;
    at.nct = nct;
    at.theta = ly.theta;
    at.scale = 1.0f;
    at.rope = -1;
    for (int r = 0; r < A.nrope; r++)
      if (A.rope_theta[r] == ly.theta && A.rope_angles[r] == ly.rope_angles) at.rope = r;
    if (at.rope < 0) {
      if (A.nrope == kMaxRope) return fail(e4b_fail(c, E4B_EINVAL, "dense plan: more than %d RoPE kinds", kMaxRope));
      A.rope_theta[A.nrope] = ly.theta;
      A.rope_angles[A.nrope] = ly.rope_angles;
      at.rope = A.nrope++;
    }
    b.ph.back().a = at;   // the q|k|v phase prefetches this layer's cache
    {
      MkPhase& P = b.add(PH_ATTN);
      P.a = at;
    }
    {   // o
      MkPhase& P = b.add(PH_GEMV);
      P.xb = XB_ATTN;
      P.a = at;
      if ((rc = b.gemv(P, ly.o, qdim, H, 0, 0, XK_SMEM_F16, nullptr, 0, to_s[pb], nullptr, l, &to_src)))
        return fail(rc);
    }
    {   // gate|up + GeGLU
      MkPhase& P = b.add(PH_GEMV);
      P.res = 1;
      P.rt = to_src;
      P.rw = ly.post_attn;
      P.rmul = 1.f;
      P.xb = XB_NORM;
      P.xw = ly.ffn_norm;
      if ((rc = b.gemv(P, ly.gu, H, 2 * FF, 1, FF, XK_SMEM_F16, nullptr, 0, nullptr, geglu[pb], l, nullptr)))
        return fail(rc);
    }
    {   // down
      MkPhase& P = b.add(PH_GEMV);
      P.xb = XB_NONE;
      if ((rc = b.gemv(P, ly.down, FF, H, 0, 0, XK_STAGED_F16, geglu[pb], l, td_s[pb], nullptr, l, &td_src)))
        return fail(rc);
      if (!PD) P.sync_after = 1;
    }
    if (PD) {
      {   // PLE gate: h += rms(t_d) post_ffw; x = f16(h)
        MkPhase& P = b.add(PH_GEMV);
        P.res = 1;
        P.rt = td_src;
        P.rw = ly.post_ffw;
        P.rmul = 1.f;
        P.xb = XB_RAW;
        if ((rc = b.gemv(P, ly.ple_gate, H, PD, 0, 0, XK_SMEM_F16, nullptr, 0, pg_s[pb], nullptr, l, &pg_src)))
          return fail(rc);
      }
      {   // PLE projection
        MkPhase& P = b.add(PH_GEMV);
        P.xb = XB_PLE;
        P.xw = m->ple_norm;
        P.layer = l;
        P.ple_gate = pg_src;
        if ((rc = b.gemv(P, ly.ple_proj, PD, H, 0, 0, XK_SMEM_F16, nullptr, 0, tp_s[pb], nullptr, l, &tp_src)))
          return fail(rc);
        P.sync_after = 1;
      }
      prev_t = tp_src;
      prev_w = ly.post_norm;
    } else {
      prev_t = td_src;
      prev_w = ly.post_ffw;
    }
    prev_mul = ly.scale;
  }
  {
    MkPhase& P = b.add(PH_FINAL);
    P.xw = m->out_norm;
    P.res = 1;
    P.rt = prev_t;
    P.rw = prev_w;
    P.rmul = prev_mul;
    P.dump = m->dump ? m->dump + (size_t)(L - 1) * H : nullptr;
  }

  // ---- device copies: phases and every warp's weight schedule
  MkPhase* d_ph = nullptr;
  SchedEnt* d_sched = nullptr;
  int2* d_rng = nullptr;
  if ((rc = b.alloc(b.ph.size() * sizeof(MkPhase), (void**)&d_ph))) return fail(rc);
  std::vector<SchedEnt> sched;
  std::vector<int2> rng((size_t)G * kWarps);
  int max_tiles = 1;
  for (int cc = 0; cc < G; cc++)
    for (int w = 0; w < kWarps; w++) {
      rng[(size_t)cc * kWarps + w].x = (int)sched.size();
      for (size_t i = 0; i < b.ph.size(); i++) {
        const MkPhase& P = b.ph[i];
        if (P.kind != PH_GEMV) continue;
        const Work W = cta_work(P.g.T, P.g.qpr, P.g.s, P.g.rot, G, cc);
        max_tiles = std::max(max_tiles, W.nt);
        const int nw = warp_items(W, w);
        if (nw == 0) continue;
        SchedEnt e;
        e.wt = b.wt_of_phase[i];
        e.nq = P.g.qpr;
        e.t0 = W.t0;
        e.k0 = W.k0;
        e.kq = W.kq;
        e.nw = nw;
        e.gu = P.g.gu;
        e.ff = P.g.ff;
        sched.push_back(e);
      }
      rng[(size_t)cc * kWarps + w].y = (int)sched.size() - rng[(size_t)cc * kWarps + w].x;
    }
  if ((rc = b.alloc(std::max<size_t>(1, sched.size()) * sizeof(SchedEnt), (void**)&d_sched))) return fail(rc);
  if ((rc = b.alloc(rng.size() * sizeof(int2), (void**)&d_rng))) return fail(rc);
  cudaError_t e = cudaMemcpyAsync(d_ph, b.ph.data(), b.ph.size() * sizeof(MkPhase), cudaMemcpyHostToDevice, c->stream);
  if (e == cudaSuccess && !sched.empty())
    e = cudaMemcpyAsync(d_sched, sched.data(), sched.size() * sizeof(SchedEnt), cudaMemcpyHostToDevice, c->stream);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(d_rng, rng.data(), rng.size() * sizeof(int2), cudaMemcpyHostToDevice, c->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) return fail(e4b_fail(c, E4B_ECUDA, "dense plan upload: %s", cudaGetErrorString(e)));
  A.ph = d_ph;
  A.nph = (int)b.ph.size();
  {
    // phase names for traces, from the order the list was built in
    int k = 0;
    if (PD) plan->kinds.push_back(0), k++;
    for (int l = 0; l < L; l++) {
      for (int t : {1, 2, 3, 4, 5}) plan->kinds.push_back(t);
      if (PD) plan->kinds.push_back(6), plan->kinds.push_back(7);
    }
    plan->kinds.push_back(8);
    (void)k;
  }
  A.sched = d_sched;
  A.sched_rng = d_rng;

  // ---- shared memory
  int maxCH = 32, nch_unused = 0;
  chunking((uint32_t)max_slots, nct, maxCH, nch_unused);
  size_t xs_need = (size_t)std::max(std::max(2 * H, 2 * qdim), 2 * std::max(PD, 1));
  for (const MkPhase& P : b.ph)
    if (P.kind == PH_GEMV && P.g.xk == XK_STAGED_F16)
      for (int cc = 0; cc < G; cc++)
        xs_need = std::max(xs_need, (size_t)512 * cta_work(P.g.T, P.g.qpr, P.g.s, P.g.rot, G, cc).kq);
  const size_t xs_bytes = (xs_need + 127) & ~(size_t)127;
  const size_t scr_bytes =
      (std::max(std::max((size_t)max_tiles * kWarps * 32 * 4, (size_t)(4 * (HD / 4 + 4) + 2 * HD + kThreads * 8 + maxCH) * 4),
                (size_t)(QH * nct + QH) * 4) + 127) & ~(size_t)127;
  const size_t smem = (size_t)kWarps * kStages * kQuantumBytes + (size_t)H * 4 + xs_bytes + scr_bytes +
                      (size_t)(2 * H + 2 * HD) * 4 + 3 * sizeof(MkPhase) + (size_t)kWarps * kStages * 8 + 36 * 4 +
                      (size_t)kMaxRope * HD * 4 + 16;
  A.xs_bytes = (int)xs_bytes;
  A.scr_bytes = (int)scr_bytes;
  e = cudaFuncSetAttribute(k_decode_dense, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess)
    return fail(e4b_fail(c, E4B_ECUDA, "dense plan: %zu B of shared memory: %s", smem, cudaGetErrorString(e)));
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode_dense, kThreads, smem);
  if (e != cudaSuccess || per_sm < 1)
    return fail(e4b_fail(c, E4B_ECUDA, "dense plan: kernel does not fit one CTA per SM (%zu B shared)", smem));
  plan->G = G;
  plan->smem = smem;
  auto& reg = registry(c);
  reg.push_back(plan);
  *handle = (int)reg.size() - 1;
  return E4B_OK;
}

}  // namespace

namespace e4b {
void dense_plans_release(e4b_ctx* c) {
  auto& reg = registry(c);
  for (auto*& p : reg)
    if (p) {
      plan_free(p);
      p = nullptr;
    }
  reg.clear();
}
}  // namespace e4b

extern "C" {

E4B_API int e4b_dense_plan_create(e4b_ctx* c, const e4b_dense_model* m, int* handle) {
  E4B_CHECK_CTX(c);
  cudaSetDevice(c->device);
  return plan_create(c, m, handle);
}

E4B_API int e4b_dense_plan_run(e4b_ctx* c, int handle) {
  E4B_CHECK_CTX(c);
  auto& reg = registry(c);
  E4B_REQUIRE(c, handle >= 0 && handle < (int)reg.size() && reg[handle], "bad dense plan %d", handle);
  DensePlan* p = reg[handle];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p->G);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = p->smem;
  cfg.stream = c->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, k_decode_dense, p->args);
  if (e != cudaSuccess) return e4b_fail(c, E4B_ECUDA, "dense plan launch: %s", cudaGetErrorString(e));
  return E4B_OK;
}

E4B_API int e4b_dense_plan_trace(e4b_ctx* c, int handle, unsigned long long* buf) {
  E4B_CHECK_CTX(c);
  auto& reg = registry(c);
  E4B_REQUIRE(c, handle >= 0 && handle < (int)reg.size() && reg[handle], "bad dense plan %d", handle);
  reg[handle]->args.trace = buf;
  return E4B_OK;
}

E4B_API int e4b_dense_plan_phases(e4b_ctx* c, int handle, int* kinds, int max) {
  E4B_CHECK_CTX(c);
  auto& reg = registry(c);
  E4B_REQUIRE(c, handle >= 0 && handle < (int)reg.size() && reg[handle], "bad dense plan %d", handle);
  DensePlan* p = reg[handle];
  E4B_REQUIRE(c, kinds && max >= p->args.nph, "dense plan phases: need room for %d entries", p->args.nph);
  for (int i = 0; i < p->args.nph; i++) kinds[i] = p->kinds[i];
  return p->args.nph;
}

E4B_API int e4b_dense_plan_destroy(e4b_ctx* c, int handle) {
  E4B_CHECK_CTX(c);
  auto& reg = registry(c);
  E4B_REQUIRE(c, handle >= 0 && handle < (int)reg.size() && reg[handle], "bad dense plan %d", handle);
  E4B_CUDA(c, cudaStreamSynchronize(c->stream));
  plan_free(reg[handle]);
  reg[handle] = nullptr;
  return E4B_OK;
}

}  // extern "C"
