// Batched split-KV decode attention on the tensor cores (kernels/attsplit.wgsl
// + attcomb.wgsl semantics for nseq sequences at one common position).
//
// Work item = (sequence, KV head, chunk of 64 cache slots); only chunks that
// hold live slots are visited, by a persistent grid.  Per item the CTA loads
// the chunk's K and V tiles with 4-D TMA boxes of [64 slots x 64 dims] (the
// cache viewed as [nseq][slots][KVH][HD], 128-byte swizzle, so the MMA reads
// are bank-conflict free) up to two items ahead of use, and does both products
// on mma.sync m16n8k16 with the G query heads of the KV head as the 8 MMA
// columns, so each KV row is read once for the whole GQA group:
//   S^T[slot][head] = K[slot][:] . q[head][:]   (A = K rows, B = q as f16 hi + lo)
//   O^T[d][head]    = V^T[d][slot] . P^T[slot][head]   (A = V via ldmatrix.trans,
//                                                        B = p as f16 hi + lo)
// K and V are f16 in the cache, so with the hi + lo split every product is the
// reference's f32 product to ~2^-22; sums are f32.  Per chunk the kernel writes
// the unnormalised sum_t p_t v_t with its (max, sum p) as the reference's
// phase A does; the combine kernel merges the live chunks (phase B).
#include "attn.cuh"
#include "q40_frag.cuh"
#include "q40_stream.cuh"

namespace {
using namespace e4b;

constexpr int kAC = 64;            // slots per chunk
constexpr int kAW = 4;             // warps per CTA
constexpr int kAS = 3;             // stages (items in flight)
constexpr int kPP = kAC + 8;       // padded p row (halves)
constexpr int kSub = kAC * 128;    // bytes of one [64 slots x 64 dims] swizzled box

struct AttP {
  const float* q;                  // [nseq][QH][HD]
  const uint16_t* kc;
  const uint16_t* vc;
  const uint32_t* params;
  float* part_o;                   // [nseq][QH][max_chunks][HD]
  float* part_ml;                  // [nseq][QH][max_chunks][2]
  uint32_t* status;
  int QH, KVH, HD, G, window, cachemode, ring, max_chunks, nseq, keqv;
  float scale;
  size_t seq_stride;               // halves between sequences' caches
  uint64_t wait_ns;                // bound of every wait (time-out -> E4B_ST_TIMEOUT)
};

// Tiles are HD/64 boxes of [64 slots x 128 bytes] under the 128-byte swizzle:
// the 16-byte chunk c of slot row r sits at chunk c ^ (r & 7) of its row.
E4B_DEV void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

E4B_DEV void ldsm_x4_trans(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* ptr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(ptr)));
}
E4B_DEV uint32_t lds32(const uint16_t* ptr) { return *reinterpret_cast<const uint32_t*>(ptr); }

// The cache as a 4-D f16 tensor [nseq][slots][KVH][HD] for TMA boxes of
// [64 dims x 1 head x 64 slots x 1 sequence] with the 128-byte swizzle.
bool cache_map(CUtensorMap* m, const uint16_t* base, int HD, int KVH, int slots, int nseq) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  const cuuint64_t dim[4] = {(cuuint64_t)HD, (cuuint64_t)KVH, (cuuint64_t)slots, (cuuint64_t)nseq};
  const cuuint64_t stride[3] = {(cuuint64_t)HD * 2, (cuuint64_t)KVH * HD * 2, (cuuint64_t)slots * KVH * HD * 2};
  const cuuint32_t box[4] = {64, 1, kAC, 1};
  const cuuint32_t es[4] = {1, 1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<uint16_t*>(base), dim, stride, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

E4B_DEV SlotRule att_rule(const AttP& p) {
  SlotRule r{p.cachemode, p.ring, p.window, 0, 0};
  r.qp = p.params[0];
  r.len = p.cachemode == 2 ? p.params[5] : p.params[1];
  return r;
}
// First chunk holding a valid slot: a windowed linear cache skips the slots
// before its window; rings and unwindowed caches start at 0.
E4B_DEV int first_chunk(const SlotRule& r) {
  if (r.cachemode == 0 && r.window > 0 && r.len > (uint32_t)r.window) return (int)((r.len - r.window) / kAC);
  return 0;
}

// Two groups of kAW warps per CTA take alternate items of the CTA's run (named
// barriers per group), so one group's MMAs and softmax overlap the other's
// waits; both draw from one kAS-deep ring of K/V stages.
constexpr int kAG = 2;             // warp groups per CTA

E4B_DEV void group_sync(int grp) { asm volatile("bar.sync %0, %1;" ::"r"(1 + grp), "r"(32 * kAW) : "memory"); }

// Stage ring protocol.  Item `local` of a CTA's run uses stage local % kAS and
// is that stage's (local / kAS)-th load, i.e. barrier phase local / kAS.  The
// two groups alternate items and kAS is odd, so consecutive uses of a stage
// belong to different groups, and a parity wait alone cannot tell phase k from
// phase k - 2 (a consumer that runs ahead would pass on the stage's previous
// load).  So the issuing thread publishes, per stage, the item it issued last
// (release), and a consumer first waits until its own item is the one issued
// (acquire): the stage's previous item has then been consumed, and the next one
// cannot be issued before this consumer is done, so the parity of phase
// local / kAS is unambiguous.  Every wait is bounded and also ends when another
// CTA has recorded a time-out in the status word.
E4B_DEV void st_release_cta(int* a, int v) {
  asm volatile("st.release.cta.shared::cta.s32 [%0], %1;" ::"r"(smem_u32(a)), "r"(v) : "memory");
}
E4B_DEV int ld_acquire_cta(const int* a) {
  int v;
  asm volatile("ld.acquire.cta.shared::cta.s32 %0, [%1];" : "=r"(v) : "r"(smem_u32(a)) : "memory");
  return v;
}
E4B_DEV bool aborted(const uint32_t* status) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(status) : "memory");
  return (v & E4B_ST_TIMEOUT) != 0;
}
// Spin until `pred()`; false after `limit_ns` (recording E4B_ST_TIMEOUT) or as
// soon as another CTA has recorded one.
template <class Pred>
E4B_DEV bool bounded_spin(Pred pred, uint32_t* status, uint64_t limit_ns) {
  if (pred()) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0;; i++) {
    if (pred()) return true;
    if ((i & 63u) == 63u) {
      if (aborted(status)) return false;
      if (globaltimer_ns() - t0 > limit_ns) {
        set_status(status, E4B_ST_TIMEOUT);
        return false;
      }
    }
  }
}

__global__ void __launch_bounds__(32 * kAW * kAG, 1) k_attdec(const AttP p, const __grid_constant__ CUtensorMap kmap,
                                                              const __grid_constant__ CUtensorMap vmap) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kAS];
  __shared__ int issued[kAS];                           // per stage: the item issued into it last
  __shared__ float red_m[kAG][kAW][8], red_l[kAG][kAW][8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int grp = warp / kAW, wg = warp % kAW;          // warp group, warp within the group
  const int gtid = threadIdx.x - grp * 32 * kAW;        // thread within the group
  const int tile = (p.HD / 64) * kSub;                  // bytes per K or V tile
  // swizzled boxes need 1024-byte aligned destinations
  uint8_t* kv = smem + ((1024u - (smem_u32(smem) & 1023u)) & 1023u);          // [kAS stages][K tile | V tile]
  uint4* qf = reinterpret_cast<uint4*>(kv + (size_t)kAS * 2 * tile) + (size_t)grp * (p.HD / 16) * 32;
  uint16_t* ph = reinterpret_cast<uint16_t*>(reinterpret_cast<uint4*>(kv + (size_t)kAS * 2 * tile) +
                                             (size_t)kAG * (p.HD / 16) * 32) + (size_t)grp * 2 * 8 * kPP;
  uint16_t* pl = ph + 8 * kPP;                          // this group's p rows: hi, lo [8 heads][kPP]
  for (int i = gtid; i < 2 * 8 * kPP; i += 32 * kAW) ph[i] = 0;
  if (threadIdx.x == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&kmap)) : "memory");
    if (!p.keqv) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&vmap)) : "memory");
    for (int s = 0; s < kAS; s++) {
      mbar_init(&full[s], 1);
      issued[s] = -1;
    }
    fence_barrier_init();
  }
  __syncthreads();
  pdl_trigger();
  pdl_wait();
  const SlotRule rule = att_rule(p);
  const uint32_t n = rule.nslots();
  const int nch_all = (int)((n + kAC - 1) / kAC);
  if (nch_all > p.max_chunks) {
    if (threadIdx.x == 0) set_status(p.status, E4B_ST_BADINDEX);
    return;
  }
  const int c_lo = first_chunk(rule), nch = nch_all - c_lo;       // live chunks [c_lo, nch_all)
  const int per_seq = p.KVH * nch, items = p.nseq * per_seq;
  // a contiguous run of items per CTA: consecutive chunks of one (sequence, KV head)
  const int i0 = (int)((long long)items * blockIdx.x / gridDim.x);
  const int i1 = (int)((long long)items * (blockIdx.x + 1) / gridDim.x);

  // one thread issues an item's boxes into stage (item - i0) % kAS: HD/64 for
  // K (+ HD/64 for V); slots past the cache's end read as zeros, slots past the
  // live ones are finite cache contents that only meet p = 0
  auto issue = [&](int it) {
    const int s = (it - i0) % kAS;
    const int b = it / per_seq, rem = it % per_seq, kvh = rem / nch, c = c_lo + rem % nch;
    uint8_t* dk = kv + (size_t)s * 2 * tile;
    mbar_expect_tx(&full[s], (uint32_t)tile * (p.keqv ? 1u : 2u));
    for (int j = 0; j < p.HD / 64; j++) {
      tma_load_4d(dk + j * kSub, &kmap, 64 * j, kvh, c * kAC, b, &full[s]);
      if (!p.keqv) tma_load_4d(dk + tile + j * kSub, &vmap, 64 * j, kvh, c * kAC, b, &full[s]);
    }
    st_release_cta(&issued[s], it);
  };
  if (threadIdx.x == 0)
    for (int k = 0; k < kAS; k++)
      if (i0 + k < i1) issue(i0 + k);

  // lane-constant shared-memory offsets of the swizzled tiles:
  //   scores A: rows r0 = 16 wg + g (+8), chunk 2u (+1) of box j/4 -> xor with r0 & 7 = g
  //   P.V A (ldmatrix.trans): row 16 ks + lrow, chunk 2 (dt & 3) + hbit of box dt / 4, xor with lane & 7
  const int r0 = 16 * wg + g;
  uint32_t koff[8];
#pragma unroll
  for (int u = 0; u < 8; u++) koff[u] = (uint32_t)(r0 * 128 + ((u ^ g) << 4) + 4 * t);
  const int dtiles = p.HD / 16 / kAW;           // 1..4
  const int lrow = (lane & 7) + ((lane >> 4) << 3), hbit = (lane >> 3) & 1;
  uint32_t voff[4];
#pragma unroll
  for (int u = 0; u < 4; u++) {
    const int dt = wg * dtiles + u;
    voff[u] = (uint32_t)((dt >> 2) * kSub + lrow * 128 + (((2 * (dt & 3) + hbit) ^ (lane & 7)) << 4));
  }
  bool ok = true;
  int qb = -1, qk = -1;                          // (sequence, KV head) whose q fragments qf holds
  for (int it = i0 + grp; it < i1; it += kAG) {
    const int local = it - i0, s = local % kAS;
    const int b = it / per_seq, rem = it % per_seq, kvh = rem / nch, c = c_lo + rem % nch;
    const uint32_t t0 = (uint32_t)c * kAC;
    // q fragments of the group's heads: (q[k], q[k+1]) and (q[k+8], q[k+9]), k = 16 j + 2 t, hi and lo;
    // rebuilt when this group moves to another (sequence, KV head)
    if (b != qb || kvh != qk) {
      for (int i = gtid; i < (p.HD / 16) * 32; i += 32 * kAW) {
        const int j = i >> 5, gg = (i & 31) >> 2, tt = i & 3;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (gg < p.G) {
          const float* qr = p.q + ((size_t)b * p.QH + kvh * p.G + gg) * p.HD + 16 * j + 2 * tt;
          const float x[4] = {qr[0], qr[1], qr[8], qr[9]};
          uint16_t h[4], l[4];
#pragma unroll
          for (int k = 0; k < 4; k++) {
            const __half hh = __float2half_rn(x[k]);
            h[k] = __half_as_ushort(hh);
            l[k] = f2h(x[k] - __half2float(hh));
          }
          v = make_uint4(pack_h2(h[0], h[1]), pack_h2(h[2], h[3]), pack_h2(l[0], l[1]), pack_h2(l[2], l[3]));
        }
        qf[i] = v;
      }
      qb = b;
      qk = kvh;
      group_sync(grp);
    }
    // this item issued into its stage (so the stage's previous load is consumed),
    // then the stage's phase local / kAS complete
    if (ok) ok = bounded_spin([&] { return ld_acquire_cta(&issued[s]) >= it; }, p.status, p.wait_ns);
    if (ok) {
      const uint32_t par = (uint32_t)((local / kAS) & 1);
      ok = bounded_spin([&] { return mbar_try_wait(&full[s], par); }, p.status, p.wait_ns);
    }
    const uint8_t* Kt = kv + (size_t)s * 2 * tile;
    const uint8_t* Vt = p.keqv ? Kt : Kt + tile;
    // ---- scores of this warp's 16 slots x the group's heads
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
    if (ok) {
      // four independent accumulation chains over the dims, summed in a fixed order
      float sp[4][4];
#pragma unroll
      for (int u = 0; u < 4; u++) sp[u][0] = sp[u][1] = sp[u][2] = sp[u][3] = 0.f;
      for (int j0 = 0; j0 < p.HD / 16; j0 += 4) {
        const uint8_t* kb = Kt + (j0 >> 2) * kSub;
#pragma unroll
        for (int u = 0; u < 4; u++) {
          const int j = j0 + u;
          const uint32_t a0 = *reinterpret_cast<const uint32_t*>(kb + koff[2 * u]);
          const uint32_t a1 = *reinterpret_cast<const uint32_t*>(kb + koff[2 * u] + 1024);
          const uint32_t a2 = *reinterpret_cast<const uint32_t*>(kb + koff[2 * u + 1]);
          const uint32_t a3 = *reinterpret_cast<const uint32_t*>(kb + koff[2 * u + 1] + 1024);
          const uint4 qv = qf[j * 32 + lane];
          mma16816(sp[u], a0, a1, a2, a3, qv.x, qv.y);
          mma16816(sp[u], a0, a1, a2, a3, qv.z, qv.w);
        }
      }
#pragma unroll
      for (int r = 0; r < 4; r++) sc[r] = (sp[0][r] + sp[1][r]) + (sp[2][r] + sp[3][r]);
    }
    // sc: [0] (slot g, head 2t) [1] (slot g, head 2t+1) [2] (slot g+8, head 2t) [3] (slot g+8, head 2t+1)
    const uint32_t sa = t0 + 16 * wg + g, sb = sa + 8;
    const bool va = sa < n && rule.valid(sa), vb = sb < n && rule.valid(sb);
    float s0 = va ? sc[0] * p.scale : -INFINITY, s1 = va ? sc[1] * p.scale : -INFINITY;
    float s2 = vb ? sc[2] * p.scale : -INFINITY, s3 = vb ? sc[3] * p.scale : -INFINITY;
    float m0 = fmaxf(s0, s2), m1 = fmaxf(s1, s3);
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
      m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, o));
    }
    if (g == 0) {
      red_m[grp][wg][2 * t] = m0;
      red_m[grp][wg][2 * t + 1] = m1;
    }
    group_sync(grp);
    float M0 = red_m[grp][0][2 * t], M1 = red_m[grp][0][2 * t + 1];
#pragma unroll
    for (int w = 1; w < kAW; w++) {
      M0 = fmaxf(M0, red_m[grp][w][2 * t]);
      M1 = fmaxf(M1, red_m[grp][w][2 * t + 1]);
    }
    const float p0 = (va && M0 != -INFINITY) ? expf(s0 - M0) : 0.f;
    const float p1 = (va && M1 != -INFINITY) ? expf(s1 - M1) : 0.f;
    const float p2 = (vb && M0 != -INFINITY) ? expf(s2 - M0) : 0.f;
    const float p3 = (vb && M1 != -INFINITY) ? expf(s3 - M1) : 0.f;
    float l0 = p0 + p2, l1 = p1 + p3;
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, o);
      l1 += __shfl_xor_sync(0xffffffffu, l1, o);
    }
    if (g == 0) {
      red_l[grp][wg][2 * t] = l0;
      red_l[grp][wg][2 * t + 1] = l1;
    }
    // p as f16 hi + lo, [head][slot] (heads >= G keep their zeros)
    {
      const int la = 16 * wg + g, lb = la + 8;
      const float pv[4] = {p0, p1, p2, p3};
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const int head = 2 * t + (k & 1), slot = (k & 2) ? lb : la;
        if (head < p.G) {
          const __half hh = __float2half_rn(pv[k]);
          ph[head * kPP + slot] = __half_as_ushort(hh);
          pl[head * kPP + slot] = f2h(pv[k] - __half2float(hh));
        }
      }
    }
    group_sync(grp);
    // ---- O^T[d][head] for this warp's d tiles
    const size_t part_row = (size_t)b * p.QH + kvh * p.G;
    if (ok) {
      // this warp's d tiles interleaved: independent accumulators
      float acc[4][4];
#pragma unroll
      for (int u = 0; u < 4; u++) acc[u][0] = acc[u][1] = acc[u][2] = acc[u][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < kAC / 16; ks++) {
        const uint16_t* bh = ph + g * kPP + 16 * ks + 2 * t;
        const uint16_t* bl = pl + g * kPP + 16 * ks + 2 * t;
        const uint32_t h0 = lds32(bh), h1 = lds32(bh + 8), l0 = lds32(bl), l1 = lds32(bl + 8);
#pragma unroll
        for (int u = 0; u < 4; u++) {
          if (u >= dtiles) break;
          uint32_t a0, a1, a2, a3;
          ldsm_x4_trans(a0, a1, a2, a3, Vt + voff[u] + ks * 16 * 128);
          mma16816(acc[u], a0, a1, a2, a3, h0, h1);
          mma16816(acc[u], a0, a1, a2, a3, l0, l1);
        }
      }
      // acc[u]: [0] (d g, head 2t) [1] (d g, head 2t+1) [2] (d g+8, head 2t) [3] (d g+8, head 2t+1)
      const size_t hstride = (size_t)p.max_chunks * p.HD;
      float* o0 = p.part_o + ((part_row + 2 * t) * p.max_chunks + c) * p.HD + 16 * wg * dtiles + g;
#pragma unroll
      for (int u = 0; u < 4; u++) {
        if (u >= dtiles) break;
        if (2 * t < p.G) {
          o0[16 * u] = acc[u][0];
          o0[16 * u + 8] = acc[u][2];
        }
        if (2 * t + 1 < p.G) {
          o0[hstride + 16 * u] = acc[u][1];
          o0[hstride + 16 * u + 8] = acc[u][3];
        }
      }
    }
    if (wg == 0 && g == 0 && ok) {
      float L0 = 0.f, L1 = 0.f;
#pragma unroll
      for (int w = 0; w < kAW; w++) {
        L0 += red_l[grp][w][2 * t];
        L1 += red_l[grp][w][2 * t + 1];
      }
      if (2 * t < p.G) {
        float* ml = p.part_ml + ((part_row + 2 * t) * p.max_chunks + c) * 2;
        ml[0] = L0 > 0.f ? M0 : -INFINITY;
        ml[1] = L0;
      }
      if (2 * t + 1 < p.G) {
        float* ml = p.part_ml + ((part_row + 2 * t + 1) * p.max_chunks + c) * 2;
        ml[0] = L1 > 0.f ? M1 : -INFINITY;
        ml[1] = L1;
      }
    }
    // every warp of the group is done with this stage, its p rows and q fragments
    group_sync(grp);
    if (gtid == 0 && ok && it + kAS < i1) issue(it + kAS);
  }
  // After a time-out some issued loads may not have been consumed: let them land
  // (bounded) before the CTA's shared memory is released.  On the normal path
  // every issued item was consumed and these waits pass at once.
  __syncthreads();
  if (threadIdx.x == 0)
    for (int s = 0; s < kAS; s++) {
      const int last = issued[s];
      if (last < 0) continue;
      const uint32_t par = (uint32_t)(((last - i0) / kAS) & 1);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&full[s], par) && globaltimer_ns() - t0 < p.wait_ns) {
      }
    }
}

// Phase B over the live chunks: out[h][d] = sum_c o_c e^(m_c - M) / sum_c l_c e^(m_c - M).
// The chunk weights e^(m_c - M) are formed once per head in shared memory; the
// sums over chunks then issue independent loads (same order and arithmetic).
__global__ void k_attcomb_dec(const AttP p, uint16_t* __restrict__ out_h, int xfo) {
  pdl_wait();
  extern __shared__ float wc[];            // [max_chunks]
  __shared__ float sh[32];
  const SlotRule rule = att_rule(p);
  const int nch = min((int)((rule.nslots() + kAC - 1) / kAC), p.max_chunks);
  const int c_lo = min(first_chunk(rule), nch);
  const int h = blockIdx.x, b = blockIdx.y;
  const size_t row = (size_t)b * p.QH + h;
  const float* ml = p.part_ml + row * p.max_chunks * 2;
  float m = -INFINITY;
  for (int c = c_lo + threadIdx.x; c < nch; c += blockDim.x)
    if (ml[2 * c + 1] > 0.f) m = fmaxf(m, ml[2 * c]);
  const float M = block_max(m, sh);
  for (int c = c_lo + threadIdx.x; c < nch; c += blockDim.x)
    wc[c] = ml[2 * c + 1] > 0.f ? expf(ml[2 * c] - M) : 0.f;
  __syncthreads();
  float den = 0.f;                          // in chunk order, as a single thread would
  for (int c = c_lo; c < nch; c++)
    if (ml[2 * c + 1] > 0.f) den += ml[2 * c + 1] * wc[c];
  uint16_t* out = out_h + (size_t)b * p.QH * p.HD;
  const float* po = p.part_o + row * p.max_chunks * p.HD;
  // four dims per thread (HD % 4 == 0), sixteen chunks' loads in flight
  for (int d = 4 * (int)threadIdx.x; d < p.HD; d += 4 * (int)blockDim.x) {
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    for (int c = c_lo; c < nch; c += 16) {
      float4 o[16];
#pragma unroll
      for (int u = 0; u < 16; u++)
        o[u] = c + u < nch && wc[c + u] != 0.f ? *reinterpret_cast<const float4*>(po + (size_t)(c + u) * p.HD + d)
                                                : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < 16; u++)
        if (c + u < nch && wc[c + u] != 0.f) {
          const float w = wc[c + u];
          a0 = fmaf(o[u].x, w, a0);
          a1 = fmaf(o[u].y, w, a1);
          a2 = fmaf(o[u].z, w, a2);
          a3 = fmaf(o[u].w, w, a3);
        }
    }
    const float r[4] = {a0, a1, a2, a3};
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const int i = h * p.HD + d + e;
      out[xfo ? xfo_pos(i) : i] = f2h(den > 0.f ? r[e] / den : 0.f);
    }
  }
}

// ---------------------------------------------------------------- prefill
// Causal attention of a batched-prefill chunk: npos consecutive positions of
// nseq sequences (rows position-major, row = p * nseq + b) whose K/V rows are
// already in the caches (e4b_headprep_rows), as the reference's prefill runs
// its attention per prompt token (src/engine-a4b.js:478-479).  Work item =
// (sequence, KV head, block of kPC / G positions): the block's G heads x
// positions are the 64 MMA columns, so every K/V tile is read once per block
// instead of once per query.  Online softmax over the live 64-slot chunks
// with f32 running (max, sum) per column; the products are k_attdec's (f16
// K/V x f16 hi + lo q and p, f32 sums).
constexpr int kPC = 64;                  // query columns per item
constexpr int kPW = 4;                   // warps per CTA

struct PreP {
  const float* q;                        // [npos * nseq][QH][HD]
  const uint32_t* params;                // the chunk's first position (src/engine-a4b.js:697 layout)
  uint16_t* out;                         // [npos * nseq][QH * HD] f16
  uint32_t* status;
  int QH, KVH, HD, G, window, cachemode, ring, nseq, npos, keqv, pb;
  float scale;
  uint64_t wait_ns;
};

struct PreItem {
  int b, kvh, p0, np, c0, c1;
};
E4B_DEV PreItem pre_item(const PreP& p, int it) {
  const int nqb = (p.npos + p.pb - 1) / p.pb;
  PreItem I;
  I.b = it / (p.KVH * nqb);
  const int rem = it % (p.KVH * nqb);
  I.kvh = rem / nqb;
  const int qb = rem % nqb;
  I.p0 = qb * p.pb;
  I.np = min(p.pb, p.npos - I.p0);
  const uint32_t qp_last = p.params[0] + (uint32_t)(I.p0 + I.np - 1);
  const uint32_t len0 = p.cachemode == 2 ? p.params[5] : p.params[1];
  if (p.cachemode == 1) {
    I.c0 = 0;
    I.c1 = (int)((min(qp_last + 1, (uint32_t)p.ring) + kAC - 1) / kAC);
  } else {
    const uint32_t len_first = len0 + (uint32_t)I.p0, len_last = len0 + (uint32_t)(I.p0 + I.np - 1);
    I.c0 = (p.cachemode == 0 && p.window > 0 && len_first > (uint32_t)p.window)
               ? (int)((len_first - (uint32_t)p.window) / kAC) : 0;
    I.c1 = (int)((len_last + kAC - 1) / kAC);
  }
  I.c1 = max(I.c1, I.c0 + 1);         // every item consumes at least one load (issuer and consumers agree)
  return I;
}

__global__ void __launch_bounds__(32 * kPW, 1) k_attpre(const PreP p, const __grid_constant__ CUtensorMap kmap,
                                                        const __grid_constant__ CUtensorMap vmap) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[2];
  __shared__ float red_m[kPW][kPC], red_l[kPW][kPC], m_run[kPC], l_run[kPC];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int tile = (p.HD / 64) * kSub;
  uint8_t* kv = smem + ((1024u - (smem_u32(smem) & 1023u)) & 1023u);          // [2 stages][K tile | V tile]
  uint4* qf = reinterpret_cast<uint4*>(kv + (size_t)2 * 2 * tile);            // [(HD/16) * 8 n-tiles][32 lanes]
  uint16_t* ph = reinterpret_cast<uint16_t*>(qf + (size_t)(p.HD / 16) * 8 * 32);   // [kPC][kPP] hi
  uint16_t* pl = ph + kPC * kPP;                                                    // lo
  if (threadIdx.x == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&kmap)) : "memory");
    if (!p.keqv) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&vmap)) : "memory");
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    fence_barrier_init();
  }
  __syncthreads();
  pdl_trigger();
  pdl_wait();
  const int nqb = (p.npos + p.pb - 1) / p.pb;
  const int items = p.nseq * p.KVH * nqb;
  const uint32_t len0 = p.cachemode == 2 ? p.params[5] : p.params[1];
  const uint32_t qp0 = p.params[0];

  // thread 0 issues the K/V loads of this CTA's (item, chunk) sequence, two ahead
  int is_it = blockIdx.x, is_c = 0, is_c1 = 0;
  uint32_t n_issued = 0;
  if (threadIdx.x == 0 && is_it < items) {
    const PreItem I = pre_item(p, is_it);
    is_c = I.c0;
    is_c1 = I.c1;
  }
  auto issue_next = [&]() {
    if (is_it >= items) return;
    const PreItem I = pre_item(p, is_it);
    const int st = n_issued & 1;
    uint8_t* dk = kv + (size_t)st * 2 * tile;
    mbar_expect_tx(&full[st], (uint32_t)tile * (p.keqv ? 1u : 2u));
    for (int j = 0; j < p.HD / 64; j++) {
      tma_load_4d(dk + j * kSub, &kmap, 64 * j, I.kvh, is_c * kAC, I.b, &full[st]);
      if (!p.keqv) tma_load_4d(dk + tile + j * kSub, &vmap, 64 * j, I.kvh, is_c * kAC, I.b, &full[st]);
    }
    n_issued++;
    if (++is_c >= is_c1) {
      is_it += gridDim.x;
      if (is_it < items) {
        const PreItem J = pre_item(p, is_it);
        is_c = J.c0;
        is_c1 = J.c1;
      }
    }
  };
  if (threadIdx.x == 0) {
    issue_next();
    issue_next();
  }

  const int r0 = 16 * warp + g;
  uint32_t koff[8];
#pragma unroll
  for (int u = 0; u < 8; u++) koff[u] = (uint32_t)(r0 * 128 + ((u ^ g) << 4) + 4 * t);
  const int dtiles = p.HD / 16 / kPW;           // 1..4
  const int lrow = (lane & 7) + ((lane >> 4) << 3), hbit = (lane >> 3) & 1;
  uint32_t voff[4];
#pragma unroll
  for (int u = 0; u < 4; u++) {
    const int dt = warp * dtiles + u;
    voff[u] = (uint32_t)((dt >> 2) * kSub + lrow * 128 + (((2 * (dt & 3) + hbit) ^ (lane & 7)) << 4));
  }
  bool ok = true;
  uint32_t L = 0;                                 // loads consumed
  for (int it = blockIdx.x; it < items; it += gridDim.x) {
    const PreItem I = pre_item(p, it);
    // q fragments of the 64 columns (col = position-in-block * G + head-in-group), hi and lo
    for (int i = threadIdx.x; i < (p.HD / 16) * 8 * 32; i += 32 * kPW) {
      const int j = i >> 8, nt = (i >> 5) & 7, gg = (i & 31) >> 2, tt = i & 3;
      const int col = 8 * nt + gg, pp = col / p.G, gi = col % p.G;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (pp < I.np) {
        const size_t row = (size_t)(I.p0 + pp) * p.nseq + I.b;
        const float* qr = p.q + (row * p.QH + I.kvh * p.G + gi) * p.HD + 16 * j + 2 * tt;
        const float x[4] = {qr[0], qr[1], qr[8], qr[9]};
        uint16_t h[4], l[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
          const __half hh = __float2half_rn(x[k]);
          h[k] = __half_as_ushort(hh);
          l[k] = f2h(x[k] - __half2float(hh));
        }
        v = make_uint4(pack_h2(h[0], h[1]), pack_h2(h[2], h[3]), pack_h2(l[0], l[1]), pack_h2(l[2], l[3]));
      }
      qf[i] = v;
    }
    if (threadIdx.x < kPC) {
      m_run[threadIdx.x] = -INFINITY;
      l_run[threadIdx.x] = 0.f;
    }
    float acc[4][8][4];
#pragma unroll
    for (int u = 0; u < 4; u++)
#pragma unroll
      for (int nt = 0; nt < 8; nt++) acc[u][nt][0] = acc[u][nt][1] = acc[u][nt][2] = acc[u][nt][3] = 0.f;
    // per column of this lane (n-tile nt, column 8 nt + 2 t + e): the query's slot rule
    __syncthreads();
    for (int c = I.c0; c < I.c1; c++, L++) {
      const int st = L & 1;
      if (ok) ok = bounded_spin([&] { return mbar_try_wait(&full[st], (L >> 1) & 1u); }, p.status, p.wait_ns);
      const uint8_t* Kt = kv + (size_t)st * 2 * tile;
      const uint8_t* Vt = p.keqv ? Kt : Kt + tile;
      // ---- S^T[slot][col] for this warp's 16 slots
      float sc[8][4];
#pragma unroll
      for (int nt = 0; nt < 8; nt++) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
      if (ok) {
        for (int j0 = 0; j0 < p.HD / 16; j0 += 4) {
          const uint8_t* kb = Kt + (j0 >> 2) * kSub;
#pragma unroll
          for (int u = 0; u < 4; u++) {
            const int j = j0 + u;
            const uint32_t a0 = *reinterpret_cast<const uint32_t*>(kb + koff[2 * u]);
            const uint32_t a1 = *reinterpret_cast<const uint32_t*>(kb + koff[2 * u] + 1024);
            const uint32_t a2 = *reinterpret_cast<const uint32_t*>(kb + koff[2 * u + 1]);
            const uint32_t a3 = *reinterpret_cast<const uint32_t*>(kb + koff[2 * u + 1] + 1024);
#pragma unroll
            for (int nt = 0; nt < 8; nt++) {
              const uint4 qv = qf[(j * 8 + nt) * 32 + lane];
              mma16816(sc[nt], a0, a1, a2, a3, qv.x, qv.y);
              mma16816(sc[nt], a0, a1, a2, a3, qv.z, qv.w);
            }
          }
        }
      }
      // ---- mask, column maxima
      const uint32_t sa = (uint32_t)c * kAC + 16 * warp + g, sb = sa + 8;
#pragma unroll
      for (int nt = 0; nt < 8; nt++) {
#pragma unroll
        for (int e = 0; e < 2; e++) {
          const int col = 8 * nt + 2 * t + e, pp = col / p.G;
          SlotRule r{p.cachemode, p.ring, p.window, qp0 + (uint32_t)(I.p0 + pp), len0 + (uint32_t)(I.p0 + pp)};
          const uint32_t n = r.nslots();
          const bool live = pp < I.np && ok;
          const bool va = live && sa < n && r.valid(sa), vb = live && sb < n && r.valid(sb);
          sc[nt][e] = va ? sc[nt][e] * p.scale : -INFINITY;
          sc[nt][2 + e] = vb ? sc[nt][2 + e] * p.scale : -INFINITY;
        }
        float m0 = fmaxf(sc[nt][0], sc[nt][2]), m1 = fmaxf(sc[nt][1], sc[nt][3]);
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
          m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, o));
        }
        if (g == 0) {
          red_m[warp][8 * nt + 2 * t] = m0;
          red_m[warp][8 * nt + 2 * t + 1] = m1;
        }
      }
      __syncthreads();
      // ---- new running max, p = e^(s - M), rescale factors
      float alpha[8][2];
#pragma unroll
      for (int nt = 0; nt < 8; nt++) {
        float l0 = 0.f, l1 = 0.f;
#pragma unroll
        for (int e = 0; e < 2; e++) {
          const int col = 8 * nt + 2 * t + e;
          float M = red_m[0][col];
#pragma unroll
          for (int w = 1; w < kPW; w++) M = fmaxf(M, red_m[w][col]);
          const float mo = m_run[col];
          const float Mn = fmaxf(mo, M);
          alpha[nt][e] = (mo == -INFINITY) ? 0.f : expf(mo - Mn);
          const float pa = (sc[nt][e] == -INFINITY) ? 0.f : expf(sc[nt][e] - Mn);
          const float pb2 = (sc[nt][2 + e] == -INFINITY) ? 0.f : expf(sc[nt][2 + e] - Mn);
          const int la = 16 * warp + g, lb = la + 8;
          const __half ha = __float2half_rn(pa), hb = __float2half_rn(pb2);
          ph[col * kPP + la] = __half_as_ushort(ha);
          pl[col * kPP + la] = f2h(pa - __half2float(ha));
          ph[col * kPP + lb] = __half_as_ushort(hb);
          pl[col * kPP + lb] = f2h(pb2 - __half2float(hb));
          if (e == 0) l0 = pa + pb2;
          else l1 = pa + pb2;
        }
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          l0 += __shfl_xor_sync(0xffffffffu, l0, o);
          l1 += __shfl_xor_sync(0xffffffffu, l1, o);
        }
        if (g == 0) {
          red_l[warp][8 * nt + 2 * t] = l0;
          red_l[warp][8 * nt + 2 * t + 1] = l1;
        }
      }
      __syncthreads();
      if (threadIdx.x < kPC) {
        const int col = threadIdx.x;
        float M = red_m[0][col];
        for (int w = 1; w < kPW; w++) M = fmaxf(M, red_m[w][col]);
        const float mo = m_run[col], Mn = fmaxf(mo, M);
        const float al = (mo == -INFINITY) ? 0.f : expf(mo - Mn);
        float ls = 0.f;
        for (int w = 0; w < kPW; w++) ls += red_l[w][col];
        l_run[col] = l_run[col] * al + ls;
        m_run[col] = Mn;
      }
      // ---- O^T[d][col] = alpha O^T + V^T P^T for this warp's d tiles
      if (ok) {
#pragma unroll
        for (int u = 0; u < 4; u++)
#pragma unroll
          for (int nt = 0; nt < 8; nt++) {
            acc[u][nt][0] *= alpha[nt][0];
            acc[u][nt][1] *= alpha[nt][1];
            acc[u][nt][2] *= alpha[nt][0];
            acc[u][nt][3] *= alpha[nt][1];
          }
#pragma unroll
        for (int ks = 0; ks < kAC / 16; ks++) {
          uint32_t bh[8][2], bl[8][2];
#pragma unroll
          for (int nt = 0; nt < 8; nt++) {
            const uint16_t* rh = ph + (8 * nt + g) * kPP + 16 * ks + 2 * t;
            const uint16_t* rl = pl + (8 * nt + g) * kPP + 16 * ks + 2 * t;
            bh[nt][0] = lds32(rh);
            bh[nt][1] = lds32(rh + 8);
            bl[nt][0] = lds32(rl);
            bl[nt][1] = lds32(rl + 8);
          }
#pragma unroll
          for (int u = 0; u < 4; u++) {
            if (u >= dtiles) break;
            uint32_t a0, a1, a2, a3;
            ldsm_x4_trans(a0, a1, a2, a3, Vt + voff[u] + ks * 16 * 128);
#pragma unroll
            for (int nt = 0; nt < 8; nt++) {
              mma16816(acc[u][nt], a0, a1, a2, a3, bh[nt][0], bh[nt][1]);
              mma16816(acc[u][nt], a0, a1, a2, a3, bl[nt][0], bl[nt][1]);
            }
          }
        }
      }
      __syncthreads();                          // stage and p rows free
      if (threadIdx.x == 0 && ok) issue_next();
    }
    // ---- out = O / l (f16), rows (position, sequence), head kvh * G + head-in-group
    if (ok) {
#pragma unroll
      for (int nt = 0; nt < 8; nt++)
#pragma unroll
        for (int e = 0; e < 2; e++) {
          const int col = 8 * nt + 2 * t + e, pp = col / p.G, gi = col % p.G;
          if (pp >= I.np) continue;
          const float l = l_run[col];
          const float inv = l > 0.f ? 1.f / l : 0.f;
          uint16_t* o = p.out + ((size_t)(I.p0 + pp) * p.nseq + I.b) * (size_t)p.QH * p.HD +
                        (size_t)(I.kvh * p.G + gi) * p.HD + 16 * warp * dtiles + g;
#pragma unroll
          for (int u = 0; u < 4; u++) {
            if (u >= dtiles) break;
            o[16 * u] = f2h(acc[u][nt][e] * inv);
            o[16 * u + 8] = f2h(acc[u][nt][2 + e] * inv);
          }
        }
    }
    __syncthreads();                            // m_run / l_run / qf reused by the next item
  }
  // loads issued but not consumed (only after a time-out) land before the CTA ends
  if (threadIdx.x == 0)
    for (uint32_t k = L; k < n_issued; k++) {
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&full[k & 1], (k >> 1) & 1u) && globaltimer_ns() - t0 < p.wait_ns) {
      }
    }
}

}  // namespace

extern "C" {

E4B_API int e4b_attdec_seq(e4b_ctx* c, const float* q, const uint16_t* kcache, const uint16_t* vcache,
                           const uint32_t* params, float* part_o, float* part_ml, uint16_t* out_h, int QH, int KVH,
                           int HD, int window, int cachemode, int ring, int max_chunks, float scale, int cache_slots,
                           int nseq, int xfo) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, q && kcache && vcache && params && part_o && part_ml && out_h && nseq > 0 && cache_slots > 0,
              "attdec_seq: bad args");
  E4B_REQUIRE(c, QH > 0 && KVH > 0 && QH % KVH == 0 && QH / KVH <= 8, "attdec_seq: %d query heads per KV head (max 8)",
              KVH > 0 ? QH / KVH : 0);
  E4B_REQUIRE(c, HD % 64 == 0 && HD <= 256, "attdec_seq: HD=%d must be a multiple of 64 up to 256", HD);
  E4B_REQUIRE(c, cachemode >= 0 && cachemode <= 2 && (cachemode != 1 || (ring > 0 && window > 0 && ring <= cache_slots)),
              "attdec_seq: bad cache mode");
  const int scan = cachemode == 1 ? ring : cache_slots;
  E4B_REQUIRE(c, (long long)max_chunks * kAC >= scan, "attdec_seq: max_chunks=%d < %d slots / %d", max_chunks, scan,
              kAC);
  E4B_REQUIRE(c, reinterpret_cast<uintptr_t>(kcache) % 16 == 0 && reinterpret_cast<uintptr_t>(vcache) % 16 == 0,
              "attdec_seq: caches must be 16-byte aligned");
  E4B_REQUIRE(c, !xfo || (QH * HD) % 32 == 0, "attdec_seq: fragment order needs QH*HD %% 32 == 0");
  AttP p = {};
  p.q = q; p.kc = kcache; p.vc = vcache; p.params = params; p.part_o = part_o; p.part_ml = part_ml;
  p.status = c->status;
  p.QH = QH; p.KVH = KVH; p.HD = HD; p.G = QH / KVH; p.window = window; p.cachemode = cachemode; p.ring = ring;
  p.max_chunks = max_chunks; p.nseq = nseq; p.keqv = kcache == vcache; p.scale = scale;
  p.seq_stride = (size_t)cache_slots * KVH * HD;
  p.wait_ns = c->wait_ns;
  CUtensorMap kmap, vmap;
  E4B_REQUIRE(c, cache_map(&kmap, kcache, HD, KVH, cache_slots, nseq), "attdec_seq: K cache tensor map failed");
  if (p.keqv) vmap = kmap;
  else E4B_REQUIRE(c, cache_map(&vmap, vcache, HD, KVH, cache_slots, nseq), "attdec_seq: V cache tensor map failed");
  const size_t smem = (size_t)kAS * 2 * (HD / 64) * kSub + (size_t)kAG * ((size_t)(HD / 16) * 32 * 16 + 2 * 8 * kPP * 2) +
                      1024;
  cudaError_t e = cudaFuncSetAttribute(k_attdec, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e4b_fail(c, E4B_ECUDA, "attdec smem attr: %s", cudaGetErrorString(e));
  const long long most = (long long)nseq * KVH * max_chunks;
  const int cap = c->attn_grid_cap > 0 ? c->attn_grid_cap : c->sm_count;
  const int grid = (int)(most < cap ? most : cap);
  if (int r = e4b_launch(c, "attdec", k_attdec, dim3(grid), dim3(32 * kAW * kAG), smem, p, kmap, vmap)) return r;
  // one thread per four dims of a head
  const int comb_threads = std::max(32, (HD / 4 + 31) / 32 * 32);
  return e4b_launch(c, "attcomb_dec", k_attcomb_dec, dim3(QH, nseq), dim3(comb_threads), (size_t)max_chunks * 4, p, out_h,
                    xfo);
}

E4B_API int e4b_attn_prefill(e4b_ctx* c, const float* q, const uint16_t* kcache, const uint16_t* vcache,
                             const uint32_t* params, uint16_t* out, int QH, int KVH, int HD, int window, int cachemode,
                             int ring, float scale, int cache_slots, int nseq, int npos) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, q && kcache && vcache && params && out && nseq > 0 && npos > 0 && cache_slots > 0,
              "attn_prefill: bad args");
  E4B_REQUIRE(c, QH > 0 && KVH > 0 && QH % KVH == 0 && (QH / KVH) <= kPC && kPC % (QH / KVH) == 0,
              "attn_prefill: %d query heads per KV head (must divide %d)", KVH > 0 ? QH / KVH : 0, kPC);
  E4B_REQUIRE(c, HD % 64 == 0 && HD <= 256, "attn_prefill: HD=%d must be a multiple of 64 up to 256", HD);
  E4B_REQUIRE(c, cachemode >= 0 && cachemode <= 2 && (cachemode != 1 || (ring > 0 && window > 0 && ring <= cache_slots)),
              "attn_prefill: bad cache mode");
  E4B_REQUIRE(c, cachemode != 1 || npos + window <= ring + 1,
              "attn_prefill: %d positions per chunk overwrite ring slots still in a window (ring %d, window %d)", npos,
              ring, window);
  E4B_REQUIRE(c, reinterpret_cast<uintptr_t>(kcache) % 16 == 0 && reinterpret_cast<uintptr_t>(vcache) % 16 == 0,
              "attn_prefill: caches must be 16-byte aligned");
  PreP p = {};
  p.q = q; p.params = params; p.out = out; p.status = c->status;
  p.QH = QH; p.KVH = KVH; p.HD = HD; p.G = QH / KVH; p.window = window; p.cachemode = cachemode; p.ring = ring;
  p.nseq = nseq; p.npos = npos; p.keqv = kcache == vcache; p.pb = kPC / p.G; p.scale = scale; p.wait_ns = c->wait_ns;
  CUtensorMap kmap, vmap;
  E4B_REQUIRE(c, cache_map(&kmap, kcache, HD, KVH, cache_slots, nseq), "attn_prefill: K cache tensor map failed");
  if (p.keqv) vmap = kmap;
  else E4B_REQUIRE(c, cache_map(&vmap, vcache, HD, KVH, cache_slots, nseq), "attn_prefill: V cache tensor map failed");
  const size_t smem = 1024 + (size_t)2 * 2 * (HD / 64) * kSub + (size_t)(HD / 16) * 8 * 32 * 16 + (size_t)2 * kPC * kPP * 2;
  cudaError_t e = cudaFuncSetAttribute(k_attpre, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e4b_fail(c, E4B_ECUDA, "attn_prefill smem attr: %s", cudaGetErrorString(e));
  const long long items = (long long)nseq * KVH * ((npos + p.pb - 1) / p.pb);
  const int grid = (int)(items < c->sm_count ? items : c->sm_count);
  return e4b_launch(c, "attn_prefill", k_attpre, dim3(grid), dim3(32 * kPW), smem, p, kmap, vmap);
}

}  // extern "C"
