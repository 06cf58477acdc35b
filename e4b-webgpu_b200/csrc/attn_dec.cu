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
  for (int d = threadIdx.x; d < p.HD; d += blockDim.x) {
    float acc = 0.f;
    int c = c_lo;
    for (; c + 8 <= nch; c += 8) {
      float o[8];
#pragma unroll
      for (int u = 0; u < 8; u++) o[u] = wc[c + u] != 0.f ? po[(size_t)(c + u) * p.HD + d] : 0.f;
#pragma unroll
      for (int u = 0; u < 8; u++)
        if (wc[c + u] != 0.f) acc = fmaf(o[u], wc[c + u], acc);
    }
    for (; c < nch; c++)
      if (wc[c] != 0.f) acc = fmaf(po[(size_t)c * p.HD + d], wc[c], acc);
    const float v = den > 0.f ? acc / den : 0.f;
    const int i = h * p.HD + d;
    out[xfo ? xfo_pos(i) : i] = f2h(v);
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
  return e4b_launch(c, "attcomb_dec", k_attcomb_dec, dim3(QH, nseq), dim3(128), (size_t)max_chunks * 4, p, out_h,
                    xfo);
}

}  // extern "C"
