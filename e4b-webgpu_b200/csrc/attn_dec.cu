// Batched split-KV decode attention on the tensor cores (kernels/attsplit.wgsl
// + attcomb.wgsl semantics for nseq sequences at one common position).
//
// Work item = (sequence, KV head, chunk of 64 cache slots); only chunks that
// hold live slots are visited, by a persistent grid.  Per item the CTA
// bulk-copies the chunk's K and V rows (one 512-byte copy per row, into a
// padded shared-memory layout) two items ahead of use, and does both products
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
#include "stream.cuh"

namespace {
using namespace e4b;

constexpr int kAC = 64;            // slots per chunk
constexpr int kAW = 4;             // warps per CTA
constexpr int kPP = kAC + 8;       // padded p row (halves)

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
  int kpitch;                      // halves per staged K / V row (HD + 8)
};

E4B_DEV void ldsm_x4_trans(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* ptr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(ptr)));
}
E4B_DEV uint32_t lds32(const uint16_t* ptr) { return *reinterpret_cast<const uint32_t*>(ptr); }

E4B_DEV SlotRule att_rule(const AttP& p) {
  SlotRule r{p.cachemode, p.ring, p.window, 0, 0};
  r.qp = p.params[0];
  r.len = p.cachemode == 2 ? p.params[5] : p.params[1];
  return r;
}

__global__ void __launch_bounds__(32 * kAW, 1) k_attdec(const AttP p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[2];
  __shared__ float red_m[kAW][8], red_l[kAW][8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int tile = kAC * p.kpitch;                                 // halves per K or V tile
  uint16_t* kv = reinterpret_cast<uint16_t*>(smem);                // [2 stages][K tile | V tile]
  uint4* qf = reinterpret_cast<uint4*>(smem + (size_t)4 * tile * 2);   // [HD/16][32 lanes]
  uint16_t* ph = reinterpret_cast<uint16_t*>(qf + (p.HD / 16) * 32);   // [8 heads][kPP] p hi
  uint16_t* pl = ph + 8 * kPP;                                     // p lo
  // stale rows only ever meet p = 0; start them at zero so 0 * x stays 0
  for (int i = threadIdx.x; i < 4 * tile / 8; i += blockDim.x) reinterpret_cast<uint4*>(kv)[i] = make_uint4(0, 0, 0, 0);
  for (int i = threadIdx.x; i < 2 * 8 * kPP; i += blockDim.x) ph[i] = 0;
  if (threadIdx.x == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    fence_barrier_init();
  }
  fence_proxy_async();
  __syncthreads();
  pdl_trigger();
  pdl_wait();
  const SlotRule rule = att_rule(p);
  const uint32_t n = rule.nslots();
  const int nch = (int)((n + kAC - 1) / kAC);
  if (nch > p.max_chunks) {
    if (threadIdx.x == 0) set_status(p.status, E4B_ST_BADINDEX);
    return;
  }
  const int per_seq = p.KVH * nch, items = p.nseq * per_seq;

  auto issue = [&](int it, int s) {
    const int b = it / per_seq, rem = it % per_seq, kvh = rem / nch, c = rem % nch;
    const uint32_t t0 = (uint32_t)c * kAC;
    const int rows = (int)min((uint32_t)kAC, n - t0);
    const uint32_t row_bytes = (uint32_t)p.HD * 2;
    if (lane == 0) mbar_expect_tx(&full[s], (uint32_t)rows * row_bytes * (p.keqv ? 1u : 2u));
    __syncwarp();
    uint16_t* dk = kv + (size_t)s * 2 * tile;
    for (int r = lane; r < rows; r += 32) {
      const size_t off = (size_t)b * p.seq_stride + ((size_t)(t0 + r) * p.KVH + kvh) * p.HD;
      bulk_g2s(dk + r * p.kpitch, p.kc + off, row_bytes, &full[s]);
      if (!p.keqv) bulk_g2s(dk + tile + r * p.kpitch, p.vc + off, row_bytes, &full[s]);
    }
  };
  if (warp == 0) {
    if ((int)blockIdx.x < items) issue(blockIdx.x, 0);
    if ((int)(blockIdx.x + gridDim.x) < items) issue(blockIdx.x + gridDim.x, 1);
  }

  bool ok = true;
  int local = 0;
  for (int it = blockIdx.x; it < items; it += gridDim.x, local++) {
    const int s = local & 1;
    const int b = it / per_seq, rem = it % per_seq, kvh = rem / nch, c = rem % nch;
    const uint32_t t0 = (uint32_t)c * kAC;
    // q fragments of the group's heads: (q[k], q[k+1]) and (q[k+8], q[k+9]), k = 16 j + 2 t, hi and lo
    for (int i = threadIdx.x; i < (p.HD / 16) * 32; i += blockDim.x) {
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
    __syncthreads();
    if (ok) ok = mbar_wait(&full[s], (uint32_t)((local >> 1) & 1), p.status);
    const uint16_t* Kt = kv + (size_t)s * 2 * tile;
    const uint16_t* Vt = p.keqv ? Kt : Kt + tile;
    // ---- scores of this warp's 16 slots x the group's heads
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
    if (ok) {
      const uint16_t* k0 = Kt + (16 * warp + g) * p.kpitch + 2 * t;
      const uint16_t* k1 = k0 + 8 * p.kpitch;
#pragma unroll 4
      for (int j = 0; j < p.HD / 16; j++) {
        const uint32_t a0 = lds32(k0 + 16 * j), a1 = lds32(k1 + 16 * j);
        const uint32_t a2 = lds32(k0 + 16 * j + 8), a3 = lds32(k1 + 16 * j + 8);
        const uint4 qv = qf[j * 32 + lane];
        mma16816(sc, a0, a1, a2, a3, qv.x, qv.y);
        mma16816(sc, a0, a1, a2, a3, qv.z, qv.w);
      }
    }
    // sc: [0] (slot g, head 2t) [1] (slot g, head 2t+1) [2] (slot g+8, head 2t) [3] (slot g+8, head 2t+1)
    const uint32_t sa = t0 + 16 * warp + g, sb = sa + 8;
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
      red_m[warp][2 * t] = m0;
      red_m[warp][2 * t + 1] = m1;
    }
    __syncthreads();
    float M0 = red_m[0][2 * t], M1 = red_m[0][2 * t + 1];
#pragma unroll
    for (int w = 1; w < kAW; w++) {
      M0 = fmaxf(M0, red_m[w][2 * t]);
      M1 = fmaxf(M1, red_m[w][2 * t + 1]);
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
      red_l[warp][2 * t] = l0;
      red_l[warp][2 * t + 1] = l1;
    }
    // p as f16 hi + lo, [head][slot] (heads >= G keep their zeros)
    {
      const int la = 16 * warp + g, lb = la + 8;
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
    __syncthreads();
    // ---- O^T[d][head] for this warp's d tiles
    const int dtiles = p.HD / 16 / kAW;
    const size_t part_row = (size_t)b * p.QH + kvh * p.G;
    for (int dt = warp * dtiles; dt < (warp + 1) * dtiles && ok; dt++) {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < kAC / 16; ks++) {
        uint32_t a0, a1, a2, a3;
        const int row = 16 * ks + (lane & 7) + ((lane >> 4) << 3), col = 16 * dt + ((lane >> 3) & 1) * 8;
        ldsm_x4_trans(a0, a1, a2, a3, Vt + row * p.kpitch + col);
        const uint16_t* bh = ph + g * kPP + 16 * ks + 2 * t;
        const uint16_t* bl = pl + g * kPP + 16 * ks + 2 * t;
        mma16816(acc, a0, a1, a2, a3, lds32(bh), lds32(bh + 8));
        mma16816(acc, a0, a1, a2, a3, lds32(bl), lds32(bl + 8));
      }
      // acc: [0] (d g, head 2t) [1] (d g, head 2t+1) [2] (d g+8, head 2t) [3] (d g+8, head 2t+1)
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const int head = 2 * t + (k & 1), d = 16 * dt + g + ((k & 2) ? 8 : 0);
        if (head < p.G) p.part_o[((part_row + head) * p.max_chunks + c) * p.HD + d] = acc[k];
      }
    }
    if (warp == 0 && g == 0 && ok) {
      float L0 = 0.f, L1 = 0.f;
#pragma unroll
      for (int w = 0; w < kAW; w++) {
        L0 += red_l[w][2 * t];
        L1 += red_l[w][2 * t + 1];
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
    // every warp is done with this stage, the p rows and the q fragments
    __syncthreads();
    if (warp == 0 && ok && it + 2 * (int)gridDim.x < items) issue(it + 2 * gridDim.x, s);
  }
}

// Phase B over the live chunks: out[h][d] = sum_c o_c e^(m_c - M) / sum_c l_c e^(m_c - M).
__global__ void k_attcomb_dec(const AttP p, uint16_t* __restrict__ out_h, int xfo) {
  pdl_wait();
  const SlotRule rule = att_rule(p);
  const int nch = min((int)((rule.nslots() + kAC - 1) / kAC), p.max_chunks);
  const int h = blockIdx.x, b = blockIdx.y;
  const size_t row = (size_t)b * p.QH + h;
  const float* ml = p.part_ml + row * p.max_chunks * 2;
  float M = -INFINITY;
  for (int c = 0; c < nch; c++)
    if (ml[2 * c + 1] > 0.f) M = fmaxf(M, ml[2 * c]);
  float den = 0.f;
  for (int c = 0; c < nch; c++)
    if (ml[2 * c + 1] > 0.f) den += ml[2 * c + 1] * expf(ml[2 * c] - M);
  uint16_t* out = out_h + (size_t)b * p.QH * p.HD;
  for (int d = threadIdx.x; d < p.HD; d += blockDim.x) {
    float acc = 0.f;
    for (int c = 0; c < nch; c++)
      if (ml[2 * c + 1] > 0.f) acc = fmaf(p.part_o[(row * p.max_chunks + c) * p.HD + d], expf(ml[2 * c] - M), acc);
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
  p.kpitch = HD + 8;
  const size_t smem = (size_t)4 * kAC * p.kpitch * 2 + (size_t)(HD / 16) * 32 * 16 + (size_t)2 * 8 * kPP * 2;
  cudaError_t e = cudaFuncSetAttribute(k_attdec, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e4b_fail(c, E4B_ECUDA, "attdec smem attr: %s", cudaGetErrorString(e));
  const long long most = (long long)nseq * KVH * max_chunks;
  const int grid = (int)(most < c->sm_count ? most : c->sm_count);
  if (int r = e4b_launch(c, "attdec", k_attdec, dim3(grid), dim3(32 * kAW), smem, p)) return r;
  return e4b_launch(c, "attcomb_dec", k_attcomb_dec, dim3(QH, nseq), dim3(128), 0, p, out_h, xfo);
}

}  // extern "C"
