// Batched-prefill q4_0 GEMM on the 5th-generation tensor cores (sm_100a):
//   y[t][o] = sum_b d[o][b] * sum_{i in b} (n[o][i] - 8) * x[t][i]
// for many tokens t at once -- the reference's subgroup-matrix prefill GEMM
// (kernels/q40sg.wgsl:30-124, TPREC=f32: exact dequant, f32 accumulate) and its
// grouped-expert form over expert-sorted rows (kernels/q40grpsg32.wgsl:31-129).
//
// Tile = 128 weight rows (UMMA M, TMEM lanes) x 256 tokens (UMMA N, TMEM
// columns); K in steps of 64 (one 128-byte swizzle row of f16).  Per CTA (one
// per SM, persistent over tiles), warp-specialised:
//   warp 0      TMA: token tiles [256 rows x 64 halves] of x (128-byte swizzle)
//   warp 1      TMEM owner + MMA issuer (one thread): per K-step 8 x
//               tcgen05.mma 128x256x16 into a double-buffered f32 accumulator
//   warps 2-9   dequant: two threads per weight row (one q4_0 block of each
//               K-step each); raw q4_0 bytes fetched with cp.async, decoded
//               into an f16 "hi" tile and an f16 "lo" tile in the swizzled
//               K-major layout the MMA reads (see below)
//   warps 10-13 epilogue: tcgen05.ld of the accumulator, y (f32) or, for the
//               fused gate|up, f16(gelu(gate) * up)
// Exactness: a weight d*(n-8) needs up to 15 significant bits, more than f16
// holds, so it is split as hi = f16(d*(n-8)) and lo = d*(n-8) - hi (exact in
// f16, computed by one f16 FMA) and both are multiplied with x; every product
// is exact in the f32 accumulator.  The dequantised weights are therefore the
// reference's exact f32 values and only the summation order differs (as in the
// reference's own q40sg vs q40mv).  lo is stored negated (the FMA gives
// hi - d*(n-8)) and the second MMA negates A in its instruction descriptor.
#include "q40_stream.cuh"
#include "tc.cuh"

namespace {
using namespace e4b;

constexpr int kTM = 128;                 // weight rows per tile
constexpr int kTN = 256;                 // tokens per tile
constexpr int kTK = 64;                  // K per step
constexpr int kRawBlk = 8;               // q4_0 blocks per raw stage (4 K-steps)
constexpr int kSA = 3, kSB = 2, kSR = 2; // stages: dequantised weights, tokens, raw bytes
constexpr int kRawStride = 176;          // bytes per row of a raw stage (16-byte writes conflict free)
constexpr int kTileA = kTM * 128;        // 16 KB: one f16 tile (hi or lo) of a K-step
constexpr int kTileB = kTN * 128;        // 32 KB: the token tile of a K-step
constexpr int kThreads = 448;           // 14 warps: TMA, MMA, 8 dequant, 4 epilogue
constexpr int kMaxGroups = 256;
constexpr uint32_t kTmemCols = 512;      // two 256-column f32 accumulators

struct GemmP {
  const uint8_t* w;           // [groups][wrows][IN/32 * 18]
  const uint8_t* w_end;
  float* y;                   // epi 0: [M][OUT]
  uint16_t* yh;               // epi 1: [M][OUT] (OUT = FF)
  const uint32_t* offsets;    // [groups + 1] row offsets (null: one group of M rows)
  uint32_t* status;
  int IN, OUT, M, groups, epi;
  int nb, rowbytes, wrows, nwt, nk;
  uint64_t wait_ns;
};

struct Smem {
  uint64_t a_full[kSA], a_empty[kSA], b_full[kSB], b_empty[kSB], acc_full[2], acc_empty[2], drain;
  uint32_t tmem_base;
  int ntiles;
  int tile_off[kMaxGroups + 1];
  int ntt[kMaxGroups];
  int row_off[kMaxGroups];
  int row_end[kMaxGroups];
};

// Instruction descriptor for a tile: N = the tile's token rows rounded up to
// 16 (a group's last tile is usually partial: its MMAs shrink with it).
E4B_DEV uint32_t idesc_for(int nrows, bool neg_a) {
  return idesc_m128((uint32_t)min(kTN, max(16, (nrows + 15) & ~15)), neg_a);
}

// ---------------------------------------------------------------- tiles
// Tile order: per group, weight tile major, token tile minor (consecutive CTAs
// share a weight tile through L2).
struct Tile {
  int g, wt, tt, row0, nrows;
};
E4B_DEV Tile tile_of(const Smem& S, const GemmP& p, int t) {
  int lo = 0, hi = p.groups;                 // largest g with tile_off[g] <= t
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (S.tile_off[mid] <= t) lo = mid;
    else hi = mid;
  }
  Tile T;
  T.g = lo;
  const int local = t - S.tile_off[lo], ntt = S.ntt[lo];
  T.wt = local / ntt;
  T.tt = local - T.wt * ntt;
  T.row0 = S.row_off[lo] + T.tt * kTN;
  T.nrows = min(kTN, S.row_end[lo] - T.row0);
  return T;
}

// ---------------------------------------------------------------- dequant
// f16 pairs (n_a - 8, n_b - 8) from two nibble bytes, via 0x6400 | n = 1024 + n.
E4B_DEV uint32_t nib_pair(uint32_t nibbles, uint32_t sel) {
  return hsub2(__byte_perm(nibbles, 0x64u, sel), 0x64086408u);
}
// One q4_0 block (d, 16 nibble bytes q[0..3]) -> 4 chunks of 8 halves each for
// hi and for -lo: chunk 0 = elements 0-7 (low nibbles of bytes 0-7), 1 = 8-15
// (low nibbles of bytes 8-15), 2 = 16-23 (high nibbles of 0-7), 3 = 24-31.
E4B_DEV void decode_block(uint32_t d16, const uint32_t (&q)[4], uint4 (&hi)[4], uint4 (&nlo)[4]) {
  const uint32_t d2 = d16 | (d16 << 16);
  const uint32_t nd2 = d2 ^ 0x80008000u;
  uint32_t h[16], l[16];
#pragma unroll
  for (int w = 0; w < 4; w++) {
    const uint32_t lo4 = q[w] & 0x0F0F0F0Fu, hi4 = (q[w] >> 4) & 0x0F0F0F0Fu;
    const uint32_t v[4] = {nib_pair(lo4, 0x4140u), nib_pair(lo4, 0x4342u), nib_pair(hi4, 0x4140u),
                           nib_pair(hi4, 0x4342u)};
#pragma unroll
    for (int k = 0; k < 4; k++) {
      // low-nibble pairs of word w are elements 4w + 2(k&1) ...; high ones 16 + ...
      const int e = (k < 2 ? 0 : 16) + 4 * w + 2 * (k & 1);   // first element of the pair
      const uint32_t hh = hmul2(v[k], d2);
      h[e >> 1] = hh;
      l[e >> 1] = hfma2(v[k], nd2, hh);              // hi - d*(n-8) = -lo, exact
    }
  }
#pragma unroll
  for (int c = 0; c < 4; c++) {
    hi[c] = make_uint4(h[4 * c], h[4 * c + 1], h[4 * c + 2], h[4 * c + 3]);
    nlo[c] = make_uint4(l[4 * c], l[4 * c + 1], l[4 * c + 2], l[4 * c + 3]);
  }
}

// ---------------------------------------------------------------- kernel
__global__ void __launch_bounds__(kThreads, 1) k_tcgemm(const GemmP p, const __grid_constant__ CUtensorMap xmap) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ Smem S;
  uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* sA = base;                                           // [kSA][hi 16 KB | -lo 16 KB]
  uint8_t* sB = sA + (size_t)kSA * 2 * kTileA;                  // [kSB][32 KB]
  uint8_t* sR = sB + (size_t)kSB * kTileB;                      // [kSR][128 rows][176 B]
  float* sG = reinterpret_cast<float*>(sR + (size_t)kSR * kTM * kRawStride);   // [64][33] gate exchange
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kSA; i++) {
      mbar_init(&S.a_full[i], 2 * kTM);     // two dequant threads per weight row
      mbar_init(&S.a_empty[i], 1);
    }
    for (int i = 0; i < kSB; i++) {
      mbar_init(&S.b_full[i], 1);
      mbar_init(&S.b_empty[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&S.acc_full[i], 1);
      mbar_init(&S.acc_empty[i], kTM);
    }
    mbar_init(&S.drain, 1);
    fence_barrier_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&xmap)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&S.tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  pdl_wait();
  // group row offsets and the tile prefix (every CTA computes the same table)
  if (threadIdx.x == 0) {
    int tot = 0;
    for (int g = 0; g < p.groups; g++) {
      // row ranges clamped to [0, M]: inconsistent offsets can skip rows, never address outside x or y
      const int r0 = p.offsets ? (int)min(p.offsets[g], (uint32_t)p.M) : 0;
      const int r1 = p.offsets ? (int)min(max(p.offsets[g + 1], (uint32_t)r0), (uint32_t)p.M) : p.M;
      const int ntt = r1 > r0 ? (r1 - r0 + kTN - 1) / kTN : 0;
      S.row_off[g] = r0;
      S.row_end[g] = r1;
      S.ntt[g] = ntt > 0 ? ntt : 1;
      S.tile_off[g] = tot;
      tot += ntt * p.nwt;
    }
    S.tile_off[p.groups] = tot;
    S.ntiles = tot;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem_base;
  const int ntiles = S.ntiles;

  if (warp == 0) {
    // ---------------- TMA producer: token tiles
    if (lane == 0) {
      uint32_t cb = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        const Tile T = tile_of(S, p, t);
        for (int s = 0; s < p.nk && ok; s++, cb++) {
          const int st = cb % kSB;
          ok = wait_bar(&S.b_empty[st], ((cb / kSB) & 1u) ^ 1u, p.status, p.wait_ns);
          if (!ok) break;
          mbar_expect_tx(&S.b_full[st], (uint32_t)kTileB);
          tma_load_2d(sB + (size_t)st * kTileB, &xmap, s * kTK, T.row0, &S.b_full[st]);
        }
      }
      // let loads still in flight land before the CTA ends (bounded)
      for (uint32_t k = 0; k < kSB && k < cb; k++) {
        const uint32_t c = cb - 1 - k, st = c % kSB;
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&S.b_full[st], (c / kSB) & 1u) && globaltimer_ns() - t0 < p.wait_ns) {
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      uint32_t ca = 0, cb = 0, lt = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, lt++) {
        const uint32_t buf = lt & 1u;
        ok = wait_bar(&S.acc_empty[buf], ((lt >> 1) & 1u) ^ 1u, p.status, p.wait_ns);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + buf * (uint32_t)kTN;
        const Tile T = tile_of(S, p, t);
        const uint32_t idp = idesc_for(T.nrows, false), idn = idesc_for(T.nrows, true);
        for (int s = 0; s < p.nk; s++, ca++, cb++) {
          const int sa = ca % kSA, sb = cb % kSB;
          ok = wait_bar(&S.a_full[sa], (ca / kSA) & 1u, p.status, p.wait_ns) &&
               wait_bar(&S.b_full[sb], (cb / kSB) & 1u, p.status, p.wait_ns);
          if (!ok) break;
          tc_fence_after();
          const uint32_t a_hi = smem_u32(sA + (size_t)sa * 2 * kTileA), a_lo = a_hi + kTileA;
          const uint32_t b0 = smem_u32(sB + (size_t)sb * kTileB);
#pragma unroll
          for (int ks = 0; ks < kTK / 16; ks++) {
            const uint64_t bd = sw128_desc(b0 + 32 * ks);
            tc_mma(d_tmem, sw128_desc(a_hi + 32 * ks), bd, idp, (s | ks) != 0);
            tc_mma(d_tmem, sw128_desc(a_lo + 32 * ks), bd, idn, 1u);
          }
          tc_commit(&S.a_empty[sa]);
          tc_commit(&S.b_empty[sb]);
        }
        if (ok) tc_commit(&S.acc_full[buf]);
      }
      // every MMA this thread issued has completed before TMEM is released
      tc_commit(&S.drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&S.drain, 0) && globaltimer_ns() - t0 < p.wait_ns) {
      }
    }
    __syncwarp();
  } else if (warp < 10) {
    // ---------------- dequant: threads 2m, 2m+1 own weight row m of each tile;
    // thread h decodes block h of every K-step (two q4_0 blocks per K-step)
    const int dt = threadIdx.x - 64, m = dt >> 1, hh = dt & 1;
    uint8_t* raw = sR + (size_t)m * kRawStride;                 // + stage * kTM * kRawStride, shared by the pair
    uint32_t ca = 0;
    bool ok = true;
    const int nraw = (p.nb + kRawBlk - 1) / kRawBlk;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
      const Tile T = tile_of(S, p, t);
      int wrow;
      bool valid;
      if (p.epi == 1) {
        const int i = T.wt * (kTM / 2) + (m & (kTM / 2 - 1));
        valid = i < p.OUT;
        wrow = (m < kTM / 2) ? i : p.OUT + i;
      } else {
        wrow = T.wt * kTM + m;
        valid = wrow < p.OUT;
      }
      const uint8_t* src = p.w + ((size_t)T.g * p.wrows + (valid ? wrow : 0)) * p.rowbytes;
      // raw stage r: blocks [8r, 8r + nblk) of this row: the 16-byte aligned
      // cover, its chunks split between the row's two threads
      auto fetch = [&](int r) {
        if (!valid) return;
        const uint8_t* s0 = src + (size_t)r * kRawBlk * 18;
        const int nblk = min(kRawBlk, p.nb - r * kRawBlk);
        const uint8_t* a0 = reinterpret_cast<const uint8_t*>(reinterpret_cast<uintptr_t>(s0) & ~(uintptr_t)15);
        const uint8_t* a1 = s0 + nblk * 18;
        uint8_t* dst = raw + (size_t)(r % kSR) * kTM * kRawStride;
        for (int i = hh; i < 10 && a0 + 16 * i < a1; i += 2) {
          const uint8_t* q = a0 + 16 * i;
          const long long left = p.w_end - q;
          cp_async16z(dst + 16 * i, q, left >= 16 ? 16u : (uint32_t)left);
        }
      };
      fetch(0);
      cp_async_commit_group();
      for (int r = 0; r < nraw && ok; r++) {
        __syncwarp();                       // the pair is done reading the buffer about to be refilled
        if (r + 1 < nraw) fetch(r + 1);
        cp_async_commit_group();
        cp_async_wait_group<1>();
        __syncwarp();                       // the partner's chunks of stage r are visible
        uint32_t wd[36];
        {
          // the 16-byte aligned cover as ten 16-byte reads (row stride 176 = 11
          // chunks: the 8 rows of a quarter warp hit 8 distinct bank groups; a
          // row's two threads read the same addresses), then the row's bytes
          // from word offset (sh / 4), shifted by (sh % 4)
          const uint8_t* s0 = src + (size_t)r * kRawBlk * 18;
          const int sh = (int)(reinterpret_cast<uintptr_t>(s0) & 15);
          const uint4* rb = reinterpret_cast<const uint4*>(raw + (size_t)(r % kSR) * kTM * kRawStride);
          const uint32_t fs = (uint32_t)(sh & 2) * 8;
          uint32_t cw[40];
#pragma unroll
          for (int i = 0; i < 10; i++) {
            const uint4 v = rb[i];
            cw[4 * i] = v.x;
            cw[4 * i + 1] = v.y;
            cw[4 * i + 2] = v.z;
            cw[4 * i + 3] = v.w;
          }
          switch (sh >> 2) {     // compile-time register indices in every branch
#define E4B_WD(O)                                                                          \
  case O:                                                                                  \
    _Pragma("unroll") for (int j = 0; j < 36; j++) wd[j] = __funnelshift_r(cw[j + O], cw[j + O + 1], fs); \
    break;
            E4B_WD(0) E4B_WD(1) E4B_WD(2)
            default:
#pragma unroll
              for (int j = 0; j < 36; j++) wd[j] = __funnelshift_r(cw[j + 3], cw[j + 4], fs);
#undef E4B_WD
          }
          if (!valid)
#pragma unroll
            for (int j = 0; j < 36; j++) wd[j] = 0u;
        }
        const int nblk = min(kRawBlk, p.nb - r * kRawBlk);
#pragma unroll
        for (int k2 = 0; k2 < kRawBlk / 2; k2++) {
          if (2 * k2 >= nblk || !ok) break;
          const int sa = ca % kSA;
          ok = wait_bar(&S.a_empty[sa], ((ca / kSA) & 1u) ^ 1u, p.status, p.wait_ns);
          ok = __all_sync(0xffffffffu, ok);  // the pair's __syncwarp()s need the whole warp on one path
          if (!ok) break;
          uint8_t* th = sA + (size_t)sa * 2 * kTileA + (size_t)m * 128;
          uint8_t* tl = th + kTileA;
          // block 2 k2 + hh: d at byte 18 b, nibbles at 18 b + 2; even b is
          // word aligned, odd b two bytes past a word (both selected, no branch)
          const int we = (18 * (2 * k2)) / 4, wo = (18 * (2 * k2 + 1) - 2) / 4;
          const uint32_t d16 = hh ? (wd[wo] >> 16) : (wd[we] & 0xFFFFu);
          uint32_t q[4];
#pragma unroll
          for (int i = 0; i < 4; i++) q[i] = hh ? wd[wo + 1 + i] : __funnelshift_r(wd[we + i], wd[we + i + 1], 16);
          uint4 hi[4], nlo[4];
          decode_block(d16, q, hi, nlo);
#pragma unroll
          for (int c = 0; c < 4; c++) {
            const int chunk = 4 * hh + c;
            const uint32_t off = (uint32_t)((chunk ^ (m & 7)) << 4);
            *reinterpret_cast<uint4*>(th + off) = hi[c];
            *reinterpret_cast<uint4*>(tl + off) = nlo[c];
          }
          fence_proxy_async();              // generic-proxy writes -> the tensor core's reads
          mbar_arrive(&S.a_full[sa]);
          ca++;
        }
      }
    }
    cp_async_wait_group<0>();
  } else {
    // ---------------- epilogue: warp w reads TMEM lanes 32 (w % 4) ..
    const int q = warp & 3, m = 32 * q + lane;
    uint32_t lt = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, lt++) {
      const Tile T = tile_of(S, p, t);
      const uint32_t buf = lt & 1u;
      ok = wait_bar(&S.acc_full[buf], (lt >> 1) & 1u, p.status, p.wait_ns);
      ok = __all_sync(0xffffffffu, ok);     // the warp-collective TMEM loads below need every lane
      if (!ok) break;
      tc_fence_after();
      const uint32_t taddr = tmem + buf * (uint32_t)kTN + ((uint32_t)(32 * q) << 16);
      for (int cc = 0; cc < kTN / 32; cc++) {
        if (32 * cc >= T.nrows) break;
        float v[32];
        tc_ld32(taddr + 32 * cc, v);
        const int tok0 = T.row0 + 32 * cc, nt = min(32, T.nrows - 32 * cc);
        if (p.epi == 0) {
          const int o = T.wt * kTM + m;
          if (o < p.OUT) {
            float* yp = p.y + (size_t)tok0 * p.OUT + o;
#pragma unroll
            for (int j = 0; j < 32; j++)
              if (j < nt) yp[(size_t)j * p.OUT] = v[j];
          }
        } else {
          // gate rows (m < 64) hand their values to the up rows (m + 64)
          if (m < kTM / 2) {
#pragma unroll
            for (int j = 0; j < 32; j++) sG[m * 33 + j] = v[j];
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (m >= kTM / 2) {
            const int i = T.wt * (kTM / 2) + (m - kTM / 2);
            if (i < p.OUT) {
              uint16_t* yp = p.yh + (size_t)tok0 * p.OUT + i;
              const float* g = sG + (m - kTM / 2) * 33;
#pragma unroll
              for (int j = 0; j < 32; j++)
                if (j < nt) yp[(size_t)j * p.OUT] = f2h(gelu_tanh(g[j]) * v[j]);
            }
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
        }
      }
      tc_fence_before();
      mbar_arrive(&S.acc_empty[buf]);
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

bool x_map(CUtensorMap* m, const uint16_t* x, int IN, int M) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  const cuuint64_t dim[2] = {(cuuint64_t)IN, (cuuint64_t)M};
  const cuuint64_t stride[1] = {(cuuint64_t)IN * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kTK, (cuuint32_t)kTN};
  const cuuint32_t es[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<uint16_t*>(x), dim, stride, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

constexpr size_t kSmemBytes = 1024 + (size_t)kSA * 2 * kTileA + (size_t)kSB * kTileB + (size_t)kSR * kTM * kRawStride +
                              (size_t)(kTM / 2) * 33 * 4;

}  // namespace

extern "C" {

E4B_API int e4b_q40gemm(e4b_ctx* c, const uint16_t* x, const uint8_t* w, float* y, uint16_t* yh,
                        const uint32_t* offsets, int IN, int OUT, int M, int groups, int epi) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, x && w && M > 0 && OUT > 0 && groups >= 1 && groups <= kMaxGroups, "q40gemm: bad args");
  E4B_REQUIRE(c, IN > 0 && IN % kTK == 0, "q40gemm: IN=%d must be a multiple of %d", IN, kTK);
  E4B_REQUIRE(c, epi == 0 ? y != nullptr : (epi == 1 && yh != nullptr), "q40gemm: epi %d needs its output", epi);
  E4B_REQUIRE(c, groups == 1 || offsets, "q40gemm: grouped GEMM needs row offsets");
  E4B_REQUIRE(c, reinterpret_cast<uintptr_t>(x) % 16 == 0, "q40gemm: x must be 16-byte aligned");
  GemmP p = {};
  p.w = w; p.y = y; p.yh = yh; p.offsets = offsets; p.status = c->status;
  p.IN = IN; p.OUT = OUT; p.M = M; p.groups = groups; p.epi = epi;
  p.nb = IN / 32; p.rowbytes = p.nb * 18; p.nk = IN / kTK;
  p.wrows = epi == 1 ? 2 * OUT : OUT;
  p.nwt = epi == 1 ? (OUT + kTM / 2 - 1) / (kTM / 2) : (OUT + kTM - 1) / kTM;
  p.w_end = w + (size_t)groups * p.wrows * p.rowbytes;
  p.wait_ns = c->wait_ns;
  CUtensorMap xm;
  E4B_REQUIRE(c, x_map(&xm, x, IN, M), "q40gemm: activation tensor map failed");
  cudaError_t e = cudaFuncSetAttribute(k_tcgemm, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
  if (e != cudaSuccess) return e4b_fail(c, E4B_ECUDA, "q40gemm smem attr: %s", cudaGetErrorString(e));
  const long long tiles_max = ((long long)(M + kTN - 1) / kTN + (groups > 1 ? groups : 0)) * p.nwt;
  const int grid = (int)(tiles_max < c->sm_count ? tiles_max : c->sm_count);
  return e4b_launch(c, "q40gemm", k_tcgemm, dim3(grid), dim3(kThreads), kSmemBytes, p, xm);
}

}  // extern "C"
