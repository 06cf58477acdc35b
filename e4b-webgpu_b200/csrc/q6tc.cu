// Batched q6_K LM head on the 5th-generation tensor cores (sm_100a):
//   y[t][o] = softcap( sum_b d[o][b] * sum_{j<16} sc[o][b][j] * sum_{i in j} (q[o][i] - 32) * x[t][i] )
// for up to 64 token rows t -- the reference's LM head (kernels/q6kmv.wgsl,
// f32 dequantisation and accumulation; its batched-decode form runs it once
// per sequence) for a whole decode batch at once.
//
// Tile = 128 vocabulary rows (UMMA M, TMEM lanes); the batch's tokens are the
// UMMA N side: B = [x_hi (NP rows); x_lo (NP rows)], x = x_hi + x_lo split into
// two f16 halves by k_q6tc_prep, NP = 32 or 64.  K in steps of 64 (one
// 128-byte swizzle row of f16).  Per CTA (one per SM, persistent over tiles),
// warp-specialised:
//   warp 0      TMA: the [2 NP x 64] slab of B for each K-step
//   warp 1      TMEM owner + MMA issuer (one thread)
//   warps 2-17  dequant: four threads per vocabulary row, one q6_K
//               superblock (256 k = 4 K-steps) per raw stage
//   warps 18-21 epilogue: per superblock, tcgen05.ld of its accumulator,
//               times d, added to the tile's running sum (kept in TMEM);
//               softcap and store at the tile's end
//   warp 22     raw weights (tile-packed layout): per superblock one 1-D TMA
//               bulk copy of the tile's 128 x 212 contiguous bytes, three
//               superblocks in flight.  With the row-major layout the dequant
//               threads fetch their rows' 224-byte covers with cp.async instead.
//
// Measured on B200 (A4B 262144 x 2816, n = 64): 500 us on the packed layout,
// 525 us row-major (the mma.sync kernel: 965 us).  For 1..32 rows the packed
// copy goes to the warp-MMA kernels below instead (k_q6gv, k_q6gm).  The time barely depends on
// n: dequantisation, the per-K-step MMA issue and the hand-offs between the
// warp roles bound it, not HBM (605 MB would stream in ~93 us).
//
// Exactness.  The superblock scale d (f16) is applied in f32 by the epilogue;
// inside a superblock the weight is the integer m = sc * (q - 32), |m| <= 4096,
// which f16 holds exactly only up to 2048.  So A is split like the q4_0 GEMM
// does: hi = f16(m) (one f16 multiply) and lo = m - hi in {-1, 0, 1} (one f16
// FMA, exact), lo stored negated and the MMA negating it back.  Per K = 16:
//   MMA 1: hi x [x_hi; x_lo]  (N = 2 NP: columns [0, NP) and [NP, 2 NP))
//   MMA 2: lo x  x_hi         (N = NP, into columns [0, NP))
// Every product is exact in the f32 accumulator; the dropped lo * x_lo term is
// below 2^-23 of the hi * x terms it sits beside (|lo| <= 1 where |m| > 2048,
// |x_lo| <= 2^-11 |x|).  Each superblock accumulates into its own 2 NP
// TMEM columns (three buffers rotate), which the epilogue folds into the
// running sum as y += d * (C[t] + C[NP + t]).
#include "q40_stream.cuh"
#include "tc.cuh"

namespace {
using namespace e4b;

constexpr int kQM = 128;                   // vocabulary rows per tile
constexpr int kQK = 64;                    // K per step
constexpr int kQSA = 3, kQSB = 2, kQSR = 3;  // stages: dequantised A, token slabs, raw superblocks
constexpr int kQCover = 224;               // 16-byte aligned cover of a 210-byte superblock
constexpr int kPk = 212;                   // packed superblock entry: the 210 bytes + 2 zero bytes (4-byte aligned rows)
constexpr int kQRawStride = 240;           // bytes per row of a raw stage (15 x 16: odd chunk count)
constexpr int kQTileA = kQM * 128;         // 16 KB: one f16 tile (hi or -lo) of a K-step
constexpr int kQMaxNP = 64;
constexpr int kQTileB = 2 * kQMaxNP * 128; // 16 KB: [x_hi; x_lo] slab of a K-step
constexpr int kQBufs = 3;                  // superblock accumulators in TMEM
constexpr int kQBufCols = 2 * kQMaxNP;
constexpr int kQTotal = kQBufs * kQBufCols;  // TMEM columns of the tile's running sum (NP of them)
constexpr uint32_t kQTmemCols = 512;
constexpr int kQDeqWarps = 16;             // four threads per vocabulary row
constexpr int kQEpiWarp0 = 2 + kQDeqWarps;  // four epilogue warps, then the raw-weight producer
constexpr int kQRawWarp = kQEpiWarp0 + 4;
constexpr int kQThreads = 32 * (kQRawWarp + 1);

struct Q6P {
  const uint8_t* w;
  const uint8_t* w_end;
  float* y;                 // [n][OUT]
  uint32_t* status;
  int N, OUT, n, NP, nsb, rowbytes, ntiles;
  float softcap;
  uint64_t wait_ns;
};

struct Q6Smem {
  uint64_t a_full[kQSA], a_empty[kQSA], b_full[kQSB], b_empty[kQSB], acc_full[kQBufs], acc_empty[kQBufs], drain;
  uint64_t r_full[kQSR], r_empty[kQSR];
  uint32_t tmem_base;
};

// xs[r][k]: r < NP: f16(x[r][k]); NP <= r < 2 NP: f16(x[r-NP][k] - that); 0 for tokens >= n.
__global__ void k_q6tc_prep(const float* __restrict__ x, uint16_t* __restrict__ xs, int n, int N, int NP) {
  pdl_wait();
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (size_t)NP * N) return;
  const int t = (int)(idx / N);
  const size_t k = idx - (size_t)t * N;
  uint16_t h = 0, l = 0;
  if (t < n) {
    const float v = x[(size_t)t * N + k];
    const __half hh = __float2half_rn(v);
    h = __half_as_ushort(hh);
    l = f2h(v - __half2float(hh));
  }
  xs[(size_t)t * N + k] = h;
  xs[(size_t)(NP + t) * N + k] = l;
}

// four 6-bit values (one per byte) -> f16 pairs (v0 - 32, v1 - 32), (v2 - 32, v3 - 32)
E4B_DEV void q6_quad(uint32_t v, uint32_t& p01, uint32_t& p23) {
  p01 = hsub2(__byte_perm(v, 0x64646464u, 0x5140u), 0x64206420u);
  p23 = hsub2(__byte_perm(v, 0x64646464u, 0x5342u), 0x64206420u);
}
E4B_DEV uint32_t sc_pair(uint32_t scw, int byte) {
  const int s = (int)(int8_t)((scw >> (8 * byte)) & 0xFFu);
  const uint32_t h = __half_as_ushort(__int2half_rn(s));
  return h | (h << 16);
}

// Tile-packed copy of a row-major q6_K matrix: dst entry (t, sb, m) = row
// 128 t + m's superblock sb (210 bytes, then 2 zero bytes so every entry is
// 4-byte aligned), zero for rows >= OUT (one thread per 2 bytes).
__global__ void k_q6_pack(const uint16_t* __restrict__ src, uint16_t* __restrict__ dst, int OUT, int nsb,
                          size_t total) {
  pdl_wait();
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const size_t blk = i / (kPk / 2);
  const int hw = (int)(i - blk * (kPk / 2));
  const int m = (int)(blk % kQM);
  const size_t ts = blk / kQM;
  const int sb = (int)(ts % nsb);
  const size_t t = ts / nsb;
  const size_t row = t * kQM + m;
  dst[i] = row < (size_t)OUT && hw < 105 ? src[(row * nsb + sb) * 105 + hw] : (uint16_t)0;
}

// PACKED: w is the tile-packed copy (k_q6_pack): superblock sb of row 128 t + m
// at byte ((t * nsb + sb) * 128 + m) * 212, so a raw stage is one contiguous
// 27136-byte TMA bulk copy.  Otherwise w is row-major q6_K and the dequant
// threads fetch their rows' 224-byte covers with cp.async.
template <bool PACKED>
__global__ void __launch_bounds__(kQThreads, 1) k_q6tc(const Q6P p, const __grid_constant__ CUtensorMap xmap) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ Q6Smem S;
  uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* sA = base;                                            // [kQSA][hi 16 KB | -lo 16 KB]
  uint8_t* sB = sA + (size_t)kQSA * 2 * kQTileA;                 // [kQSB][16 KB]
  uint8_t* sR = sB + (size_t)kQSB * kQTileB;                     // [kQSR][128 rows][240 B]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kQSA; i++) {
      mbar_init(&S.a_full[i], kQDeqWarps);
      mbar_init(&S.a_empty[i], 1);
    }
    for (int i = 0; i < kQSB; i++) {
      mbar_init(&S.b_full[i], 1);
      mbar_init(&S.b_empty[i], 1);
    }
    for (int i = 0; i < kQBufs; i++) {
      mbar_init(&S.acc_full[i], 1);
      mbar_init(&S.acc_empty[i], kQM);
    }
    for (int i = 0; i < kQSR; i++) {
      mbar_init(&S.r_full[i], 1);
      mbar_init(&S.r_empty[i], kQDeqWarps);
    }
    mbar_init(&S.drain, 1);
    fence_barrier_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&xmap)) : "memory");
  }
  if (warp == 1) tc_alloc(&S.tmem_base, kQTmemCols);
  pdl_wait();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem_base;
  const int nk = 4 * p.nsb;

  if (warp == 0) {
    // ---------------- TMA producer: the token slab of every K-step
    if (lane == 0) {
      const uint32_t bbytes = (uint32_t)(2 * p.NP * 128);
      uint32_t cb = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.ntiles && ok; t += gridDim.x) {
        for (int s = 0; s < nk; s++, cb++) {
          const int st = cb % kQSB;
          ok = wait_bar(&S.b_empty[st], ((cb / kQSB) & 1u) ^ 1u, p.status, p.wait_ns);
          if (!ok) break;
          mbar_expect_tx(&S.b_full[st], bbytes);
          tma_load_2d(sB + (size_t)st * kQTileB, &xmap, s * kQK, 0, &S.b_full[st]);
        }
      }
      for (uint32_t k = 0; k < kQSB && k < cb; k++) {
        const uint32_t c = cb - 1 - k;
        drain_bar(&S.b_full[c % kQSB], (c / kQSB) & 1u, p.wait_ns);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      const uint32_t id_hi = idesc_m128((uint32_t)(2 * p.NP), false), id_lo = idesc_m128((uint32_t)p.NP, true);
      uint32_t ca = 0, cb = 0, j = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.ntiles && ok; t += gridDim.x) {
        for (int sb = 0; sb < p.nsb && ok; sb++, j++) {
          const uint32_t buf = j % kQBufs;
          ok = wait_bar(&S.acc_empty[buf], ((j / kQBufs) & 1u) ^ 1u, p.status, p.wait_ns);
          if (!ok) break;
          tc_fence_after();
          const uint32_t d_tmem = tmem + buf * (uint32_t)kQBufCols;
          for (int s = 0; s < 4; s++, ca++, cb++) {
            const int sa = ca % kQSA, sbb = cb % kQSB;
            ok = wait_bar(&S.a_full[sa], (ca / kQSA) & 1u, p.status, p.wait_ns) &&
                 wait_bar(&S.b_full[sbb], (cb / kQSB) & 1u, p.status, p.wait_ns);
            if (!ok) break;
            tc_fence_after();
            const uint32_t a_hi = smem_u32(sA + (size_t)sa * 2 * kQTileA), a_lo = a_hi + kQTileA;
            const uint32_t b0 = smem_u32(sB + (size_t)sbb * kQTileB);
#pragma unroll
            for (int ks = 0; ks < kQK / 16; ks++) {
              const uint64_t bd = sw128_desc(b0 + 32 * ks);
              tc_mma(d_tmem, sw128_desc(a_hi + 32 * ks), bd, id_hi, (s | ks) != 0);
              tc_mma(d_tmem, sw128_desc(a_lo + 32 * ks), bd, id_lo, 1u);
            }
            tc_commit(&S.a_empty[sa]);
            tc_commit(&S.b_empty[sbb]);
          }
          if (ok) tc_commit(&S.acc_full[buf]);
        }
      }
      // every MMA this thread issued has completed before TMEM is released
      tc_commit(&S.drain);
      drain_bar(&S.drain, 0, p.wait_ns);
    }
    __syncwarp();
  } else if (warp < 2 + kQDeqWarps) {
    // ---------------- dequant: threads 4m .. 4m+3 own vocabulary row m of each
    // tile.  For K-step s = 2 h + odd (half h of the superblock) thread qq
    // produces elements 16 qq .. 16 qq + 15 of the step (one sub-block):
    // 6-bit values from ql[64 h + 16 qq + i] (low nibble for even steps, high
    // for odd) and bits (2 (qq / 2) + 4 odd) of qh[32 h + 16 (qq % 2) + i],
    // scale sc[8 h + 4 odd + qq].
    const int dt = threadIdx.x - 64, m = dt >> 2, qq = dt & 3;
    uint32_t ca = 0, cr = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < p.ntiles && ok; t += gridDim.x) {
      const int row = t * kQM + m;
      const bool valid = row < p.OUT;
      const uint8_t* src = p.w + (size_t)(valid ? row : 0) * p.rowbytes;
      auto fetch = [&](int sb) {              // row-major layout: this thread's chunks of the row's cover
        if (!valid) return;
        const uint8_t* a0 =
            reinterpret_cast<const uint8_t*>(reinterpret_cast<uintptr_t>(src + (size_t)sb * 210) & ~(uintptr_t)15);
        uint8_t* dst = sR + ((size_t)(sb % kQSR) * kQM + m) * kQRawStride;
        for (int i = qq; i < kQCover / 16; i += 4) {
          const uint8_t* q = a0 + 16 * i;
          const long long left = p.w_end - q;
          if (left > 0) cp_async16z(dst + 16 * i, q, left >= 16 ? 16u : (uint32_t)left);
        }
      };
      if constexpr (!PACKED) {                // raw superblocks two ahead of the one being decoded
        fetch(0);
        cp_async_commit_group();
        if (p.nsb > 1) fetch(1);
        cp_async_commit_group();
      }
      for (int sb = 0; sb < p.nsb && ok; sb++, cr++) {
        int st, sh;
        const uint8_t* slot;
        if constexpr (PACKED) {
          st = cr % kQSR;
          ok = wait_bar(&S.r_full[st], (cr / kQSR) & 1u, p.status, p.wait_ns);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
          sh = (m * kPk) & 15;
          slot = sR + (size_t)st * kQM * kQRawStride + ((m * kPk) & ~15);
        } else {
          st = sb % kQSR;
          __syncwarp();                       // the row's threads are done reading the stage about to be refilled
          if (sb + 2 < p.nsb) fetch(sb + 2);
          cp_async_commit_group();
          cp_async_wait_group<2>();
          __syncwarp();                       // the other threads' chunks of this stage are visible
          sh = (int)(reinterpret_cast<uintptr_t>(src + (size_t)sb * 210) & 15);
          slot = sR + ((size_t)st * kQM + m) * kQRawStride;
        }
        const uint32_t* rw = reinterpret_cast<const uint32_t*>(slot);   // sh is even
        const uint32_t fs = (uint32_t)(sh & 2) * 8;
        const int w0 = sh >> 2;
#pragma unroll
        for (int h = 0; h < 2; h++) {
          uint32_t ql[4], qh[4], scw[2];
          {
            uint32_t a[5], b[5], c[3];
            const int oq = w0 + 16 * h + 4 * qq, oh = w0 + 32 + 8 * h + 4 * (qq & 1), os = w0 + 48 + 2 * h;
#pragma unroll
            for (int i = 0; i < 5; i++) {
              a[i] = rw[oq + i];
              b[i] = rw[oh + i];
            }
#pragma unroll
            for (int i = 0; i < 3; i++) c[i] = rw[os + i];
#pragma unroll
            for (int i = 0; i < 4; i++) {
              ql[i] = __funnelshift_r(a[i], a[i + 1], fs);
              qh[i] = __funnelshift_r(b[i], b[i + 1], fs);
            }
            scw[0] = __funnelshift_r(c[0], c[1], fs);
            scw[1] = __funnelshift_r(c[1], c[2], fs);
            if (!valid) scw[0] = scw[1] = 0u;    // rows past OUT: zero weights (never stored)
          }
          if (PACKED && h == 1) {                  // this warp's reads of the raw stage are done
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.r_empty[st]);
          }
#pragma unroll
          for (int odd = 0; odd < 2; odd++) {
            const int sa = ca % kQSA;
            ok = wait_bar(&S.a_empty[sa], ((ca / kQSA) & 1u) ^ 1u, p.status, p.wait_ns);
            ok = __all_sync(0xffffffffu, ok);  // the __syncwarp()s above need the whole warp on one path
            if (!ok) break;
            uint8_t* th = sA + (size_t)sa * 2 * kQTileA + (size_t)m * 128;
            uint8_t* tl = th + kQTileA;
            const uint32_t sc2 = sc_pair(scw[odd], qq), nsc2 = sc2 ^ 0x80008000u;
            const int qhs = 2 * (qq >> 1) + 4 * odd;   // qh bits of this thread's elements
#pragma unroll
            for (int c = 0; c < 2; c++) {
              uint32_t hi[4], nlo[4];
#pragma unroll
              for (int wq = 0; wq < 2; wq++) {
                const uint32_t lo4 = (odd ? (ql[2 * c + wq] >> 4) : ql[2 * c + wq]) & 0x0F0F0F0Fu;
                const uint32_t hb = ((qh[2 * c + wq] >> qhs) & 0x03030303u) << 4;
                uint32_t p01, p23;
                q6_quad(lo4 | hb, p01, p23);
                hi[2 * wq] = hmul2(p01, sc2);
                hi[2 * wq + 1] = hmul2(p23, sc2);
                nlo[2 * wq] = hfma2(p01, nsc2, hi[2 * wq]);          // hi - m = -lo, exact
                nlo[2 * wq + 1] = hfma2(p23, nsc2, hi[2 * wq + 1]);
              }
              const uint32_t off = (uint32_t)(((2 * qq + c) ^ (m & 7)) << 4);
              *reinterpret_cast<uint4*>(th + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
              *reinterpret_cast<uint4*>(tl + off) = make_uint4(nlo[0], nlo[1], nlo[2], nlo[3]);
            }
            fence_proxy_async();              // generic-proxy writes -> the tensor core's reads
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.a_full[sa]);   // one arrival per warp
            ca++;
          }
          if (!ok) break;
        }
      }
    }
    if constexpr (!PACKED) cp_async_wait_group<0>();
  } else if (warp < kQRawWarp) {
    // ---------------- epilogue: warp w reads TMEM lanes 32 (w % 4) .. ; the
    // tile's running sum over superblocks lives in TMEM columns [kQTotal, + NP)
    const int q = warp & 3, m = 32 * q + lane;
    const int NP = p.NP;
    const uint32_t lanes = (uint32_t)(32 * q) << 16, ttot = tmem + (uint32_t)kQTotal + lanes;
    uint32_t j = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < p.ntiles && ok; t += gridDim.x) {
      const int row = t * kQM + m;
      const bool valid = row < p.OUT;
      for (int sb = 0; sb < p.nsb; sb++, j++) {
        const size_t doff = PACKED ? (((size_t)t * p.nsb + sb) * kQM + m) * kPk + 208
                                   : (size_t)(valid ? row : 0) * p.rowbytes + (size_t)sb * 210 + 208;
        const float d = valid ? h2f(*reinterpret_cast<const uint16_t*>(p.w + doff)) : 0.f;
        const uint32_t buf = j % kQBufs;
        ok = wait_bar(&S.acc_full[buf], (j / kQBufs) & 1u, p.status, p.wait_ns);
        ok = __all_sync(0xffffffffu, ok);     // the warp-collective TMEM accesses below need every lane
        if (!ok) break;
        tc_fence_after();
        const uint32_t taddr = tmem + buf * (uint32_t)kQBufCols + lanes;
        for (int cc = 0; 32 * cc < NP; cc++) {
          uint32_t hi[32], lo[32];
          tc_ld32_nowait(taddr + 32 * cc, hi);
          tc_ld32_nowait(taddr + NP + 32 * cc, lo);
          tc_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; i++) hi[i] = __float_as_uint(d * (__uint_as_float(hi[i]) + __uint_as_float(lo[i])));
          if (sb > 0) {
            tc_ld32_nowait(ttot + 32 * cc, lo);
            tc_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; i++) hi[i] = __float_as_uint(__uint_as_float(hi[i]) + __uint_as_float(lo[i]));
          }
          tc_st32(ttot + 32 * cc, hi);
        }
        tc_wait_st();
        tc_fence_before();
        mbar_arrive(&S.acc_empty[buf]);
      }
      if (!ok) break;
      // the whole warp reads its lanes' sums (tcgen05.ld is warp-collective);
      // only rows inside the vocabulary are stored
      for (int cc = 0; 32 * cc < NP; cc++) {
        uint32_t v[32];
        tc_ld32_nowait(ttot + 32 * cc, v);
        tc_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; i++) {
          const int tok = 32 * cc + i;
          if (valid && tok < p.n) {
            const float x = __uint_as_float(v[i]);
            p.y[(size_t)tok * p.OUT + row] = p.softcap != 0.f ? p.softcap * tanhf(x / p.softcap) : x;
          }
        }
      }
    }
  } else {
    // ---------------- raw-weight producer (tile-packed layout): per superblock
    // one 1-D TMA bulk copy of the tile's 128 x 212 contiguous bytes
    if (PACKED && lane == 0) {
      constexpr uint32_t kStage = (uint32_t)kQM * kPk;
      uint32_t cr = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.ntiles && ok; t += gridDim.x) {
        for (int sb = 0; sb < p.nsb; sb++, cr++) {
          const int st = cr % kQSR;
          ok = wait_bar(&S.r_empty[st], ((cr / kQSR) & 1u) ^ 1u, p.status, p.wait_ns);
          if (!ok) break;
          mbar_expect_tx(&S.r_full[st], kStage);
          bulk_g2s(sR + (size_t)st * kQM * kQRawStride, p.w + ((size_t)t * p.nsb + sb) * kStage, kStage,
                   &S.r_full[st]);
        }
      }
      // let copies still in flight land before the CTA ends (bounded)
      for (uint32_t k = 0; k < kQSR && k < cr; k++) {
        const uint32_t c = cr - 1 - k;
        drain_bar(&S.r_full[c % kQSR], (c / kQSR) & 1u, p.wait_ns);
      }
    }
    __syncwarp();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tc_dealloc(tmem, kQTmemCols);
  }
}

constexpr size_t kQSmemBytes =
    1024 + (size_t)kQSA * 2 * kQTileA + (size_t)kQSB * kQTileB + (size_t)kQSR * kQM * kQRawStride;

// ---------------------------------------------------------------- one token
// LM head for ONE token row on the tile-packed copy (decode at batch 1), on
// the warp-level tensor cores.  Work unit = 16 consecutive rows (8 per
// 128-row tile); a unit's superblock sb is one contiguous 16 x 212-byte
// stretch of the packed copy, which the warp's lane 0 brings into the warp's
// ring with one bulk copy, three stages ahead.  Per superblock half (128 k,
// 8 sub-blocks of 16) the lanes run 16 m16n8k16 MMAs (x as f16 hi + lo) with
// the block-diagonal B of the q4_0 GEMV: sub-block j's x sits in column j, so
// column j of the accumulator is sub-block j's dot product and gets its own
// scale d * sc[j] in f32 afterwards.  A = q - 32, exact in f16; within a
// sub-block the k order is permuted (lane t's MMA slots 2t, 2t+1, 2t+8, 2t+9
// hold elements 4t .. 4t+3, the 4 bytes of one word) on both A and B.  The
// products are exact in the f32 accumulator; only the summation order
// differs from kernels/q6k.wgsl.
constexpr int kGW = 16;                    // warps per CTA
constexpr int kGS = 3;                     // ring stages per warp
constexpr int kGStage = 16 * kPk;          // one unit's superblock: 3392 bytes

// xs[s][t] for sub-block s (16 elements) and lane slot t: {hi(x[16s+4t], +1),
// hi(+2, +3), lo(..), lo(..)} with x = hi + lo split into f16.
E4B_DEV uint4 x_slot(const float* __restrict__ x, int s, int t) {
  const float4 v = *reinterpret_cast<const float4*>(x + 16 * s + 4 * t);
  const float f[4] = {v.x, v.y, v.z, v.w};
  uint16_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const __half hh = __float2half_rn(f[i]);
    h[i] = __half_as_ushort(hh);
    l[i] = f2h(f[i] - __half2float(hh));
  }
  return make_uint4(pack_h2(h[0], h[1]), pack_h2(h[2], h[3]), pack_h2(l[0], l[1]), pack_h2(l[2], l[3]));
}
// (a & m) | c as one LOP3 (truth table 0xEA)
E4B_DEV uint32_t lop_and_or(uint32_t a, uint32_t m, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(m), "r"(c));
  return d;
}
// 4 six-bit values of one word of a sub-block: nibbles of ql (hi4: the high
// ones) with bits `qsh` of each qh byte above them, as f16 pairs of (q - 32).
E4B_DEV void q6_word(uint32_t ql, uint32_t qh, bool hi4, int qsh, uint32_t& p01, uint32_t& p23) {
  const uint32_t lo4 = hi4 ? (ql >> 4) : ql;
  const uint32_t hb = ((qh >> qsh) << 4) & 0x30303030u;
  q6_quad(lop_and_or(lo4, 0x0F0F0F0Fu, hb), p01, p23);
}

__global__ void __launch_bounds__(32 * kGW, 1) k_q6gv(const uint8_t* __restrict__ wt, const float* __restrict__ x,
                                                    float* __restrict__ y, int N, int OUT, float softcap,
                                                    uint32_t* status, uint64_t wait_ns) {
  extern __shared__ __align__(16) uint8_t gsm[];
  __shared__ __align__(8) uint64_t full[kGW][kGS];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int nsb = N >> 8, nsub = N >> 4;
  uint4* xs = reinterpret_cast<uint4*>(gsm);                                   // [nsub][4]
  uint8_t* ring = gsm + (size_t)nsub * 4 * 16 + (size_t)warp * kGS * kGStage;  // this warp's stages
  if (lane == 0) {
    for (int s = 0; s < kGS; s++) mbar_init(&full[warp][s], 1);
    fence_barrier_init();
  }
  __syncwarp();
  const int units = ((OUT + 127) / 128) * 8;                 // 16-row units of whole tiles
  const int w0 = blockIdx.x * kGW + warp, wstep = gridDim.x * kGW;
  const int nmine = w0 < units ? (units - w0 + wstep - 1) / wstep : 0;
  const int steps = nmine * nsb;                             // (unit, superblock) stages of this warp
  auto issue = [&](int k) {                                  // lane 0: stage k into ring slot k % kGS
    const int u = w0 + (k / nsb) * wstep, sb = k % nsb;
    const int tile = u >> 3, rg = u & 7;
    const uint8_t* src = wt + (((size_t)tile * nsb + sb) * 8 + rg) * (size_t)kGStage;
    mbar_expect_tx(&full[warp][k % kGS], (uint32_t)kGStage);
    bulk_g2s(ring + (size_t)(k % kGS) * kGStage, src, (uint32_t)kGStage, &full[warp][k % kGS]);
  };
  // the weights do not depend on the previous kernel: request them first
  if (lane == 0)
    for (int k = 0; k < kGS && k < steps; k++) issue(k);
  pdl_wait();
  for (int i = threadIdx.x; i < nsub * 4; i += blockDim.x) xs[i] = x_slot(x, i >> 2, i & 3);
  __syncthreads();

  const int ra = g * kPk, rb = (g + 8) * kPk;                // this lane's rows in a stage
  bool ok = true;
  int k = 0;
  for (int j = 0; j < nmine; j++) {
    const int u = w0 + j * wstep;
    float acc_a = 0.f, acc_b = 0.f;
    for (int sb = 0; sb < nsb; sb++, k++) {
      const int st = k % kGS;
      if (ok) ok = mbar_wait(&full[warp][st], (uint32_t)((k / kGS) & 1), status);
      ok = __all_sync(0xffffffffu, ok);      // the MMAs below need the whole warp on one path
      const uint8_t* sg = ring + (size_t)st * kGStage;
      if (ok) {
        const float da = h2f(*reinterpret_cast<const uint16_t*>(sg + ra + 208));
        const float db = h2f(*reinterpret_cast<const uint16_t*>(sg + rb + 208));
#pragma unroll
        for (int h = 0; h < 2; h++) {
          // this lane's B: x of sub-block g of the half (column g), hi and lo
          const uint4 xv = xs[(16 * sb + 8 * h + g) * 4 + t];
          uint32_t qla[4], qlb[4], qha[2], qhb[2];
#pragma unroll
          for (int q = 0; q < 4; q++) {      // ql words (jj & 1, lh) = (q >> 1, q & 1)
            const int o = 64 * h + 32 * (q >> 1) + 16 * (q & 1) + 4 * t;
            qla[q] = *reinterpret_cast<const uint32_t*>(sg + ra + o);
            qlb[q] = *reinterpret_cast<const uint32_t*>(sg + rb + o);
          }
#pragma unroll
          for (int lh = 0; lh < 2; lh++) {
            const int o = 128 + 32 * h + 16 * lh + 4 * t;
            qha[lh] = *reinterpret_cast<const uint32_t*>(sg + ra + o);
            qhb[lh] = *reinterpret_cast<const uint32_t*>(sg + rb + o);
          }
          float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int jb = 0; jb < 8; jb++) {   // sub-block jb = 2 jj + lh of the half
            const int jj = jb >> 1, lh = jb & 1, q = 2 * (jj & 1) + lh;
            uint32_t a01, a23, b01, b23;
            q6_word(qla[q], qha[lh], jj >= 2, 2 * jj, a01, a23);
            q6_word(qlb[q], qhb[lh], jj >= 2, 2 * jj, b01, b23);
            const bool mine = g == jb;
            mma16816(c, a01, b01, a23, b23, mine ? xv.x : 0u, mine ? xv.y : 0u);
            mma16816(c, a01, b01, a23, b23, mine ? xv.z : 0u, mine ? xv.w : 0u);
          }
          // c[0], c[1]: row g, sub-blocks 2t, 2t+1 of the half; c[2], c[3]: row g + 8
          const int so = 192 + 8 * h + 2 * t;
          const uint32_t sa = *reinterpret_cast<const uint16_t*>(sg + ra + so);
          const uint32_t sbv = *reinterpret_cast<const uint16_t*>(sg + rb + so);
          acc_a = fmaf(da, fmaf((float)(int8_t)(sa & 0xFFu), c[0], (float)(int8_t)(sa >> 8) * c[1]), acc_a);
          acc_b = fmaf(db, fmaf((float)(int8_t)(sbv & 0xFFu), c[2], (float)(int8_t)(sbv >> 8) * c[3]), acc_b);
        }
      }
      __syncwarp();                  // every lane's reads of the stage are done before it is refilled
      if (lane == 0 && ok && k + kGS < steps) issue(k + kGS);
    }
    // the 4 lanes of a row group hold its sub-block columns: sum them
    acc_a += __shfl_xor_sync(0xffffffffu, acc_a, 1);
    acc_a += __shfl_xor_sync(0xffffffffu, acc_a, 2);
    acc_b += __shfl_xor_sync(0xffffffffu, acc_b, 1);
    acc_b += __shfl_xor_sync(0xffffffffu, acc_b, 2);
    const int r0 = 16 * u + g;
    if (t == 0 && ok) {
      if (r0 < OUT) y[r0] = softcap != 0.f ? softcap * tanhf(acc_a / softcap) : acc_a;
      if (r0 + 8 < OUT) y[r0 + 8] = softcap != 0.f ? softcap * tanhf(acc_b / softcap) : acc_b;
    }
  }
  // copies still in flight after a time-out land (bounded) before the CTA ends
  if (lane == 0 && !ok)
    for (int q = k; q < k + kGS && q < steps; q++) {
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&full[warp][q % kGS], (uint32_t)((q / kGS) & 1)) && globaltimer_ns() - t0 < wait_ns) {
      }
    }
}

// ---------------------------------------------------------------- a few tokens
// LM head for 2..64 token rows on the tile-packed copy, on the warp-level
// tensor cores.  A CTA takes whole 128-row tiles; per superblock its producer
// warp brings in the tile's 128 x 212 bytes (one bulk copy) and the
// superblock's activation slab (x as f16 hi + lo in B-fragment order, built
// once by k_q6gm_prep, NG x 8 KB), and each of 8 MMA warps runs its 16 rows
// against every token group: per sub-block of 16 elements, for each group of 8
// tokens, two m16n8k16 MMAs (x hi, x lo) and the sub-block's scale d * sc
// applied to the four results in f32.  A = q - 32 (exact in f16), the k order
// inside a sub-block permuted on A and B alike as in k_q6gv.
constexpr int kMW = 8;                      // MMA warps (16 rows each)
constexpr int kMWS = 3;                     // weight stages
constexpr int kMXS = 2;                     // activation stages
constexpr int kMStage = kQM * kPk;          // 27136 bytes
constexpr int kMXSlab = 16 * 8 * 32 * 16;   // one superblock, 8 groups: 64 KB

// xp[sb][s16][q][lane] = {hi(x[8q + g][k], x[..][k + 1]), hi(+2, +3), lo(..), lo(..)},
// k = 256 sb + 16 s16 + 4 t, lane = 4 g + t; zero for tokens >= n.
__global__ void k_q6gm_prep(const float* __restrict__ x, uint4* __restrict__ xp, int n, int N, int NG) {
  pdl_wait();
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t total = (size_t)(N / 16) * NG * 32;
  if (idx >= total) return;
  const int lane = (int)(idx & 31);
  const size_t sq = idx >> 5;
  const int q = (int)(sq % NG);
  const int s = (int)(sq / NG);                   // global sub-block: 16 sb + s16
  const int tok = 8 * q + (lane >> 2), k = 16 * s + 4 * (lane & 3);
  uint16_t h[4] = {0, 0, 0, 0}, l[4] = {0, 0, 0, 0};
  if (tok < n) {
    const float4 v = *reinterpret_cast<const float4*>(x + (size_t)tok * N + k);
    const float f[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const __half hh = __float2half_rn(f[i]);
      h[i] = __half_as_ushort(hh);
      l[i] = f2h(f[i] - __half2float(hh));
    }
  }
  xp[idx] = make_uint4(pack_h2(h[0], h[1]), pack_h2(h[2], h[3]), pack_h2(l[0], l[1]), pack_h2(l[2], l[3]));
}

template <int NG>   // token groups of 8 (n <= 8 NG)
__global__ void __launch_bounds__(32 * (kMW + 1), 1) k_q6gm(const uint8_t* __restrict__ wt, const uint4* __restrict__ xp,
                                                          float* __restrict__ y, int N, int OUT, int n, float softcap,
                                                          uint32_t* status) {
  extern __shared__ __align__(16) uint8_t msm[];
  __shared__ __align__(8) uint64_t wfull[kMWS], wempty[kMWS], xfull[kMXS], xempty[kMXS];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int nsb = N >> 8, ntiles = (OUT + kQM - 1) / kQM;
  const uint32_t xbytes = (uint32_t)NG * (kMXSlab / 8);
  uint8_t* wring = msm;                                       // [kMWS][27136]
  uint8_t* xring = msm + (size_t)kMWS * kMStage;              // [kMXS][xbytes = NG x 8 KB]
  if (threadIdx.x == 0) {
    for (int i = 0; i < kMWS; i++) {
      mbar_init(&wfull[i], 1);
      mbar_init(&wempty[i], kMW);
    }
    for (int i = 0; i < kMXS; i++) {
      mbar_init(&xfull[i], 1);
      mbar_init(&xempty[i], kMW);
    }
    fence_barrier_init();
  }
  __syncthreads();
  const int mytiles = (int)blockIdx.x < ntiles ? (ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
  const int steps = mytiles * nsb;
  if (warp == kMW) {
    // ---------------- producer: weights (which need nothing from the previous kernel) and activation slabs
    if (lane == 0) {
      bool ok = true;
      for (int k = 0; k < steps && ok; k++) {
        const int tile = (int)blockIdx.x + (k / nsb) * (int)gridDim.x, sb = k % nsb;
        const int ws = k % kMWS, xs = k % kMXS;
        if (k >= kMWS) ok = mbar_wait(&wempty[ws], (uint32_t)(((k / kMWS) - 1) & 1), status);
        if (!ok) break;
        mbar_expect_tx(&wfull[ws], (uint32_t)kMStage);
        bulk_g2s(wring + (size_t)ws * kMStage, wt + ((size_t)tile * nsb + sb) * kMStage, (uint32_t)kMStage, &wfull[ws]);
        if (k == 0) pdl_wait();          // the activation slabs come from the previous kernel
        if (k >= kMXS) ok = mbar_wait(&xempty[xs], (uint32_t)(((k / kMXS) - 1) & 1), status);
        if (!ok) break;
        mbar_expect_tx(&xfull[xs], xbytes);
        bulk_g2s(xring + (size_t)xs * xbytes, xp + (size_t)sb * 16 * NG * 32, xbytes, &xfull[xs]);
      }
      if (steps == 0) pdl_wait();
    }
    return;
  }
  // ---------------- MMA warps: rows 16 warp + g and + 8 of the tile
  const int ra = (16 * warp + g) * kPk, rb = ra + 8 * kPk;
  bool ok = true;
  int k = 0;
  for (int j = 0; j < mytiles; j++) {
    const int tile = (int)blockIdx.x + j * (int)gridDim.x;
    float acc[NG][4];
#pragma unroll
    for (int q = 0; q < NG; q++) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
    for (int sb = 0; sb < nsb; sb++, k++) {
      const int ws = k % kMWS, xs = k % kMXS;
      if (ok) ok = mbar_wait(&wfull[ws], (uint32_t)((k / kMWS) & 1), status);
      if (ok) ok = mbar_wait(&xfull[xs], (uint32_t)((k / kMXS) & 1), status);
      ok = __all_sync(0xffffffffu, ok);      // the MMAs below need the whole warp on one path
      if (ok) {
        const uint8_t* sg = wring + (size_t)ws * kMStage;
        const uint4* xsl = reinterpret_cast<const uint4*>(xring + (size_t)xs * xbytes);
        const float da = h2f(*reinterpret_cast<const uint16_t*>(sg + ra + 208));
        const float db = h2f(*reinterpret_cast<const uint16_t*>(sg + rb + 208));
#pragma unroll
        for (int h = 0; h < 2; h++) {
          uint32_t qla[4], qlb[4], qha[2], qhb[2];
#pragma unroll
          for (int q = 0; q < 4; q++) {
            const int o = 64 * h + 32 * (q >> 1) + 16 * (q & 1) + 4 * t;
            qla[q] = *reinterpret_cast<const uint32_t*>(sg + ra + o);
            qlb[q] = *reinterpret_cast<const uint32_t*>(sg + rb + o);
          }
#pragma unroll
          for (int lh = 0; lh < 2; lh++) {
            const int o = 128 + 32 * h + 16 * lh + 4 * t;
            qha[lh] = *reinterpret_cast<const uint32_t*>(sg + ra + o);
            qhb[lh] = *reinterpret_cast<const uint32_t*>(sg + rb + o);
          }
          // the half's 8 scales of rows g and g + 8
          const uint2 sca = make_uint2(*reinterpret_cast<const uint32_t*>(sg + ra + 192 + 8 * h),
                                       *reinterpret_cast<const uint32_t*>(sg + ra + 196 + 8 * h));
          const uint2 scb = make_uint2(*reinterpret_cast<const uint32_t*>(sg + rb + 192 + 8 * h),
                                       *reinterpret_cast<const uint32_t*>(sg + rb + 196 + 8 * h));
#pragma unroll
          for (int jb = 0; jb < 8; jb++) {
            const int jj = jb >> 1, lh = jb & 1, q = 2 * (jj & 1) + lh;
            uint32_t a01, a23, b01, b23;
            q6_word(qla[q], qha[lh], jj >= 2, 2 * jj, a01, a23);
            q6_word(qlb[q], qhb[lh], jj >= 2, 2 * jj, b01, b23);
            const uint32_t wa = jb < 4 ? sca.x : sca.y, wb = jb < 4 ? scb.x : scb.y;
            const float sa = da * (float)(int8_t)((wa >> (8 * (jb & 3))) & 0xFFu);
            const float sbb = db * (float)(int8_t)((wb >> (8 * (jb & 3))) & 0xFFu);
            const uint4* xq = xsl + (size_t)(8 * h + jb) * NG * 32 + lane;
#pragma unroll
            for (int q2 = 0; q2 < NG; q2++) {
              const uint4 xv = xq[q2 * 32];
              float c[4] = {0.f, 0.f, 0.f, 0.f};
              mma16816(c, a01, b01, a23, b23, xv.x, xv.y);
              mma16816(c, a01, b01, a23, b23, xv.z, xv.w);
              acc[q2][0] = fmaf(sa, c[0], acc[q2][0]);
              acc[q2][1] = fmaf(sa, c[1], acc[q2][1]);
              acc[q2][2] = fmaf(sbb, c[2], acc[q2][2]);
              acc[q2][3] = fmaf(sbb, c[3], acc[q2][3]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&wempty[ws]);
        mbar_arrive(&xempty[xs]);
      }
    }
    if (!ok) continue;
    // c[0], c[1]: row g, tokens 8 q + 2 t, + 1; c[2], c[3]: row g + 8
    const int row = tile * kQM + 16 * warp + g;
#pragma unroll
    for (int q2 = 0; q2 < NG; q2++)
#pragma unroll
      for (int r = 0; r < 4; r++) {
        const int rr = row + 8 * (r >> 1), tok = 8 * q2 + 2 * t + (r & 1);
        if (rr < OUT && tok < n) {
          const float v = acc[q2][r];
          y[(size_t)tok * OUT + rr] = softcap != 0.f ? softcap * tanhf(v / softcap) : v;
        }
      }
  }
}

}  // namespace

namespace e4b {

bool q6tc_supported(const uint8_t* w, const void* scratch, int N, int OUT, int n) {
  return n >= 1 && n <= kQMaxNP && N % 256 == 0 && OUT % 8 == 0 && reinterpret_cast<uintptr_t>(w) % 16 == 0 &&
         reinterpret_cast<uintptr_t>(scratch) % 16 == 0;
}

size_t q6_packed_bytes(int N, int OUT) { return (size_t)((OUT + kQM - 1) / kQM) * (N / 256) * kQM * kPk; }

// scratch: 2 * NP * N halves (NP = 32 for n <= 32, else 64).
int q6tc_lmhead(e4b_ctx* c, const uint8_t* w, bool packed, const float* x, uint16_t* scratch, float* y, int N,
                int OUT, float softcap, int n) {
  const int NP = n <= 32 ? 32 : 64;
  const size_t tot = (size_t)NP * N;
  if (int r = e4b_launch(c, "q6tc_prep", k_q6tc_prep, dim3((unsigned)((tot + 255) / 256)), dim3(256), 0, x, scratch,
                         n, N, NP))
    return r;
  auto enc = tensor_map_encoder();
  if (!enc) return e4b_fail(c, E4B_ECUDA, "q6tc: cuTensorMapEncodeTiled unavailable");
  CUtensorMap xmap;
  const cuuint64_t dim[2] = {(cuuint64_t)N, (cuuint64_t)(2 * NP)};
  const cuuint64_t stride[1] = {(cuuint64_t)N * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kQK, (cuuint32_t)(2 * NP)};
  const cuuint32_t es[2] = {1, 1};
  if (enc(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, scratch, dim, stride, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return e4b_fail(c, E4B_ECUDA, "q6tc: tensor map encode failed (N=%d)", N);
  Q6P p;
  p.w = w;
  p.rowbytes = (N / 256) * 210;
  p.w_end = w + (packed ? q6_packed_bytes(N, OUT) : (size_t)OUT * p.rowbytes);
  p.y = y;
  p.status = c->status;
  p.N = N;
  p.OUT = OUT;
  p.n = n;
  p.NP = NP;
  p.nsb = N / 256;
  p.ntiles = (OUT + kQM - 1) / kQM;
  p.softcap = softcap;
  p.wait_ns = c->wait_ns;
  auto launch = [&](auto kern) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kQSmemBytes);
    if (e != cudaSuccess) return e4b_fail(c, E4B_ECUDA, "q6tc smem attr: %s", cudaGetErrorString(e));
    const int grid = p.ntiles < c->sm_count ? p.ntiles : c->sm_count;
    return e4b_launch(c, "q6tc", kern, dim3((unsigned)grid), dim3(kQThreads), kQSmemBytes, p, xmap);
  };
  return packed ? launch(k_q6tc<true>) : launch(k_q6tc<false>);
}

int q6_pack(e4b_ctx* c, const uint8_t* w, uint8_t* wt, int N, int OUT) {
  const size_t total = q6_packed_bytes(N, OUT) / 2;
  return e4b_launch(c, "q6_pack", k_q6_pack, dim3((unsigned)((total + 255) / 256)), dim3(256), 0,
                    reinterpret_cast<const uint16_t*>(w), reinterpret_cast<uint16_t*>(wt), OUT, N / 256, total);
}

}  // namespace e4b

extern "C" {

E4B_API size_t e4b_q6k_packed_bytes(int N, int OUT) {
  return N > 0 && N % 256 == 0 && OUT > 0 ? e4b::q6_packed_bytes(N, OUT) : 0;
}

E4B_API int e4b_q6k_pack_tiles(e4b_ctx* c, const uint8_t* w, uint8_t* wt, int N, int OUT) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, w && wt && N > 0 && N % 256 == 0 && OUT > 0, "q6k_pack_tiles: bad args (N=%d OUT=%d)", N, OUT);
  E4B_REQUIRE(c, reinterpret_cast<uintptr_t>(w) % 2 == 0 && reinterpret_cast<uintptr_t>(wt) % 16 == 0,
              "q6k_pack_tiles: w must be 2-byte and wt 16-byte aligned");
  return e4b::q6_pack(c, w, wt, N, OUT);
}

E4B_API int e4b_q6k_lmhead_tiles(e4b_ctx* c, const uint8_t* wt, const float* x, uint16_t* scratch, float* y, int N,
                                 int OUT, float softcap, int n) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, wt && x && y && N > 0 && N % 256 == 0 && OUT > 0, "q6k_lmhead_tiles: bad args");
  E4B_REQUIRE(c, n >= 1 && n <= kQMaxNP, "q6k_lmhead_tiles: n=%d must be 1..%d", n, kQMaxNP);
  E4B_REQUIRE(c, reinterpret_cast<uintptr_t>(wt) % 16 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0,
              "q6k_lmhead_tiles: wt and x must be 16-byte aligned");
  if (n == 1) {
    // one token: the warp-level GEMV (k_q6gv), no scratch
    const size_t smem = (size_t)N * 4 + (size_t)kGW * kGS * kGStage;
    E4B_REQUIRE(c, smem <= 227 * 1024, "q6k_lmhead_tiles: N=%d too large for one token's staged x", N);
    cudaError_t e = cudaFuncSetAttribute(k_q6gv, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e4b_fail(c, E4B_ECUDA, "q6gv smem attr: %s", cudaGetErrorString(e));
    return e4b_launch(c, "q6gv", k_q6gv, dim3((unsigned)c->sm_count), dim3(32 * kGW), smem, wt, x, y, N, OUT, softcap,
                      c->status, c->wait_ns);
  }
  E4B_REQUIRE(c, scratch && reinterpret_cast<uintptr_t>(scratch) % 16 == 0,
              "q6k_lmhead_tiles: scratch must be 16-byte aligned");
  // measured (A4B shape): the warp-MMA kernel wins up to 32 rows, the tcgen05 one above
  const bool tc = c->lmhead_tiles_tc == 1 || (c->lmhead_tiles_tc == 0 && n > 32);
  if (tc) return e4b::q6tc_lmhead(c, wt, true, x, scratch, y, N, OUT, softcap, n);
  // a few tokens: the warp-MMA kernel over activation slabs built once into scratch
  const int NG = n <= 8 ? 1 : (n <= 16 ? 2 : (n <= 32 ? 4 : 8));
  const size_t tot = (size_t)(N / 16) * NG * 32;
  uint4* xp = reinterpret_cast<uint4*>(scratch);
  if (int r = e4b_launch(c, "q6gm_prep", k_q6gm_prep, dim3((unsigned)((tot + 255) / 256)), dim3(256), 0, x, xp, n, N,
                         NG))
    return r;
  const size_t smem = (size_t)kMWS * kMStage + (size_t)kMXS * NG * (kMXSlab / 8);
  const int ntiles = (OUT + kQM - 1) / kQM;
  const int grid = ntiles < c->sm_count ? ntiles : c->sm_count;
  auto launch = [&](auto kern) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e4b_fail(c, E4B_ECUDA, "q6gm smem attr: %s", cudaGetErrorString(e));
    return e4b_launch(c, "q6gm", kern, dim3((unsigned)grid), dim3(32 * (kMW + 1)), smem, wt, (const uint4*)xp, y, N,
                      OUT, n, softcap, c->status);
  };
  if (NG == 1) return launch(k_q6gm<1>);
  if (NG == 2) return launch(k_q6gm<2>);
  if (NG == 4) return launch(k_q6gm<4>);
  return launch(k_q6gm<8>);
}

}  // extern "C"
