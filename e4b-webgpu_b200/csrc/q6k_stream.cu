// Streaming q6_K LM head (kernels/q6k.wgsl MODE 1 + softcap) for bs1 decode.
//
// y[o] = softcap * tanh((sum_b d[o][b] sum_s sc[o][b][s] sum_{i in s} (q-32) x[i]) / softcap)
// over the raw GGUF q6_K rows (210-byte blocks of 256 weights).
//
// Data movement: every warp owns a strided set of rows and a private ring of
// row-sized shared-memory stages filled by 1-D TMA bulk copies (cp.async.bulk,
// whole rows: 8 blocks = 1680 B for hidden 2048), so the weight stream is
// issued ahead of the math and never touches the register file.  x sits in
// shared memory (f32).
//
// Math: lane l owns, in every block, the 4 ql bytes of word l and the matching
// qh word; they hold 8 weights in two sub-blocks (lo / hi nibbles):
//   h = l / 16, j = (l / 8) % 2, l' = 4 (l % 8) + k, k = 0..3
//   lo nibble: element 128h + 32j + l'        (qh bits 2j)
//   hi nibble: element 128h + 32(j+2) + l'    (qh bits 2j+4)
// The 6-bit values are assembled four at a time with byte-parallel masks,
// turned into exact f32 (q - 32) with the 2^23 magic-number trick, multiplied
// by x in f32, and scaled per sub-block by sc * d (kernels/q6k.wgsl:44-68).
#include "q40_stream.cuh"
#include "stream.cuh"

namespace {
using namespace e4b;

constexpr int kLW = 8;     // warps per CTA
constexpr int kLS = 6;     // row stages per warp

__global__ void __launch_bounds__(32 * kLW, 2) k_lmhead_stream(const uint8_t* __restrict__ w, const float* __restrict__ x,
                                                                float* __restrict__ y, int N, int OUT, float softcap,
                                                                uint32_t* status) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kLW][kLS];
  const int nb = N >> 8, rowbytes = nb * 210;
  float* xs = reinterpret_cast<float*>(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* ring = smem + (size_t)N * 4 + (size_t)warp * kLS * rowbytes;
  const int GW = gridDim.x * kLW, gw = blockIdx.x * kLW + warp;
  const int nr = OUT > gw ? (OUT - gw + GW - 1) / GW : 0;

  pdl_trigger();
  if (lane == 0) {
    for (int s = 0; s < kLS; s++) mbar_init(&full[warp][s], 1);
    fence_barrier_init();
  }
  __syncwarp();
  // weights never depend on the previous kernel: start the stream first
  if (lane == 0)
    for (int s = 0; s < kLS && s < nr; s++) {
      mbar_expect_tx(&full[warp][s], (uint32_t)rowbytes);
      bulk_g2s(ring + (size_t)s * rowbytes, w + (size_t)(gw + (size_t)GW * s) * rowbytes, (uint32_t)rowbytes,
               &full[warp][s]);
    }
  pdl_wait();
  for (int i = threadIdx.x; i < N / 4; i += blockDim.x)
    reinterpret_cast<float4*>(xs)[i] = reinterpret_cast<const float4*>(x)[i];
  __syncthreads();

  const int h = lane >> 4, jb = (lane >> 3) & 1, l8 = lane & 7;
  const int qi = 8 * h + l8;                       // qh word
  const int sb = 8 * h + 2 * jb + (l8 >> 2);       // sub-block of the lo nibbles (hi: sb + 4)
  const int xo = 128 * h + 32 * jb + 4 * l8;       // element of lo nibble k = 0 (hi: + 64)
  const int sh_lo = 2 * jb, sh_hi = 2 * jb + 4;
  const float kMagic = 8388640.0f;                 // 2^23 + 32: (2^23 + q) - kMagic = q - 32
  bool ok = true;
  for (int i = 0; i < nr; i++) {
    const int s = i % kLS;
    if (ok) ok = mbar_wait(&full[warp][s], (uint32_t)((i / kLS) & 1), status);
    const uint8_t* row = ring + (size_t)s * rowbytes;
    float acc = 0.f;
    if (ok) {
#pragma unroll 2
      for (int b = 0; b < nb; b++) {
        const uint8_t* blk = row + 210 * b;
        uint32_t wq, wh;
        if ((b & 1) == 0) {
          wq = *reinterpret_cast<const uint32_t*>(blk + 4 * lane);
          wh = *reinterpret_cast<const uint32_t*>(blk + 128 + 4 * qi);
        } else {   // odd blocks start 2 bytes past a word boundary
          const uint32_t* a = reinterpret_cast<const uint32_t*>(blk - 2 + 4 * lane);
          const uint32_t* c = reinterpret_cast<const uint32_t*>(blk + 126 + 4 * qi);
          wq = __byte_perm(a[0], a[1], 0x5432);
          wh = __byte_perm(c[0], c[1], 0x5432);
        }
        const uint32_t qlo = (wq & 0x0F0F0F0Fu) | (((wh >> sh_lo) & 0x03030303u) << 4);
        const uint32_t qhi = ((wq >> 4) & 0x0F0F0F0Fu) | (((wh >> sh_hi) & 0x03030303u) << 4);
        const float4 xl = *reinterpret_cast<const float4*>(xs + 256 * b + xo);
        const float4 xh = *reinterpret_cast<const float4*>(xs + 256 * b + xo + 64);
        float slo = (__int_as_float(__byte_perm(qlo, 0x4B000000u, 0x7540)) - kMagic) * xl.x;
        slo = fmaf(__int_as_float(__byte_perm(qlo, 0x4B000000u, 0x7541)) - kMagic, xl.y, slo);
        slo = fmaf(__int_as_float(__byte_perm(qlo, 0x4B000000u, 0x7542)) - kMagic, xl.z, slo);
        slo = fmaf(__int_as_float(__byte_perm(qlo, 0x4B000000u, 0x7543)) - kMagic, xl.w, slo);
        float shi = (__int_as_float(__byte_perm(qhi, 0x4B000000u, 0x7540)) - kMagic) * xh.x;
        shi = fmaf(__int_as_float(__byte_perm(qhi, 0x4B000000u, 0x7541)) - kMagic, xh.y, shi);
        shi = fmaf(__int_as_float(__byte_perm(qhi, 0x4B000000u, 0x7542)) - kMagic, xh.z, shi);
        shi = fmaf(__int_as_float(__byte_perm(qhi, 0x4B000000u, 0x7543)) - kMagic, xh.w, shi);
        const float d = h2f(*reinterpret_cast<const uint16_t*>(blk + 208));
        const float sl = (float)(int8_t)blk[192 + sb], shh = (float)(int8_t)blk[196 + sb];
        acc = fmaf(d, fmaf(sl, slo, shh * shi), acc);
      }
    }
    acc = warp_sum(acc);
    const int r = gw + GW * i;
    if (lane == 0 && ok) y[r] = softcap != 0.f ? softcap * tanhf(acc / softcap) : acc;
    // every lane's reads of the stage are done before it is refilled
    __syncwarp();
    if (lane == 0 && ok && i + kLS < nr) {
      mbar_expect_tx(&full[warp][s], (uint32_t)rowbytes);
      bulk_g2s(ring + (size_t)s * rowbytes, w + (size_t)(gw + (size_t)GW * (i + kLS)) * rowbytes, (uint32_t)rowbytes,
               &full[warp][s]);
    }
  }
}

}  // namespace

namespace e4b {

bool lmhead_stream_supported(const uint8_t* w, const float* x, int N) {
  return N > 0 && N % 2048 == 0 && N <= 8192 && reinterpret_cast<uintptr_t>(w) % 16 == 0 &&
         reinterpret_cast<uintptr_t>(x) % 16 == 0;
}

int lmhead_stream(e4b_ctx* c, const uint8_t* w, const float* x, float* y, int N, int OUT, float softcap) {
  const int rowbytes = N / 256 * 210;
  const size_t smem = (size_t)N * 4 + (size_t)kLW * kLS * rowbytes;
  cudaError_t e = cudaFuncSetAttribute(k_lmhead_stream, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e4b_fail(c, E4B_ECUDA, "lmhead smem attr: %s", cudaGetErrorString(e));
  int per_sm = 1;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_lmhead_stream, 32 * kLW, smem);
  if (per_sm < 1) per_sm = 1;
  if (per_sm > 2) per_sm = 2;
  int G = c->sm_count * per_sm;
  const int need = (OUT + kLW - 1) / kLW;
  if (G > need) G = need;
  return e4b_launch(c, "q6k_lmhead_stream", k_lmhead_stream, dim3((unsigned)G), dim3(32 * kLW), smem, w, x, y, N,
                    OUT, softcap, c->status);
}

}  // namespace e4b

// ---- batched LM head: n token rows of x against every q6_K row, on the tensor
// cores (mma.sync m16n8k16, tokens as the 8 columns).  A k16 step is exactly one
// q6_K sub-block (16 weights sharing an int8 scale), so each step's products are
// scaled by sc * d in f32 and accumulated.  A = (q - 32) in f16 (exact); x is
// used as f16 hi + lo (x = hi + lo to ~2^-22), so the products carry f32-level
// precision.  One warp = 16 rows x all tokens.
namespace {

__global__ void k_split_f32(const float* __restrict__ x, uint16_t* __restrict__ hi, uint16_t* __restrict__ lo,
                            size_t n) {
  pdl_wait();
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float v = x[i];
  const __half h = __float2half_rn(v);
  hi[i] = __half_as_ushort(h);
  lo[i] = f2h(v - __half2float(h));
}

// f16x2 of (q(e) - 32, q(e+1) - 32) for elements e (even) and e+1 of a q6_K block.
E4B_DEV uint32_t q6_pair(const uint8_t* blk, int e) {
  const int h = e >> 7, r = e & 127, jj = r >> 5, l = r & 31;
  const uint32_t ql = *reinterpret_cast<const uint16_t*>(blk + h * 64 + l + 32 * (jj & 1));
  const uint32_t qh = *reinterpret_cast<const uint16_t*>(blk + 128 + h * 32 + l);
  const uint32_t lo = (ql >> (4 * (jj >> 1))) & 0x0F0Fu;           // both bytes' nibble
  const uint32_t hi = ((qh >> (2 * jj)) & 0x0303u) << 4;
  const uint32_t q = lo | hi;                                        // two 6-bit values, one per byte
  const uint32_t f = __byte_perm(q, 0x64646464u, 0x5140);            // 0x64qq halves = 1024 + q
  uint32_t r16;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r16) : "r"(f), "r"(0x64206420u));   // - 1056 -> q - 32
  return r16;
}

template <int NG>
__global__ void __launch_bounds__(256) k_q6k_mm(const uint8_t* __restrict__ w, const uint16_t* __restrict__ xh,
                                                const uint16_t* __restrict__ xl, float* __restrict__ y, int N, int OUT,
                                                int n, float softcap) {
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int r0 = (blockIdx.x * 8 + warp) * 16;
  if (r0 >= OUT) return;
  const int nb = N >> 8;
  const int ra = min(r0 + g, OUT - 1), rb = min(r0 + g + 8, OUT - 1);
  const uint8_t* wa = w + (size_t)ra * nb * 210;
  const uint8_t* wb = w + (size_t)rb * nb * 210;
  for (int g0 = 0; g0 < n; g0 += 8 * NG) {
    float acc[NG][4];
#pragma unroll
    for (int q = 0; q < NG; q++) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
    // this lane's token (column g) per group
    const uint16_t* xhr[NG];
    const uint16_t* xlr[NG];
#pragma unroll
    for (int q = 0; q < NG; q++) {
      const int tok = g0 + 8 * q + g;
      xhr[q] = tok < n ? xh + (size_t)tok * N : nullptr;
      xlr[q] = tok < n ? xl + (size_t)tok * N : nullptr;
    }
    for (int b = 0; b < nb; b++) {
      const uint8_t* ba = wa + (size_t)b * 210;
      const uint8_t* bb = wb + (size_t)b * 210;
      const float da = h2f(*reinterpret_cast<const uint16_t*>(ba + 208));
      const float db = h2f(*reinterpret_cast<const uint16_t*>(bb + 208));
      for (int sb = 0; sb < 16; sb++) {
        const int e0 = 16 * sb + 2 * t;
        const uint32_t a0 = q6_pair(ba, e0), a1 = q6_pair(bb, e0), a2 = q6_pair(ba, e0 + 8), a3 = q6_pair(bb, e0 + 8);
        const float sa = da * (float)(int8_t)ba[192 + sb], sbb = db * (float)(int8_t)bb[192 + sb];
        const int xo = 256 * b + e0;
#pragma unroll
        for (int q = 0; q < NG; q++) {
          if (g0 + 8 * q >= n) break;
          uint32_t h0 = 0, h1 = 0, l0 = 0, l1 = 0;
          if (xhr[q]) {
            h0 = *reinterpret_cast<const uint32_t*>(xhr[q] + xo);
            h1 = *reinterpret_cast<const uint32_t*>(xhr[q] + xo + 8);
            l0 = *reinterpret_cast<const uint32_t*>(xlr[q] + xo);
            l1 = *reinterpret_cast<const uint32_t*>(xlr[q] + xo + 8);
          }
          float c[4] = {0.f, 0.f, 0.f, 0.f};
          mma16816(c, a0, a1, a2, a3, h0, h1);
          mma16816(c, a0, a1, a2, a3, l0, l1);
          acc[q][0] = fmaf(sa, c[0], acc[q][0]);
          acc[q][1] = fmaf(sa, c[1], acc[q][1]);
          acc[q][2] = fmaf(sbb, c[2], acc[q][2]);
          acc[q][3] = fmaf(sbb, c[3], acc[q][3]);
        }
      }
    }
    // C: c0, c1 = row g, tokens 2t, 2t+1; c2, c3 = row g+8
#pragma unroll
    for (int q = 0; q < NG; q++) {
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int row = r0 + g + (i >> 1) * 8, tok = g0 + 8 * q + 2 * t + (i & 1);
        if (row < OUT && tok < n) {
          const float v = acc[q][i];
          y[(size_t)tok * OUT + row] = softcap != 0.f ? softcap * tanhf(v / softcap) : v;
        }
      }
    }
  }
}

// ---- batched LM head, persistent and staged.  A unit is (block of 128 rows,
// pass of up to 64 tokens); per q6_K superblock (256 k) a producer warp copies
// the pass's activations (pre-split into f16 hi / lo and laid out as the MMA
// B fragments: k_q6x_prep) with one bulk copy into a 2-deep ring shared by the
// CTA, and each of the four MMA warps stages its own 32 rows' superblocks
// (the 16-byte-aligned 224-byte cover of each 210-byte block, 16-byte
// cp.async per piece, 3 deep); two 16-row subtiles share every B fragment.
constexpr int kLmRows = 128;
constexpr int kLmSlot = 240;                      // the 224-byte cover + 16 (row pitch off the bank period)
constexpr int kLmXSlab = 8 * 16 * 32 * 16;        // 8 token groups x 16 k-steps x 32 lanes x 16 B
constexpr int kLmWS = 3;                          // weight stages per warp
constexpr int kLmWWarp = 32 * kLmSlot;            // one warp's rows of one superblock

// xp[s][q][j][lane] = {hi(x[k], x[k+1]), hi(x[k+8], x[k+9]), lo(..), lo(..)} for
// token 8q + lane/4 and k = 256 s + 16 j + 2 (lane % 4); zero beyond n.
__global__ void k_q6x_prep(const float* __restrict__ x, uint4* __restrict__ xp, int n, int N, int NG) {
  pdl_wait();
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t total = (size_t)(N / 256) * NG * 16 * 32;
  if (idx >= total) return;
  const int lane = (int)(idx & 31), j = (int)((idx >> 5) & 15);
  const size_t sq = idx >> 9;
  const int q = (int)(sq % NG), sb = (int)(sq / NG);
  const int tok = 8 * q + (lane >> 2), k = 256 * sb + 16 * j + 2 * (lane & 3);
  uint16_t h[4] = {0, 0, 0, 0}, l[4] = {0, 0, 0, 0};
  if (tok < n) {
    const float* xr = x + (size_t)tok * N + k;
    const float v[4] = {xr[0], xr[1], xr[8], xr[9]};
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const __half hh = __float2half_rn(v[i]);
      h[i] = __half_as_ushort(hh);
      l[i] = f2h(v[i] - __half2float(hh));
    }
  }
  xp[idx] = make_uint4(pack_h2(h[0], h[1]), pack_h2(h[2], h[3]), pack_h2(l[0], l[1]), pack_h2(l[2], l[3]));
}

E4B_DEV void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
E4B_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
E4B_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int NGT>   // token groups computed per step: 1, 2, 4 or 8 (>= the pass's groups)
__global__ void __launch_bounds__(160, 1) k_q6mm(const uint8_t* __restrict__ w, const uint4* __restrict__ xp,
                                                  float* __restrict__ y, int N, int OUT, int n, int NG, float softcap,
                                                  uint32_t* status) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[2], empty[2];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nsb = N >> 8, rowbytes = nsb * 210;
  const int RB = (OUT + kLmRows - 1) / kLmRows, passes = (NG + 7) / 8, units = RB * passes;
  uint8_t* xbuf = smem;
  uint8_t* wbuf = smem + 2 * kLmXSlab + (size_t)(warp < 4 ? warp : 0) * kLmWS * kLmWWarp;
  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; b++) {
      mbar_init(&full[b], 1);
      mbar_init(&empty[b], 4);
    }
    fence_barrier_init();
  }
  __syncthreads();
  pdl_trigger();
  pdl_wait();
  if (warp == 4) {
    // producer of the activation slabs
    int seq = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      const int pass = u % passes, ng = min(8, NG - 8 * pass);
      for (int sb = 0; sb < nsb && ok; sb++, seq++) {
        const int b = seq & 1;
        if (seq >= 2) ok = mbar_wait(&empty[b], (uint32_t)(((seq >> 1) - 1) & 1), status);
        if (ok && lane == 0) {
          mbar_expect_tx(&full[b], (uint32_t)(ng * (kLmXSlab / 8)));
          bulk_g2s(xbuf + b * kLmXSlab, xp + ((size_t)sb * NG + 8 * pass) * 16 * 32, (uint32_t)(ng * (kLmXSlab / 8)),
                   &full[b]);
        }
        __syncwarp();
      }
    }
    return;
  }
  // MMA warps: rows 32 warp + {g, g+8} (subtile 0) and + 16 (subtile 1)
  const int g = lane >> 2, t = lane & 3;
  const int steps = ((units - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x) * nsb;   // this CTA's steps
  // stage step k's superblock of this lane's row (row 32 warp + lane of the block)
  auto stage_w = [&](int k) {
    const int u = blockIdx.x + (k / nsb) * gridDim.x, sb = k % nsb;
    const int row = kLmRows * (u / passes) + 32 * warp + lane;
    if (row < OUT) {
      const size_t start = (size_t)row * rowbytes + 210 * sb;
      const uint8_t* src = w + (start & ~(size_t)15);
      uint8_t* dst = wbuf + (k % kLmWS) * kLmWWarp + lane * kLmSlot;
#pragma unroll
      for (int c = 0; c < 14; c++) cp_async16(dst + 16 * c, src + 16 * c);
    }
    cp_async_commit();
  };
#pragma unroll
  for (int k = 0; k < kLmWS - 1; k++)
    if (k < steps) stage_w(k);
    else cp_async_commit();
  int seq = 0;
  bool ok = true;
  for (int u = blockIdx.x; u < units; u += gridDim.x) {
    const int rb = u / passes, pass = u % passes, ng = min(8, NG - 8 * pass);
    float acc[NGT][2][4];
#pragma unroll
    for (int q = 0; q < NGT; q++)
#pragma unroll
      for (int s = 0; s < 2; s++)
#pragma unroll
        for (int r = 0; r < 4; r++) acc[q][s][r] = 0.f;
    int rr[4];
#pragma unroll
    for (int i = 0; i < 4; i++) rr[i] = 32 * warp + g + 8 * i;   // rows g, g+8, g+16, g+24 of the block
    for (int sb = 0; sb < nsb; sb++, seq++) {
      const int b = seq & 1;
      // keep kLmWS - 1 weight stages in flight; this step's has landed after the wait
      if (seq + kLmWS - 1 < steps) stage_w(seq + kLmWS - 1);
      else cp_async_commit();
      cp_async_wait<kLmWS - 1>();
      __syncwarp();
      if (ok) ok = mbar_wait(&full[b], (uint32_t)((seq >> 1) & 1), status);
      if (ok) {
        const uint8_t* wst = wbuf + (seq % kLmWS) * kLmWWarp;
        const uint8_t* blk[4];
        float d[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const size_t start = (size_t)(kLmRows * rb + rr[i]) * rowbytes + 210 * sb;
          blk[i] = wst + (g + 8 * i) * kLmSlot + (int)(start & 15);
          d[i] = h2f(*reinterpret_cast<const uint16_t*>(blk[i] + 208));
        }
        const uint4* xs = reinterpret_cast<const uint4*>(xbuf + b * kLmXSlab);
        // NGT token groups every step (a short last pass computes unused
        // columns that are not stored), up to 16 independent MMA chains per step
#pragma unroll 2
        for (int j = 0; j < 16; j++) {
          const int e0 = 16 * j + 2 * t;
          uint32_t A[2][4];
          float sc[4];
#pragma unroll
          for (int i = 0; i < 4; i++) sc[i] = d[i] * (float)(int8_t)blk[i][192 + j];
#pragma unroll
          for (int s = 0; s < 2; s++) {
            A[s][0] = q6_pair(blk[2 * s], e0);
            A[s][1] = q6_pair(blk[2 * s + 1], e0);
            A[s][2] = q6_pair(blk[2 * s], e0 + 8);
            A[s][3] = q6_pair(blk[2 * s + 1], e0 + 8);
          }
          constexpr int HQ = NGT < 4 ? NGT : 4;
#pragma unroll
          for (int hq = 0; hq < NGT; hq += HQ) {
            // HQ token groups x 2 subtiles: independent MMA chains
            uint4 xv[HQ];
#pragma unroll
            for (int q = 0; q < HQ; q++) xv[q] = xs[((hq + q) * 16 + j) * 32 + lane];
            float c[HQ][2][4];
#pragma unroll
            for (int q = 0; q < HQ; q++)
#pragma unroll
              for (int s = 0; s < 2; s++) {
                c[q][s][0] = c[q][s][1] = c[q][s][2] = c[q][s][3] = 0.f;
                mma16816(c[q][s], A[s][0], A[s][1], A[s][2], A[s][3], xv[q].x, xv[q].y);
              }
#pragma unroll
            for (int q = 0; q < HQ; q++)
#pragma unroll
              for (int s = 0; s < 2; s++) mma16816(c[q][s], A[s][0], A[s][1], A[s][2], A[s][3], xv[q].z, xv[q].w);
#pragma unroll
            for (int q = 0; q < HQ; q++)
#pragma unroll
              for (int s = 0; s < 2; s++) {
                acc[hq + q][s][0] = fmaf(sc[2 * s], c[q][s][0], acc[hq + q][s][0]);
                acc[hq + q][s][1] = fmaf(sc[2 * s], c[q][s][1], acc[hq + q][s][1]);
                acc[hq + q][s][2] = fmaf(sc[2 * s + 1], c[q][s][2], acc[hq + q][s][2]);
                acc[hq + q][s][3] = fmaf(sc[2 * s + 1], c[q][s][3], acc[hq + q][s][3]);
              }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[b]);
    }
    if (!ok) continue;
#pragma unroll
    for (int q = 0; q < NGT; q++) {
      if (q >= ng) break;
#pragma unroll
      for (int s = 0; s < 2; s++)
#pragma unroll
        for (int r = 0; r < 4; r++) {
          const int row = kLmRows * rb + rr[2 * s + (r >> 1)];
          const int tok = 64 * pass + 8 * q + 2 * t + (r & 1);
          if (row < OUT && tok < n) {
            const float v = acc[q][s][r];
            y[(size_t)tok * OUT + row] = softcap != 0.f ? softcap * tanhf(v / softcap) : v;
          }
        }
    }
  }
  cp_async_wait<0>();
}

}  // namespace

extern "C" {

E4B_API int e4b_q6k_lmhead_rows(e4b_ctx* c, const uint8_t* w, const float* x, uint16_t* scratch, float* y, int N,
                                int OUT, float softcap, int n) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, w && x && scratch && y && N > 0 && N % 256 == 0 && OUT > 0 && n > 0, "q6k_lmhead_rows: bad args");
  if (n >= c->lmhead_tc_min && e4b::q6tc_supported(w, scratch, N, OUT, n))
    return e4b::q6tc_lmhead(c, w, false, x, scratch, y, N, OUT, softcap, n);
  if (OUT % 8 == 0 && reinterpret_cast<uintptr_t>(w) % 16 == 0 && reinterpret_cast<uintptr_t>(scratch) % 16 == 0) {
    // staged path: every superblock's aligned cover lies inside [w, w + OUT * rowbytes)
    const int NG = (n + 7) / 8;
    const size_t tot = (size_t)(N / 256) * NG * 16 * 32;
    uint4* xp = reinterpret_cast<uint4*>(scratch);
    if (int r = e4b_launch(c, "q6x_prep", k_q6x_prep, dim3((unsigned)((tot + 255) / 256)), dim3(256), 0, x, xp, n, N,
                           NG))
      return r;
    const size_t smem = 2 * (size_t)kLmXSlab + 4 * (size_t)kLmWS * kLmWWarp;
    const int units = (OUT + kLmRows - 1) / kLmRows * ((NG + 7) / 8);
    const int grid = units < c->sm_count ? units : c->sm_count;
    // groups computed per step: enough for the widest pass
    auto launch = [&](auto kern) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e4b_fail(c, E4B_ECUDA, "q6mm smem attr: %s", cudaGetErrorString(e));
      return e4b_launch(c, "q6mm", kern, dim3((unsigned)grid), dim3(160), smem, w, (const uint4*)xp, y, N, OUT, n, NG,
                        softcap, c->status);
    };
    if (NG == 1) return launch(k_q6mm<1>);
    if (NG == 2) return launch(k_q6mm<2>);
    if (NG <= 4) return launch(k_q6mm<4>);
    return launch(k_q6mm<8>);
  }
  uint16_t* xh = scratch;
  uint16_t* xl = scratch + (size_t)n * N;
  const size_t tot = (size_t)n * N;
  if (int r = e4b_launch(c, "split_f32", k_split_f32, dim3((unsigned)((tot + 255) / 256)), dim3(256), 0, x, xh, xl,
                         tot))
    return r;
  const unsigned grid = (unsigned)((OUT + 127) / 128);
  if (n <= 8)
    return e4b_launch(c, "q6k_mm", k_q6k_mm<1>, dim3(grid), dim3(256), 0, w, (const uint16_t*)xh,
                      (const uint16_t*)xl, y, N, OUT, n, softcap);
  return e4b_launch(c, "q6k_mm", k_q6k_mm<8>, dim3(grid), dim3(256), 0, w, (const uint16_t*)xh, (const uint16_t*)xl,
                    y, N, OUT, n, softcap);
}

}  // extern "C"
