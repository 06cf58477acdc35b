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
