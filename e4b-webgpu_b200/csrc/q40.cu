// q4_0 GEMV family over raw GGUF blocks: q40mv, q40gu (+GeGLU), q40moedown,
// moecomb, plegatemv.  One warp per output row, lanes striding over the row's
// 18-byte blocks, f32 accumulation, warp-shuffle reduction.
#include "common.cuh"
#include "q40_stream.cuh"

namespace {

constexpr int kWarps = 8;  // rows per CTA

template <typename XT>
E4B_DEV float q40_row_dot(const uint8_t* __restrict__ row, const XT* __restrict__ x, int nb) {
  float acc = 0.f;
  for (int j = threadIdx.x & 31; j < nb; j += 32) {
    const Q40Block b = q40_load(row + (size_t)j * 18);
    acc = fmaf(b.d, q40_dot<XT>(b, x + (size_t)j * 32), acc);
  }
  return warp_sum(acc);
}

template <typename XT>
__global__ void __launch_bounds__(kWarps * 32) k_q40mv(const XT* __restrict__ x, const uint8_t* __restrict__ w,
                                                       const uint32_t* __restrict__ topk, float* __restrict__ y,
                                                       int IN, int OUT, int expert, int xslot, int nz) {
  pdl_wait();
  const int o = blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int z = blockIdx.z, b = blockIdx.y;
  if (o >= OUT) return;
  const int nb = IN >> 5;
  size_t wblk = (size_t)o * nb;
  if (expert) wblk += (size_t)topk[(size_t)b * nz + z] * OUT * nb;
  const XT* xr = x + ((size_t)b * (xslot ? nz : 1) + (xslot ? z : 0)) * IN;
  const float acc = q40_row_dot<XT>(w + wblk * 18, xr, nb);
  if ((threadIdx.x & 31) == 0) y[((size_t)b * nz + z) * OUT + o] = acc;
}

// Fused gate+up+GeGLU: a CTA owns 4 outputs e0..e0+3 of one role (dense, or
// expert slot k): warps 0-3 compute the gate rows, warps 4-7 the up rows.
__global__ void __launch_bounds__(256) k_q40gu(const uint16_t* __restrict__ x, const uint8_t* __restrict__ w,
                                               const uint32_t* __restrict__ topk, uint16_t* __restrict__ yh,
                                               const uint16_t* __restrict__ x2, const uint8_t* __restrict__ w2,
                                               uint16_t* __restrict__ yh2, int IN, int FF, int FF2, int K,
                                               int has_dense) {
  pdl_wait();
  __shared__ float vals[8];
  const int b = blockIdx.y;
  const bool dense = has_dense && blockIdx.z == 0;
  const int slot = blockIdx.z - (has_dense ? 1 : 0);
  const int ff = dense ? FF2 : FF;
  const int e0 = blockIdx.x * 4;
  if (e0 >= ff) return;  // whole CTA exits together
  const int warp = threadIdx.x >> 5;
  const int r = (warp & 3);
  const bool up = warp >= 4;
  const int nb = IN >> 5;
  float acc = 0.f;
  if (e0 + r < ff) {
    if (dense) {
      const size_t row = (size_t)(up ? FF2 : 0) + e0 + r;
      acc = q40_row_dot<uint16_t>(w2 + row * nb * 18, x2 + (size_t)b * IN, nb);
    } else {
      const size_t e = topk[(size_t)b * K + slot];
      const size_t row = e * 2 * FF + (up ? FF : 0) + e0 + r;
      acc = q40_row_dot<uint16_t>(w + row * nb * 18, x + (size_t)b * IN, nb);
    }
  }
  if ((threadIdx.x & 31) == 0) vals[warp] = acc;
  __syncthreads();
  if (threadIdx.x < 4 && e0 + threadIdx.x < ff) {
    const float g = vals[threadIdx.x], u = vals[4 + threadIdx.x];
    const uint16_t out = f2h(gelu_tanh(g) * u);
    if (dense) yh2[(size_t)b * FF2 + e0 + threadIdx.x] = out;
    else yh[((size_t)b * K + slot) * FF + e0 + threadIdx.x] = out;
  }
}

__global__ void __launch_bounds__(kWarps * 32) k_q40moedown(const uint16_t* __restrict__ x,
                                                            const uint8_t* __restrict__ w,
                                                            const uint32_t* __restrict__ topk,
                                                            const float* __restrict__ tkw, float* __restrict__ y,
                                                            int IN, int OUT, int K) {
  pdl_wait();
  const int o = blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int b = blockIdx.y;
  if (o >= OUT) return;
  const int nb = IN >> 5;
  float acc = 0.f;
  for (int k = 0; k < K; k++) {
    const size_t e = topk[(size_t)b * K + k];
    const float s = q40_row_dot<uint16_t>(w + (e * OUT + o) * nb * 18, x + ((size_t)b * K + k) * IN, nb);
    acc = fmaf(tkw[(size_t)b * K + k], s, acc);
  }
  if ((threadIdx.x & 31) == 0) y[(size_t)b * OUT + o] = acc;
}

__global__ void k_moecomb(const float* __restrict__ slots, const float* __restrict__ tw, float* __restrict__ y,
                          int H, int K) {
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= H) return;
  float acc = 0.f;
  for (int k = 0; k < K; k++) acc = fmaf(tw[k], slots[(size_t)k * H + i], acc);
  y[i] = acc;
}

__global__ void __launch_bounds__(kWarps * 32) k_plegatemv(const uint16_t* __restrict__ x,
                                                           const uint8_t* __restrict__ w,
                                                           const float* __restrict__ ple, uint16_t* __restrict__ y,
                                                           int IN, int OUT, int off) {
  pdl_wait();
  const int o = blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (o >= OUT) return;
  const int nb = IN >> 5;
  const float acc = q40_row_dot<uint16_t>(w + (size_t)o * nb * 18, x, nb);
  if ((threadIdx.x & 31) == 0) y[o] = f2h(gelu_tanh(acc) * ple[off + o]);
}

}  // namespace

extern "C" {

E4B_API int e4b_q40mv(e4b_ctx* c, const void* x, const uint8_t* w, const uint32_t* topk, float* y, int IN,
                      int OUT, int expert, int xslot, int x_f16, int nz, int batch) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, x && w && y, "q40mv: null buffer");
  E4B_REQUIRE(c, IN > 0 && IN % 32 == 0 && OUT > 0, "q40mv: IN=%d must be a positive multiple of 32, OUT=%d", IN,
              OUT);
  E4B_REQUIRE(c, !expert || topk, "q40mv: expert=1 needs topk");
  if (nz < 1) nz = 1;
  if (batch < 1) batch = 1;
  if (!expert && !xslot && nz == 1 && batch == 1 && c->ws && e4b::q40_stream_supported(w, x, IN, OUT))
    return e4b::q40_stream(c, w, x, !x_f16, y, nullptr, nullptr, IN, OUT, 0, 0, 0);
  dim3 grid((OUT + kWarps - 1) / kWarps, batch, nz);
  if (x_f16)
    return e4b_launch(c, "q40mv", k_q40mv<uint16_t>, grid, dim3(kWarps * 32), 0, (const uint16_t*)x, w, topk, y,
                      IN, OUT, expert, xslot, nz);
  return e4b_launch(c, "q40mv", k_q40mv<float>, grid, dim3(kWarps * 32), 0, (const float*)x, w, topk, y, IN, OUT,
                    expert, xslot, nz);
}

E4B_API int e4b_q40gu(e4b_ctx* c, const uint16_t* x, const uint8_t* w, const uint32_t* topk, uint16_t* yh,
                      const uint16_t* x2, const uint8_t* w2, uint16_t* yh2, int IN, int FF, int FF2, int K,
                      int batch) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, IN > 0 && IN % 32 == 0, "q40gu: IN=%d must be a positive multiple of 32", IN);
  const int has_dense = w2 != nullptr;
  E4B_REQUIRE(c, !has_dense || (x2 && yh2 && FF2 > 0), "q40gu: dense part needs x2, yh2, FF2");
  E4B_REQUIRE(c, K == 0 || (x && w && topk && yh && FF > 0), "q40gu: expert part needs x, w, topk, yh, FF");
  if (batch < 1) batch = 1;
  const int nzz = has_dense + K;
  if (nzz == 0) return E4B_OK;
  if (has_dense && K == 0 && batch == 1 && c->ws && FF2 % 16 == 0 && e4b::q40_stream_supported(w2, x2, IN, FF2))
    return e4b::q40_stream(c, w2, x2, 0, nullptr, yh2, nullptr, IN, 2 * FF2, 1, FF2, 0);
  const int ffmax = has_dense ? (FF2 > FF ? FF2 : FF) : FF;
  dim3 grid((ffmax + 3) / 4, batch, nzz);
  return e4b_launch(c, "q40gu", k_q40gu, grid, dim3(256), 0, x, w, topk, yh, x2, w2, yh2, IN, FF, FF2, K,
                    has_dense);
}

E4B_API int e4b_q40moedown(e4b_ctx* c, const uint16_t* x, const uint8_t* w, const uint32_t* topk, const float* tkw,
                           float* y, int IN, int OUT, int K, int batch) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, x && w && topk && tkw && y, "q40moedown: null buffer");
  E4B_REQUIRE(c, IN > 0 && IN % 32 == 0 && OUT > 0 && K > 0, "q40moedown: bad sizes IN=%d OUT=%d K=%d", IN, OUT,
              K);
  if (batch < 1) batch = 1;
  dim3 grid((OUT + kWarps - 1) / kWarps, batch);
  return e4b_launch(c, "q40moedown", k_q40moedown, grid, dim3(kWarps * 32), 0, x, w, topk, tkw, y, IN, OUT, K);
}

E4B_API int e4b_moecomb(e4b_ctx* c, const float* slots, const float* topk_w, float* y, int H, int K) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, slots && topk_w && y && H > 0 && K > 0, "moecomb: bad args");
  return e4b_launch(c, "moecomb", k_moecomb, dim3((H + 255) / 256), dim3(256), 0, slots, topk_w, y, H, K);
}

E4B_API int e4b_plegatemv(e4b_ctx* c, const uint16_t* x, const uint8_t* w, const float* ple, uint16_t* y, int IN,
                          int OUT, int off) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, x && w && ple && y, "plegatemv: null buffer");
  E4B_REQUIRE(c, IN > 0 && IN % 32 == 0 && OUT > 0 && off >= 0, "plegatemv: bad sizes");
  if (c->ws && e4b::q40_stream_supported(w, x, IN, OUT))
    return e4b::q40_stream(c, w, x, 0, nullptr, y, ple, IN, OUT, 2, 0, off);
  return e4b_launch(c, "plegatemv", k_plegatemv, dim3((OUT + kWarps - 1) / kWarps), dim3(kWarps * 32), 0, x, w,
                    ple, y, IN, OUT, off);
}

}  // extern "C"
