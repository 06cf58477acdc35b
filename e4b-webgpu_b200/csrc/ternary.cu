// Ternary MoE experts (the reference's Campaign-6 format, kernels/t2gu.wgsl and
// kernels/t2moedown.wgsl; conversion in scripts/ternarize_a4b.py): every expert
// row is t[i] in {-1, 0, 1} times ONE f16 row scale alpha.  Storage: 2-bit
// planes, 16 values per u32 in the shift-group layout -- element 4g + j of a
// word (group g, byte lane j) sits at bits 2g + 8j and holds t + 1 -- so
// (w >> 2g) & 0x03030303 yields four consecutive elements as bytes.
//
//   t2gu:      for expert slot k (expert e = topk[k]) and row i < FF,
//              g = alpha[e][i] * sum t[e][i] . x,  u = alpha[e][FF+i] * sum t[e][FF+i] . x,
//              yh[k][i] = f16(gelu(g) * u)                       (t2gu.wgsl expert branch)
//   t2moedown: y[o] = sum_k w_k * alpha[e_k][o] * sum t[e_k][o] . x_k   (t2moedown.wgsl)
//
// One warp per output row (pair); lanes stride over the row's words, f32
// partial sums reduced with shuffles.  Both are HBM-bound on the 2-bit planes.
#include "common.cuh"

namespace {

// sum over the 16 elements of word w (t = value - 1) times x[16 q .. 16 q + 15]
E4B_DEV float t2dot16(uint32_t w, const uint16_t* __restrict__ x) {
  const uint4 xv0 = *reinterpret_cast<const uint4*>(x);
  const uint4 xv1 = *reinterpret_cast<const uint4*>(x + 8);
  const uint32_t xs[8] = {xv0.x, xv0.y, xv0.z, xv0.w, xv1.x, xv1.y, xv1.z, xv1.w};
  float s = 0.f;
#pragma unroll
  for (int g = 0; g < 4; g++) {
    const uint32_t b = (w >> (2 * g)) & 0x03030303u;      // elements 4g .. 4g+3 as bytes
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int e = 4 * g + j;
      const float t = (float)(int)((b >> (8 * j)) & 3u) - 1.f;
      const uint32_t xw = xs[e >> 1];
      const float xf = h2f((uint16_t)((e & 1) ? (xw >> 16) : (xw & 0xFFFFu)));
      s = fmaf(t, xf, s);
    }
  }
  return s;
}

E4B_DEV float row_dot(const uint32_t* __restrict__ row, const uint16_t* __restrict__ x, int words, int lane) {
  float s = 0.f;
  for (int jw = lane; jw < words; jw += 32) s += t2dot16(__ldg(row + jw), x + 16 * jw);
  return warp_sum(s);
}

__global__ void k_t2gu(const uint16_t* __restrict__ x, const uint32_t* __restrict__ w,
                       const uint16_t* __restrict__ scale, const uint32_t* __restrict__ topk,
                       uint16_t* __restrict__ yh, int IN, int FF, int K, uint32_t* status, int E) {
  pdl_wait();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= K * FF) return;
  const int k = warp / FF, i = warp % FF;
  const uint32_t e = topk[k];
  if (e >= (uint32_t)E) {
    if (lane == 0) set_status(status, E4B_ST_BADINDEX);
    return;
  }
  const int words = IN / 16;
  const size_t rg = (size_t)e * 2 * FF + i, ru = rg + FF;
  const float g = row_dot(w + rg * words, x, words, lane) * h2f(scale[rg]);
  const float u = row_dot(w + ru * words, x, words, lane) * h2f(scale[ru]);
  if (lane == 0) yh[(size_t)k * FF + i] = f2h(gelu_tanh(g) * u);
}

__global__ void k_t2moedown(const uint16_t* __restrict__ x, const uint32_t* __restrict__ w,
                            const uint16_t* __restrict__ scale, const uint32_t* __restrict__ topk,
                            const float* __restrict__ topk_w, float* __restrict__ y, int IN, int OUT, int K,
                            uint32_t* status, int E) {
  pdl_wait();
  const int o = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (o >= OUT) return;
  const int words = IN / 16;
  float acc = 0.f;
  for (int k = 0; k < K; k++) {
    const uint32_t e = topk[k];
    if (e >= (uint32_t)E) {
      if (lane == 0) set_status(status, E4B_ST_BADINDEX);
      return;
    }
    const size_t r = (size_t)e * OUT + o;
    const float s = row_dot(w + r * words, x + (size_t)k * IN, words, lane);
    acc += topk_w[k] * s * h2f(scale[r]);
  }
  if (lane == 0) y[o] = acc;
}

}  // namespace

extern "C" {

E4B_API int e4b_t2gu(e4b_ctx* c, const uint16_t* x, const uint32_t* w, const uint16_t* scale, const uint32_t* topk,
                     uint16_t* yh, int IN, int FF, int K, int E) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, x && w && scale && topk && yh && FF > 0 && K > 0 && E > 0, "t2gu: bad args");
  E4B_REQUIRE(c, IN > 0 && IN % 16 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0,
              "t2gu: IN=%d must be a multiple of 16 and x 16-byte aligned", IN);
  const long long warps = (long long)K * FF;
  return e4b_launch(c, "t2gu", k_t2gu, dim3((unsigned)((warps + 7) / 8)), dim3(256), 0, x, w, scale, topk, yh, IN, FF,
                    K, c->status, E);
}

E4B_API int e4b_t2moedown(e4b_ctx* c, const uint16_t* x, const uint32_t* w, const uint16_t* scale,
                          const uint32_t* topk, const float* topk_w, float* y, int IN, int OUT, int K, int E) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, x && w && scale && topk && topk_w && y && OUT > 0 && K > 0 && E > 0, "t2moedown: bad args");
  E4B_REQUIRE(c, IN > 0 && IN % 16 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0,
              "t2moedown: IN=%d must be a multiple of 16 and x 16-byte aligned", IN);
  return e4b_launch(c, "t2moedown", k_t2moedown, dim3((OUT + 7) / 8), dim3(256), 0, x, w, scale, topk, topk_w, y, IN,
                    OUT, K, c->status, E);
}

}  // extern "C"
