// RMSNorm family and element-wise GeGLU / PLE products.  One CTA per row for the
// reductions (rows = batch tokens); f32 math, f16 stores where the reference
// stores f16.
#include "common.cuh"

namespace {

__global__ void k_rmsnorm(const float* __restrict__ x, const float* __restrict__ w, float* __restrict__ y,
                          float* __restrict__ sums, uint16_t* __restrict__ yh, int dim, float eps, int with_scale,
                          int sumout, int f16out) {
  pdl_wait();
  __shared__ float sh[32];
  const size_t base = (size_t)blockIdx.x * dim;
  float s = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) s = fmaf(x[base + i], x[base + i], s);
  const float inv = rms_scale(block_sum(s, sh), dim, eps);
  float s2 = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    float v = x[base + i] * inv;
    if (with_scale) v = v * w[i];
    if (f16out) yh[base + (f16out == 2 ? xfo_pos(i) : i)] = f2h(v);
    else y[base + i] = v;
    s2 += v;
  }
  if (sumout) {
    const float t = block_sum(s2, sh);
    if (threadIdx.x == 0) sums[blockIdx.x] = t;
  }
}

__global__ void k_rmsacc(const float* __restrict__ x, const float* __restrict__ w, float* __restrict__ hidden,
                         int dim, float eps, float mul) {
  pdl_wait();
  __shared__ float sh[32];
  float s = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) s = fmaf(x[i], x[i], s);
  const float inv = rms_scale(block_sum(s, sh), dim, eps);
  for (int i = threadIdx.x; i < dim; i += blockDim.x) hidden[i] = (hidden[i] + x[i] * inv * w[i]) * mul;
}

// hidden = (hidden + rms(t)*w1)*mul; yh = f16(rms(hidden)*w2) or f16(hidden).
__global__ void k_rmsaccn(const float* __restrict__ t, const float* __restrict__ w1, float* __restrict__ hidden,
                          const float* __restrict__ w2, uint16_t* __restrict__ yh, int dim, float eps, float mul,
                          int norm2) {
  pdl_wait();
  extern __shared__ float hs[];
  __shared__ float sh[32];
  float s = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) s = fmaf(t[i], t[i], s);
  const float inv1 = rms_scale(block_sum(s, sh), dim, eps);
  float s2 = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float h = (hidden[i] + t[i] * inv1 * w1[i]) * mul;
    hidden[i] = h;
    hs[i] = h;
    s2 = fmaf(h, h, s2);
  }
  float inv2 = 1.f;
  if (norm2) inv2 = rms_scale(block_sum(s2, sh), dim, eps);
  __syncthreads();
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    float v = hs[i];
    if (norm2) v = v * inv2 * w2[i];
    yh[i] = f2h(v);
  }
}

__global__ void k_rmsacc3(const float* __restrict__ t, const float* __restrict__ w_acc, const float* __restrict__ w1,
                          const float* __restrict__ w2, const float* __restrict__ w3, const float* __restrict__ h_in,
                          uint16_t* __restrict__ y1, float* __restrict__ y2, uint16_t* __restrict__ y3,
                          float* __restrict__ h_out, int dim, float eps, int xfo, int nparts, size_t part_stride) {
  pdl_wait();
  extern __shared__ float hs[];           // [dim] h, [dim] t
  __shared__ float sh[32];
  float* ts = hs + dim;
  const size_t ob = (size_t)blockIdx.x * dim;
  float s = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float v = sum_parts(t + ob + i, part_stride, nparts);   // K-part partials, in order
    ts[i] = v;
    hs[i] = h_in[ob + i];
    s = fmaf(v, v, s);
  }
  const float inv1 = rms_scale(block_sum(s, sh), dim, eps);
  float s2 = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float h = hs[i] + ts[i] * inv1 * w_acc[i];
    h_out[ob + i] = h;
    hs[i] = h;
    s2 = fmaf(h, h, s2);
  }
  const float inv2 = rms_scale(block_sum(s2, sh), dim, eps);
  __syncthreads();
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float v = hs[i] * inv2;
    const size_t oh = ob + (xfo ? xfo_pos(i) : i);
    y1[oh] = f2h(v * w1[i]);
    y2[ob + i] = v * w2[i];
    y3[oh] = f2h(v * w3[i]);
  }
}

// m = the MoE output row; with y != null it is first formed here as the
// slot-ordered combine sum_k w[row][k] * y[inv[row K + k]] (kernels/wacc.wgsl).
__global__ void k_a4btail(const float* __restrict__ t1, const float* __restrict__ w1, const float* __restrict__ m,
                          const float* __restrict__ w2, const float* __restrict__ wp, const float* __restrict__ h_in,
                          const float* __restrict__ w_next, uint16_t* __restrict__ y_next, float* __restrict__ h_out,
                          int H, float eps, float mul, int next, int xfo, const float* __restrict__ y,
                          const uint32_t* __restrict__ inv, const float* __restrict__ tkw, int K) {
  pdl_wait();
  extern __shared__ float comb[];          // [H] comb, [H] t1, [H] h_in
  __shared__ float sh[32];
  __shared__ uint32_t s_inv[32];           // this row's K slots (K <= 32) and their weights
  __shared__ float s_w[32];
  float* ts = comb + H;
  float* hs = comb + 2 * H;
  const size_t ob = (size_t)blockIdx.x * H;
  if (y && threadIdx.x < K) {
    s_inv[threadIdx.x] = inv[(size_t)blockIdx.x * K + threadIdx.x];
    s_w[threadIdx.x] = tkw[(size_t)blockIdx.x * K + threadIdx.x];
  }
  __syncthreads();
  float s1 = 0.f, s2 = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float a = t1[ob + i];
    float mv;
    if (y) {
      // the slots' rows loaded eight at a time, then added in slot order
      mv = 0.f;
      for (int k0 = 0; k0 < K; k0 += 8) {
        float yv[8];
#pragma unroll
        for (int k = 0; k < 8; k++) {
          const uint32_t r = k0 + k < K ? s_inv[k0 + k] : 0xffffffffu;   // 0xffffffff: dropped entry
          yv[k] = r != 0xffffffffu ? y[(size_t)r * H + i] : 0.f;
        }
#pragma unroll
        for (int k = 0; k < 8; k++)
          if (k0 + k < K && s_inv[k0 + k] != 0xffffffffu) mv += s_w[k0 + k] * yv[k];
      }
    } else {
      mv = m[ob + i];
    }
    ts[i] = a;
    hs[i] = h_in[ob + i];
    s1 = fmaf(a, a, s1);
    s2 = fmaf(mv, mv, s2);
    comb[i] = mv;
  }
  const float inv1 = rms_scale(block_sum(s1, sh), H, eps);
  const float inv2 = rms_scale(block_sum(s2, sh), H, eps);
  float s3 = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float cc = ts[i] * inv1 * w1[i] + comb[i] * inv2 * w2[i];
    comb[i] = cc;
    s3 = fmaf(cc, cc, s3);
  }
  const float inv3 = rms_scale(block_sum(s3, sh), H, eps);
  float s4 = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float hn = (hs[i] + comb[i] * inv3 * wp[i]) * mul;
    h_out[ob + i] = hn;
    comb[i] = hn;
    s4 = fmaf(hn, hn, s4);
  }
  if (next) {
    const float inv4 = rms_scale(block_sum(s4, sh), H, eps);
    __syncthreads();
    for (int i = threadIdx.x; i < H; i += blockDim.x) y_next[ob + (xfo ? xfo_pos(i) : i)] = f2h(comb[i] * inv4 * w_next[i]);
  }
}

__global__ void k_geglumul(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ y, int N) {
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < N) y[i] = gelu_tanh(a[i]) * b[i];
}
__global__ void k_geglusl(const float* __restrict__ gu, float* __restrict__ out, int FF, int K) {
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= K * FF) return;
  const int k = i / FF, j = i % FF;
  out[i] = gelu_tanh(gu[(size_t)k * 2 * FF + j]) * gu[(size_t)k * 2 * FF + FF + j];
}
__global__ void k_geglub(const float* __restrict__ gu, uint16_t* __restrict__ yh, int N, int rows) {
  pdl_wait();
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)rows * N) return;
  const size_t r = i / N, j = i % N;
  yh[i] = f2h(gelu_tanh(gu[r * 2 * N + j]) * gu[r * 2 * N + N + j]);
}
__global__ void k_plemul(const float* __restrict__ a, const float* __restrict__ ple, float* __restrict__ y, int N,
                         int off) {
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < N) y[i] = gelu_tanh(a[i]) * ple[off + i];
}

int set_smem(e4b_ctx* c, const void* k, size_t bytes) {
  if (bytes > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) return e4b_fail(c, E4B_ECUDA, "smem attribute: %s", cudaGetErrorString(e));
  }
  return E4B_OK;
}

}  // namespace

extern "C" {

E4B_API int e4b_rmsnorm(e4b_ctx* c, const float* x, const float* w, float* y, float* sums, uint16_t* yh, int dim,
                        int rows, float eps, int with_scale, int sumout, int f16out) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, x && dim > 0 && rows > 0, "rmsnorm: bad args");
  E4B_REQUIRE(c, f16out ? yh != nullptr : y != nullptr, "rmsnorm: missing output");
  E4B_REQUIRE(c, !with_scale || w, "rmsnorm: missing weight");
  E4B_REQUIRE(c, !sumout || sums, "rmsnorm: missing sums");
  E4B_REQUIRE(c, f16out >= 0 && f16out <= 2 && (f16out != 2 || dim % 32 == 0), "rmsnorm: bad f16out=%d", f16out);
  return e4b_launch(c, "rmsnorm", k_rmsnorm, dim3(rows), dim3(256), 0, x, w, y, sums, yh, dim, eps, with_scale,
                    sumout, f16out);
}

E4B_API int e4b_rmsacc(e4b_ctx* c, const float* x, const float* w, float* hidden, int dim, float eps, float mul) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, x && w && hidden && dim > 0, "rmsacc: bad args");
  return e4b_launch(c, "rmsacc", k_rmsacc, dim3(1), dim3(256), 0, x, w, hidden, dim, eps, mul);
}

E4B_API int e4b_rmsaccn(e4b_ctx* c, const float* t, const float* w1, float* hidden, const float* w2, uint16_t* yh,
                        int dim, float eps, float mul, int norm2) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, t && w1 && hidden && yh && dim > 0 && (!norm2 || w2), "rmsaccn: bad args");
  const size_t sm = (size_t)dim * 4;
  if (int r = set_smem(c, (const void*)k_rmsaccn, sm)) return r;
  return e4b_launch(c, "rmsaccn", k_rmsaccn, dim3(1), dim3(256), sm, t, w1, hidden, w2, yh, dim, eps, mul, norm2);
}

E4B_API int e4b_rmsacc3(e4b_ctx* c, const float* t, const float* w_acc, const float* w1, const float* w2,
                        const float* w3, const float* h_in, uint16_t* y1, float* y2, uint16_t* y3, float* h_out,
                        int dim, float eps, int rows, int xfo, int nparts) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, t && w_acc && w1 && w2 && w3 && h_in && y1 && y2 && y3 && h_out && dim > 0, "rmsacc3: bad args");
  E4B_REQUIRE(c, !xfo || dim % 32 == 0, "rmsacc3: fragment order needs dim %% 32 == 0");
  E4B_REQUIRE(c, nparts >= 1, "rmsacc3: nparts=%d", nparts);
  if (rows < 1) rows = 1;
  const size_t sm = (size_t)dim * 8;
  if (int r = set_smem(c, (const void*)k_rmsacc3, sm)) return r;
  return e4b_launch(c, "rmsacc3", k_rmsacc3, dim3(rows), dim3(1024), sm, t, w_acc, w1, w2, w3, h_in, y1, y2, y3,
                    h_out, dim, eps, xfo, nparts, (size_t)rows * dim);
}

E4B_API int e4b_a4btail(e4b_ctx* c, const float* t1, const float* w1, const float* m, const float* w2,
                        const float* wp, const float* h_in, const float* w_next, uint16_t* y_next, float* h_out, int H,
                        float eps, float mul, int next, int rows, int xfo) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, t1 && w1 && m && w2 && wp && h_in && h_out && H > 0, "a4btail: bad args");
  E4B_REQUIRE(c, !next || (w_next && y_next), "a4btail: next=1 needs w_next and y_next");
  E4B_REQUIRE(c, !xfo || H % 32 == 0, "a4btail: fragment order needs H %% 32 == 0");
  if (rows < 1) rows = 1;
  const size_t sm = (size_t)H * 12;
  if (int r = set_smem(c, (const void*)k_a4btail, sm)) return r;
  return e4b_launch(c, "a4btail", k_a4btail, dim3(rows), dim3(1024), sm, t1, w1, m, w2, wp, h_in, w_next, y_next,
                    h_out, H, eps, mul, next, xfo, (const float*)nullptr, (const uint32_t*)nullptr,
                    (const float*)nullptr, 0);
}

E4B_API int e4b_a4btail_wacc(e4b_ctx* c, const float* t1, const float* w1, const float* y, const uint32_t* inv,
                             const float* topk_w, int K, const float* w2, const float* wp, const float* h_in,
                             const float* w_next, uint16_t* y_next, float* h_out, int H, float eps, float mul, int next,
                             int rows, int xfo) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, t1 && w1 && y && inv && topk_w && K > 0 && K <= 32 && w2 && wp && h_in && h_out && H > 0 && rows > 0,
              "a4btail_wacc: bad args (K <= 32)");
  E4B_REQUIRE(c, !next || (w_next && y_next), "a4btail_wacc: next=1 needs w_next and y_next");
  E4B_REQUIRE(c, !xfo || H % 32 == 0, "a4btail_wacc: fragment order needs H %% 32 == 0");
  const size_t sm = (size_t)H * 12;
  if (int r = set_smem(c, (const void*)k_a4btail, sm)) return r;
  return e4b_launch(c, "a4btail_wacc", k_a4btail, dim3(rows), dim3(1024), sm, t1, w1, (const float*)nullptr, w2, wp,
                    h_in, w_next, y_next, h_out, H, eps, mul, next, xfo, y, inv, topk_w, K);
}

E4B_API int e4b_geglumul(e4b_ctx* c, const float* a, const float* b, float* y, int N) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, a && b && y && N > 0, "geglumul: bad args");
  return e4b_launch(c, "geglumul", k_geglumul, dim3((N + 255) / 256), dim3(256), 0, a, b, y, N);
}
E4B_API int e4b_geglusl(e4b_ctx* c, const float* gu, float* out, int FF, int K) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, gu && out && FF > 0 && K > 0, "geglusl: bad args");
  return e4b_launch(c, "geglusl", k_geglusl, dim3((K * FF + 255) / 256), dim3(256), 0, gu, out, FF, K);
}
E4B_API int e4b_geglub(e4b_ctx* c, const float* gu, uint16_t* yh, int N, int rows) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, gu && yh && N > 0 && rows > 0, "geglub: bad args");
  const size_t n = (size_t)N * rows;
  return e4b_launch(c, "geglub", k_geglub, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, gu, yh, N, rows);
}
E4B_API int e4b_plemul(e4b_ctx* c, const float* a, const float* ple, float* y, int N, int off) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, a && ple && y && N > 0 && off >= 0, "plemul: bad args");
  return e4b_launch(c, "plemul", k_plemul, dim3((N + 255) / 256), dim3(256), 0, a, ple, y, N, off);
}

}  // extern "C"
