// RMSNorm family and element-wise GeGLU / PLE products.  One CTA per row for the
// reductions (rows = batch tokens); f32 math, f16 stores where the reference
// stores f16.
#include <initializer_list>

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

// ---- float4 forms of rmsacc3 / a4btail: one float4 column per thread
// (dim % 4 == 0, dim <= 4 * blockDim, 16-byte aligned rows).  Every global
// load is issued before the first reduction and the row stays in registers
// between the reductions, so a CTA waits on memory once instead of once per
// strided element.  Per element the arithmetic is the scalar kernels'; the
// sums of squares add each thread's four elements first.
E4B_DEV float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
E4B_DEV void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
// p[0] + p[stride4] + ... in that order, per component (sum_parts on float4s)
E4B_DEV float4 sum_parts4(const float4* __restrict__ p, size_t stride4, int n) {
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int k0 = 0; k0 < n; k0 += 8) {
    float4 x[8];
#pragma unroll
    for (int k = 0; k < 8; k++) x[k] = k0 + k < n ? p[(size_t)(k0 + k) * stride4] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < 8; k++) {
      if (k0 + k >= n) break;
      if (k0 + k == 0) {
        v = x[k];
      } else {
        v.x += x[k].x;
        v.y += x[k].y;
        v.z += x[k].z;
        v.w += x[k].w;
      }
    }
  }
  return v;
}
// Two block sums with one pair of barriers (sh >= 64 floats); each adds the
// warp results in warp order, as block_sum does.
E4B_DEV float2 block_sum2(float a, float b, float* sh) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  a = warp_sum(a);
  b = warp_sum(b);
  __syncthreads();
  if (lane == 0) {
    sh[wid] = a;
    sh[32 + wid] = b;
  }
  __syncthreads();
  float ta = 0.f, tb = 0.f;
  for (int i = 0; i < nw; i++) {
    ta += sh[i];
    tb += sh[32 + i];
  }
  return make_float2(ta, tb);
}
// The sums of squares in the scalar kernels' order, so both forms give the
// same bits: the row is staged in shared memory and thread t < T adds elements
// t, t + T, ... with fmaf (T = the scalar kernel's CTA size; other threads add
// nothing), then the block sum.
E4B_DEV float strided_sumsq(const float* row, int n, int T) {
  float s = 0.f;
  if ((int)threadIdx.x < T)
    for (int k = threadIdx.x; k < n; k += T) s = fmaf(row[k], row[k], s);
  return s;
}
E4B_DEV float strided_sum(const float* row, int n, int T) {
  float s = 0.f;
  if ((int)threadIdx.x < T)
    for (int k = threadIdx.x; k < n; k += T) s += row[k];
  return s;
}
// four f16 values of elements i..i+3 (fragment order: scattered positions)
E4B_DEV void st_h4(uint16_t* __restrict__ y, size_t ob, int i, int xfo, float a, float b, float c, float d) {
  if (xfo) {
    y[ob + xfo_pos(i)] = f2h(a);
    y[ob + xfo_pos(i + 1)] = f2h(b);
    y[ob + xfo_pos(i + 2)] = f2h(c);
    y[ob + xfo_pos(i + 3)] = f2h(d);
  } else {
    *reinterpret_cast<uint2*>(y + ob + i) = make_uint2((uint32_t)f2h(a) | ((uint32_t)f2h(b) << 16),
                                                       (uint32_t)f2h(c) | ((uint32_t)f2h(d) << 16));
  }
}

__global__ void __launch_bounds__(1024, 1)
    k_rmsacc3v(const float* __restrict__ t, const float* __restrict__ w_acc, const float* __restrict__ w1,
               const float* __restrict__ w2, const float* __restrict__ w3, const float* __restrict__ h_in,
               uint16_t* __restrict__ y1, float* __restrict__ y2, uint16_t* __restrict__ y3, float* __restrict__ h_out,
               int dim, float eps, int xfo, int nparts, size_t part_stride) {
  __shared__ float sh[64];
  __shared__ __align__(16) float rowv[4096];
  const int i = 4 * (int)threadIdx.x;
  const bool on = i < dim;
  const size_t ob = (size_t)blockIdx.x * dim;
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
  // the norm vectors do not depend on the previous kernel
  const float4 wa = on ? ld4(w_acc + i) : z, a1 = on ? ld4(w1 + i) : z, a2 = on ? ld4(w2 + i) : z,
               a3 = on ? ld4(w3 + i) : z;
  pdl_wait();
  float4 tv = z, hv = z;
  if (on) {
    tv = sum_parts4(reinterpret_cast<const float4*>(t + ob + i), part_stride / 4, nparts);
    hv = ld4(h_in + ob + i);
    st4(rowv + i, tv);
  }
  __syncthreads();
  const float inv1 = rms_scale(block_sum(strided_sumsq(rowv, dim, 1024), sh), dim, eps);
  float4 h;
  h.x = hv.x + tv.x * inv1 * wa.x;
  h.y = hv.y + tv.y * inv1 * wa.y;
  h.z = hv.z + tv.z * inv1 * wa.z;
  h.w = hv.w + tv.w * inv1 * wa.w;
  if (on) {
    st4(h_out + ob + i, h);
    st4(rowv + i, h);        // every thread's reads of rowv preceded block_sum's first barrier
  }
  __syncthreads();
  const float inv2 = rms_scale(block_sum(strided_sumsq(rowv, dim, 1024), sh), dim, eps);
  if (!on) return;
  const float4 v = make_float4(h.x * inv2, h.y * inv2, h.z * inv2, h.w * inv2);
  st_h4(y1, ob, i, xfo, v.x * a1.x, v.y * a1.y, v.z * a1.z, v.w * a1.w);
  st4(y2 + ob + i, make_float4(v.x * a2.x, v.y * a2.y, v.z * a2.z, v.w * a2.w));
  st_h4(y3, ob, i, xfo, v.x * a3.x, v.y * a3.y, v.z * a3.z, v.w * a3.w);
}

__global__ void __launch_bounds__(1024, 1)
    k_a4btailv(const float* __restrict__ t1, const float* __restrict__ w1, const float* __restrict__ m,
               const float* __restrict__ w2, const float* __restrict__ wp, const float* __restrict__ h_in,
               const float* __restrict__ w_next, uint16_t* __restrict__ y_next, float* __restrict__ h_out, int H,
               float eps, float mul, int next, int xfo, const float* __restrict__ y, const uint32_t* __restrict__ inv,
               const float* __restrict__ tkw, int K) {
  __shared__ float sh[64];
  __shared__ __align__(16) float rowa[4096], rowb[4096];
  const int i = 4 * (int)threadIdx.x;
  const bool on = i < H;
  const size_t ob = (size_t)blockIdx.x * H;
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
  const float4 a1 = on ? ld4(w1 + i) : z, a2 = on ? ld4(w2 + i) : z, ap = on ? ld4(wp + i) : z,
               an = on && next ? ld4(w_next + i) : z;
  pdl_wait();
  float4 tv = z, hv = z, mv = z;
  if (on) {
    tv = ld4(t1 + ob + i);
    hv = ld4(h_in + ob + i);
    if (y) {
      // the slots' rows loaded eight at a time, then added in slot order
      // (0xffffffff: a dropped entry)
      for (int k0 = 0; k0 < K; k0 += 8) {
        float4 yv[8];
        uint32_t r[8];
        float wk[8];
#pragma unroll
        for (int k = 0; k < 8; k++) {
          r[k] = k0 + k < K ? __ldg(inv + (size_t)blockIdx.x * K + k0 + k) : 0xffffffffu;
          wk[k] = k0 + k < K ? __ldg(tkw + (size_t)blockIdx.x * K + k0 + k) : 0.f;
        }
#pragma unroll
        for (int k = 0; k < 8; k++) yv[k] = r[k] != 0xffffffffu ? ld4(y + (size_t)r[k] * H + i) : z;
#pragma unroll
        for (int k = 0; k < 8; k++)
          if (r[k] != 0xffffffffu) {
            mv.x += wk[k] * yv[k].x;
            mv.y += wk[k] * yv[k].y;
            mv.z += wk[k] * yv[k].z;
            mv.w += wk[k] * yv[k].w;
          }
      }
    } else {
      mv = ld4(m + ob + i);
    }
  }
  if (on) {
    st4(rowa + i, tv);
    st4(rowb + i, mv);
  }
  __syncthreads();
  const float2 s12 = block_sum2(strided_sumsq(rowa, H, 1024), strided_sumsq(rowb, H, 1024), sh);
  const float inv1 = rms_scale(s12.x, H, eps), inv2 = rms_scale(s12.y, H, eps);
  float4 cc;
  cc.x = tv.x * inv1 * a1.x + mv.x * inv2 * a2.x;
  cc.y = tv.y * inv1 * a1.y + mv.y * inv2 * a2.y;
  cc.z = tv.z * inv1 * a1.z + mv.z * inv2 * a2.z;
  cc.w = tv.w * inv1 * a1.w + mv.w * inv2 * a2.w;
  if (on) st4(rowa + i, cc);   // rowa's reads preceded block_sum2's first barrier
  __syncthreads();
  const float inv3 = rms_scale(block_sum(strided_sumsq(rowa, H, 1024), sh), H, eps);
  float4 hn;
  hn.x = (hv.x + cc.x * inv3 * ap.x) * mul;
  hn.y = (hv.y + cc.y * inv3 * ap.y) * mul;
  hn.z = (hv.z + cc.z * inv3 * ap.z) * mul;
  hn.w = (hv.w + cc.w * inv3 * ap.w) * mul;
  if (on) {
    st4(h_out + ob + i, hn);
    st4(rowa + i, hn);
  }
  __syncthreads();
  if (next) {
    const float inv4 = rms_scale(block_sum(strided_sumsq(rowa, H, 1024), sh), H, eps);
    if (on)
      st_h4(y_next, ob, i, xfo, hn.x * inv4 * an.x, hn.y * inv4 * an.y, hn.z * inv4 * an.z, hn.w * inv4 * an.w);
  }
}

// k_rmsnorm on float4 columns (the float4 kernels' conditions; one pass over x).
__global__ void __launch_bounds__(1024, 1)
    k_rmsnormv(const float* __restrict__ x, const float* __restrict__ w, float* __restrict__ y,
               float* __restrict__ sums, uint16_t* __restrict__ yh, int dim, float eps, int with_scale, int sumout,
               int f16out) {
  __shared__ float sh[64];
  __shared__ __align__(16) float rowv[4096];
  const int i = 4 * (int)threadIdx.x;
  const bool on = i < dim;
  const size_t ob = (size_t)blockIdx.x * dim;
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
  const float4 wv = on && with_scale ? ld4(w + i) : z;
  pdl_wait();
  const float4 xv = on ? ld4(x + ob + i) : z;
  if (on) st4(rowv + i, xv);
  __syncthreads();
  // k_rmsnorm's order: 256 threads
  const float inv = rms_scale(block_sum(strided_sumsq(rowv, dim, 256), sh), dim, eps);
  float4 v = make_float4(xv.x * inv, xv.y * inv, xv.z * inv, xv.w * inv);
  if (with_scale) v = make_float4(v.x * wv.x, v.y * wv.y, v.z * wv.z, v.w * wv.w);
  if (on) {
    if (f16out) st_h4(yh, ob, i, f16out == 2, v.x, v.y, v.z, v.w);
    else st4(y + ob + i, v);
  }
  if (sumout) {
    if (on) st4(rowv + i, v);
    __syncthreads();
    const float t = block_sum(strided_sum(rowv, dim, 256), sh);
    if (threadIdx.x == 0) sums[blockIdx.x] = t;
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

// The float4 kernels apply: width a multiple of 4 within one float4 per thread
// of a 1024-thread CTA, f32 rows 16-byte aligned, f16 rows 8-byte aligned
// (their stores are scattered in fragment order).
static bool vec4_ok(int dim, std::initializer_list<const void*> f32, std::initializer_list<const void*> f16, int xfo) {
  if (dim % 4 != 0 || dim > 4 * 1024) return false;
  for (const void* p : f32)
    if (reinterpret_cast<uintptr_t>(p) % 16 != 0) return false;
  if (!xfo)
    for (const void* p : f16)
      if (reinterpret_cast<uintptr_t>(p) % 8 != 0) return false;
  return true;
}

E4B_API int e4b_rmsnorm(e4b_ctx* c, const float* x, const float* w, float* y, float* sums, uint16_t* yh, int dim,
                        int rows, float eps, int with_scale, int sumout, int f16out) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, x && dim > 0 && rows > 0, "rmsnorm: bad args");
  E4B_REQUIRE(c, f16out ? yh != nullptr : y != nullptr, "rmsnorm: missing output");
  E4B_REQUIRE(c, !with_scale || w, "rmsnorm: missing weight");
  E4B_REQUIRE(c, !sumout || sums, "rmsnorm: missing sums");
  E4B_REQUIRE(c, f16out >= 0 && f16out <= 2 && (f16out != 2 || dim % 32 == 0), "rmsnorm: bad f16out=%d", f16out);
  if (vec4_ok(dim, {x, with_scale ? w : nullptr, f16out ? nullptr : y}, {f16out ? yh : nullptr}, f16out == 2))
    return e4b_launch(c, "rmsnorm", k_rmsnormv, dim3(rows), dim3(1024), 0, x, w, y, sums, yh, dim, eps, with_scale,
                      sumout, f16out);
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
  if (vec4_ok(dim, {t, w_acc, w1, w2, w3, h_in, y2, h_out}, {y1, y3}, xfo))
    return e4b_launch(c, "rmsacc3", k_rmsacc3v, dim3(rows), dim3(1024), 0, t, w_acc, w1, w2, w3, h_in, y1, y2, y3,
                      h_out, dim, eps, xfo, nparts, (size_t)rows * dim);
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
  if (vec4_ok(H, {t1, w1, m, w2, wp, h_in, next ? w_next : nullptr, h_out}, {next ? y_next : nullptr}, xfo))
    return e4b_launch(c, "a4btail", k_a4btailv, dim3(rows), dim3(1024), 0, t1, w1, m, w2, wp, h_in, w_next, y_next,
                      h_out, H, eps, mul, next, xfo, (const float*)nullptr, (const uint32_t*)nullptr,
                      (const float*)nullptr, 0);
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
  if (vec4_ok(H, {t1, w1, y, w2, wp, h_in, next ? w_next : nullptr, h_out}, {next ? y_next : nullptr}, xfo))
    return e4b_launch(c, "a4btail_wacc", k_a4btailv, dim3(rows), dim3(1024), 0, t1, w1, (const float*)nullptr, w2,
                      wp, h_in, w_next, y_next, h_out, H, eps, mul, next, xfo, y, inv, topk_w, K);
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
