// MoE routing (routertop / router / top8), two-stage argmax and the GPU-side
// token feedback that makes a recorded per-token plan replayable.
#include <mutex>

#include "common.cuh"
#include "q40_stream.cuh"

namespace {

// Softmax over E scores (p in shared memory, overwritten with exp(s-max)),
// then K rounds of first-maximum selection, renormalisation and x pes
// (kernels/routertop.wgsl:51-69).  Run by warp 0 of the CTA.
E4B_DEV void softmax_topk(float* p, int E, int K, const float* __restrict__ pes, uint32_t* __restrict__ idx_out,
                          float* __restrict__ w_out) {
  const int lane = threadIdx.x & 31;
  float mx = -3.0e38f;
  for (int i = lane; i < E; i += 32) mx = fmaxf(mx, p[i]);
  mx = warp_max(mx);
  for (int i = lane; i < E; i += 32) p[i] = expf(p[i] - mx);
  __syncwarp();
  float sum = 0.f;
  if (lane == 0) {   // sequential, as the reference's single-thread epilogue (vector loads, same order)
    int i = 0;
    if ((reinterpret_cast<uintptr_t>(p) & 15) == 0)
      for (; i + 4 <= E; i += 4) {
        const float4 v = *reinterpret_cast<const float4*>(p + i);
        sum += v.x;
        sum += v.y;
        sum += v.z;
        sum += v.w;
      }
    for (; i < E; i++) sum += p[i];
  }
  sum = __shfl_sync(0xffffffffu, sum, 0);
  float wsum = 0.f;
  float wk[32];
  uint32_t ik[32];
  for (int k = 0; k < K; k++) {
    float bv = -1.0f;
    int bi = 0x7fffffff;
    for (int i = lane; i < E; i += 32)
      if (p[i] > bv) { bv = p[i]; bi = i; }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    const float w = bv / sum;
    if (k < 32) { wk[k] = w; ik[k] = (uint32_t)bi; }
    wsum += w;
    __syncwarp();
    if (lane == 0) p[bi] = -2.0f;
    __syncwarp();
  }
  if (lane == 0)
    for (int k = 0; k < K && k < 32; k++) {
      idx_out[k] = ik[k];
      w_out[k] = wk[k] / wsum * pes[ik[k]];
    }
}

// One CTA per token: warps split the E expert dot products over H.
__global__ void __launch_bounds__(256) k_routertop(const float* __restrict__ x, const float* __restrict__ wr,
                                                   const float* __restrict__ pes, uint32_t* __restrict__ topk_idx,
                                                   float* __restrict__ topk_w, int H, int E, int K) {
  pdl_wait();
  extern __shared__ float p[];
  const int b = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const float* xr = x + (size_t)b * H;
  for (int e = warp; e < E; e += nw) {
    const float* w = wr + (size_t)e * H;
    float acc = 0.f;
    for (int j = lane; j < H; j += 32) acc = fmaf(xr[j], w[j], acc);
    acc = warp_sum(acc);
    if (lane == 0) p[e] = acc;
  }
  __syncthreads();
  if (warp == 0) softmax_topk(p, E, K, pes, topk_idx + (size_t)b * K, topk_w + (size_t)b * K);
}

// Batched routing (many tokens): the scores are a small f32 GEMM
// S[b][e] = x[b] . wr[e], split over kRtK-wide slices of H so that enough CTAs
// run: CTA (token tile, expert tile, slice) stages its x and wr slices in
// shared memory and writes part[slice][b][e]; then one warp per token sums the
// slices in order and runs the softmax / top-K above.
constexpr int kRtTok = 16, kRtExp = 32, kRtK = 128;

__global__ void __launch_bounds__(256) k_router_part(const float* __restrict__ x, const float* __restrict__ wr,
                                                     float* __restrict__ part, int B, int H, int E) {
  pdl_wait();
  __shared__ float xs[kRtTok][kRtK];
  __shared__ float wsm[kRtExp][kRtK + 1];
  const int b0 = blockIdx.x * kRtTok, e0 = blockIdx.y * kRtExp, k0 = blockIdx.z * kRtK;
  const int tid = threadIdx.x;
  for (int i = tid; i < kRtTok * kRtK; i += 256) {
    const int r = i / kRtK, k = i % kRtK;
    xs[r][k] = (b0 + r < B && k0 + k < H) ? x[(size_t)(b0 + r) * H + k0 + k] : 0.f;
  }
  for (int i = tid; i < kRtExp * kRtK; i += 256) {
    const int r = i / kRtK, k = i % kRtK;
    wsm[r][k] = (e0 + r < E && k0 + k < H) ? wr[(size_t)(e0 + r) * H + k0 + k] : 0.f;
  }
  __syncthreads();
  const int warp = tid >> 5, lane = tid & 31;
  float a0 = 0.f, a1 = 0.f;
#pragma unroll 8
  for (int k = 0; k < kRtK; k++) {
    const float w = wsm[lane][k];
    a0 = fmaf(xs[2 * warp][k], w, a0);
    a1 = fmaf(xs[2 * warp + 1][k], w, a1);
  }
  const int e = e0 + lane;
  if (e < E) {
    float* pp = part + (size_t)blockIdx.z * B * E;
    if (b0 + 2 * warp < B) pp[(size_t)(b0 + 2 * warp) * E + e] = a0;
    if (b0 + 2 * warp + 1 < B) pp[(size_t)(b0 + 2 * warp + 1) * E + e] = a1;
  }
}

// One CTA per token: every thread sums one expert's slices (in slice order,
// loads issued together), then warp 0 runs the softmax / top-K.
__global__ void __launch_bounds__(256) k_router_topk(const float* __restrict__ part, const float* __restrict__ pes,
                                                     uint32_t* __restrict__ topk_idx, float* __restrict__ topk_w,
                                                     int B, int E, int K, int slices) {
  pdl_wait();
  extern __shared__ __align__(16) float pw[];
  const int b = blockIdx.x;
  if (b >= B) return;
  const size_t step = (size_t)B * E;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const float* src = part + (size_t)b * E + e;
    float v = 0.f;
    int s = 0;
    for (; s + 8 <= slices; s += 8) {
      float t[8];
#pragma unroll
      for (int u = 0; u < 8; u++) t[u] = src[(s + u) * step];
#pragma unroll
      for (int u = 0; u < 8; u++) v += t[u];
    }
    for (; s < slices; s++) v += src[s * step];
    pw[e] = v;
  }
  __syncthreads();
  if (threadIdx.x < 32) softmax_topk(pw, E, K, pes, topk_idx + (size_t)b * K, topk_w + (size_t)b * K);
}

// Skewed routing for the expert-parallel benchmark (benchmark config 5: a seeded
// Zipf(s) load over the experts): token i (global index tok0 + i) at position
// params[0] of layer `salt` draws K distinct experts by inverse-CDF sampling of
// Zipf(s) over popularity ranks, mapped to expert ids by a seeded permutation,
// each with weight 1/K.  A counter-based hash makes the draw a pure function of
// (seed, salt, position, token), so every rank count routes the same way.
E4B_DEV uint32_t mix32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}
// Benchmark routing.  The Zipf(s) popularity table: cumulative popularity of
// each rank (a fixed-order inclusive scan, normalised) and a seeded
// permutation saying which experts are popular, built by one CTA into shared
// memory.  It depends on (s, seed, E) only, so an engine builds it once
// (k_zipf_table) and the per-step routing reloads it.
E4B_DEV void zipf_table_build(float* cdf, uint32_t* perm, int E, float s, uint32_t seed) {
  for (int r = threadIdx.x; r < E; r += blockDim.x) {
    cdf[r] = powf((float)(r + 1), -s);
    perm[r] = (uint32_t)r;
  }
  __syncthreads();
  for (int off = 1; off < E; off <<= 1) {          // Hillis-Steele inclusive scan, fixed order
    float v[16];
    int n = 0;
    for (int r = threadIdx.x; r < E; r += blockDim.x, n++) v[n & 15] = r >= off ? cdf[r - off] : 0.f;
    __syncthreads();
    n = 0;
    for (int r = threadIdx.x; r < E; r += blockDim.x, n++) cdf[r] += v[n & 15];
    __syncthreads();
  }
  const float tot = cdf[E - 1];
  __syncthreads();
  for (int r = threadIdx.x; r < E; r += blockDim.x) cdf[r] /= tot;
  if (threadIdx.x == 0)
    for (int r = E - 1; r > 0; r--) {     // seeded Fisher-Yates: which experts are popular
      const uint32_t j = mix32(seed ^ (0x9e3779b9u * (uint32_t)r)) % (uint32_t)(r + 1);
      const uint32_t t = perm[r];
      perm[r] = perm[j];
      perm[j] = t;
    }
  __syncthreads();
}
// One warp routes one token: the token draws from its own hash stream, 32
// attempts at a time across the lanes, and keeps the first K distinct experts
// in attempt order (exactly what drawing one attempt after another would keep).
E4B_DEV void zipf_route_token(const float* cdf, const uint32_t* perm, int E, int K, uint32_t seed, int salt,
                              uint32_t pos, uint32_t tk, uint32_t* idx_out, float* w_out, int lane) {
  uint32_t chosen = 0xffffffffu;        // lane k < K holds the k-th expert kept
  int got = 0;
  for (uint32_t a0 = 0; got < K && a0 < 4096u; a0 += 32) {
    const uint32_t attempt = a0 + (uint32_t)lane;
    const uint32_t h = mix32(seed ^ mix32((uint32_t)salt * 0x85ebca6bu ^ mix32(pos ^ mix32(tk ^ (attempt << 20)))));
    const float u = (float)(h >> 8) * (1.0f / 16777216.0f);
    int lo = 0, hi = E - 1;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (cdf[mid] > u) hi = mid;
      else lo = mid + 1;
    }
    const uint32_t e = perm[lo];
    for (int j = 0; j < 32 && got < K; j++) {      // attempts in order
      const uint32_t ej = __shfl_sync(0xffffffffu, e, j);
      const bool dup = __any_sync(0xffffffffu, lane < got && chosen == ej);
      if (!dup) {
        if (lane == got) chosen = ej;
        got++;
      }
    }
  }
  for (int r = 0; got < K && r < E; r++) {   // (never needed in practice) fill by popularity
    const uint32_t e = perm[r];
    const bool dup = __any_sync(0xffffffffu, lane < got && chosen == e);
    if (!dup) {
      if (lane == got) chosen = e;
      got++;
    }
  }
  if (lane < K) {
    idx_out[lane] = chosen;
    w_out[lane] = 1.0f / (float)K;
  }
}

// Per CTA: the table, then one warp per row i (sequence tok0 + i % nseq at
// position params[0] + i / nseq).
__global__ void __launch_bounds__(256) k_route_zipf(const uint32_t* __restrict__ params, uint32_t* __restrict__ topk_idx,
                                                    float* __restrict__ topk_w, int n_tok, int K, int E, float s,
                                                    uint32_t seed, int salt, int tok0, int nseq) {
  pdl_wait();
  extern __shared__ float cdf[];          // [E] cumulative popularity, then [E] rank -> expert (as bits)
  uint32_t* perm = reinterpret_cast<uint32_t*>(cdf + E);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  zipf_table_build(cdf, perm, E, s, seed);
  for (int i = blockIdx.x * nw + warp; i < n_tok; i += gridDim.x * nw) {
    const uint32_t pos = params[0] + (uint32_t)(i / nseq);
    const uint32_t tk = (uint32_t)(tok0 + i % nseq);
    zipf_route_token(cdf, perm, E, K, seed, salt, pos, tk, topk_idx + (size_t)i * K, topk_w + (size_t)i * K, lane);
  }
}

// The table into global memory: [E] cdf, then [E] permutation.
__global__ void __launch_bounds__(256) k_zipf_table(float* __restrict__ table, int E, float s, uint32_t seed) {
  pdl_wait();
  extern __shared__ float cdf[];
  uint32_t* perm = reinterpret_cast<uint32_t*>(cdf + E);
  zipf_table_build(cdf, perm, E, s, seed);
  for (int r = threadIdx.x; r < 2 * E; r += blockDim.x) table[r] = cdf[r];
}

// Every layer of one decode step at once: row (layer l, token i) of
// n_layers x n_tok, layer salt salt0 + l, sequence tok0 + i at position
// params[0]; outputs [n_layers][n_tok][K].  The table comes from k_zipf_table.
__global__ void __launch_bounds__(256) k_route_zipf_layers(const uint32_t* __restrict__ params,
                                                           const float* __restrict__ table,
                                                           uint32_t* __restrict__ topk_idx, float* __restrict__ topk_w,
                                                           int n_tok, int n_layers, int K, int E, uint32_t seed,
                                                           int salt0, int tok0) {
  pdl_wait();
  extern __shared__ float cdf[];
  uint32_t* perm = reinterpret_cast<uint32_t*>(cdf + E);
  for (int r = threadIdx.x; r < 2 * E; r += blockDim.x) cdf[r] = table[r];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const uint32_t pos = params[0];
  for (int i = blockIdx.x * nw + warp; i < n_tok * n_layers; i += gridDim.x * nw) {
    const int l = i / n_tok, t = i - l * n_tok;
    zipf_route_token(cdf, perm, E, K, seed, salt0 + l, pos, (uint32_t)(tok0 + t), topk_idx + (size_t)i * K,
                     topk_w + (size_t)i * K, lane);
  }
}

// kernels/router.wgsl: scale-less RMS of h, x H^-0.5 x scale, then scores + top-K.
__global__ void __launch_bounds__(256) k_router(const float* __restrict__ h, const float* __restrict__ scale,
                                                const float* __restrict__ wr, const float* __restrict__ pes,
                                                uint32_t* __restrict__ topk_idx, float* __restrict__ topk_w, int H,
                                                int E, int K, float eps) {
  pdl_wait();
  extern __shared__ float p[];
  __shared__ float sh[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  float s = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) s = fmaf(h[i], h[i], s);
  const float inv = rms_scale(block_sum(s, sh), H, eps) * (1.0f / sqrtf((float)H));
  for (int e = warp; e < E; e += nw) {
    const float* w = wr + (size_t)e * H;
    float acc = 0.f;
    for (int j = lane; j < H; j += 32) acc = fmaf(h[j] * inv * scale[j], w[j], acc);
    acc = warp_sum(acc);
    if (lane == 0) p[e] = acc;
  }
  __syncthreads();
  if (warp == 0) softmax_topk(p, E, K, pes, topk_idx, topk_w);
}

__global__ void k_top8(const float* __restrict__ scores, const float* __restrict__ pes, uint32_t* __restrict__ idx,
                       float* __restrict__ w, int E, int K) {
  pdl_wait();
  extern __shared__ float p[];
  for (int i = threadIdx.x; i < E; i += 32) p[i] = scores[i];
  __syncwarp();
  softmax_topk(p, E, K, pes, idx, w);
}

// argmax stage 0: CTA i reduces slice i -> part[2i] = index, part[2i+1] = f32 bits
// (kernels/argmax2.wgsl:15-22); ties -> lowest index.
E4B_DEV void argmax_merge(float& bv, uint32_t& bi, float ov, uint32_t oi) {
  if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
}
E4B_DEV void block_argmax(float& bv, uint32_t& bi) {
  __shared__ float sv[32];
  __shared__ uint32_t si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    argmax_merge(bv, bi, ov, oi);
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (lane == 0) { sv[wid] = bv; si[wid] = bi; }
  __syncthreads();
  if (threadIdx.x == 0)
    for (int i = 1; i < nw; i++) argmax_merge(bv, bi, sv[i], si[i]);
}
__global__ void k_argmax0(const float* __restrict__ x, uint32_t* __restrict__ part, int N, int parts) {
  pdl_wait();
  x += (size_t)blockIdx.y * N;                  // row blockIdx.y
  part += (size_t)blockIdx.y * parts * 2;
  const int per = (N + parts - 1) / parts;
  const int lo = blockIdx.x * per, hi = min(lo + per, N);
  float bv = -3.0e38f;
  uint32_t bi = 0xffffffffu;
  if ((N & 3) == 0 && (per & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    // float4 loads, four in flight per thread (the merge is order-independent:
    // larger value first, then lower index)
    const float4* x4 = reinterpret_cast<const float4*>(x);
#pragma unroll 4
    for (int i4 = lo / 4 + (int)threadIdx.x; i4 < hi / 4; i4 += blockDim.x) {
      const float4 v = x4[i4];
      const uint32_t i = 4u * (uint32_t)i4;
      argmax_merge(bv, bi, v.x, i);
      argmax_merge(bv, bi, v.y, i + 1);
      argmax_merge(bv, bi, v.z, i + 2);
      argmax_merge(bv, bi, v.w, i + 3);
    }
  } else {
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) argmax_merge(bv, bi, x[i], (uint32_t)i);
  }
  block_argmax(bv, bi);
  if (threadIdx.x == 0) {
    part[2 * blockIdx.x] = bi;
    part[2 * blockIdx.x + 1] = __float_as_uint(bv);
  }
}
__global__ void k_argmax1(const uint32_t* __restrict__ part, uint32_t* __restrict__ out, int parts) {
  pdl_wait();
  part += (size_t)blockIdx.x * parts * 2;       // row blockIdx.x
  out += (size_t)blockIdx.x * 2;
  float bv = -3.0e38f;
  uint32_t bi = 0xffffffffu;
  for (int i = threadIdx.x; i < parts; i += blockDim.x) argmax_merge(bv, bi, __uint_as_float(part[2 * i + 1]), part[2 * i]);
  block_argmax(bv, bi);
  if (threadIdx.x == 0) {
    out[0] = bi;
    out[1] = __float_as_uint(bv);
  }
}

__global__ void k_feedtok(const uint32_t* __restrict__ amax, uint32_t* __restrict__ params, uint32_t* __restrict__ ring,
                          int ring_cap) {
  pdl_wait();
  const uint32_t t = amax[0];
  if (ring) ring[params[6] % (uint32_t)ring_cap] = t;
  params[2] = t;
  params[0] += 1;
  params[1] += 1;
  params[4] += 1;
  params[5] += 1;
  params[6] += 1;
}

// Batched token feedback: token b of the step -> tok[b] and ring[b][params[6] % cap];
// the shared position block advances once.
__global__ void k_feedtok_rows(const uint32_t* __restrict__ amax, uint32_t* __restrict__ params,
                               uint32_t* __restrict__ ring, int ring_cap, uint32_t* __restrict__ tok, int rows) {
  pdl_wait();
  const uint32_t ri = params[6];
  for (int b = threadIdx.x; b < rows; b += blockDim.x) {
    const uint32_t t = amax[2 * b];
    tok[b] = t;
    if (ring) ring[(size_t)b * ring_cap + ri % (uint32_t)ring_cap] = t;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    params[2] = amax[0];
    params[0] += 1;
    params[1] += 1;
    params[4] += 1;
    params[5] += 1;
    params[6] += 1;
  }
}

}  // namespace

extern "C" {

E4B_API int e4b_routertop(e4b_ctx* c, const float* x, const float* wr, const float* pes, uint32_t* topk_idx,
                          float* topk_w, int H, int E, int K, int batch) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, x && wr && pes && topk_idx && topk_w, "routertop: null buffer");
  E4B_REQUIRE(c, H > 0 && E > 0 && E <= 4096 && K > 0 && K <= 32 && K <= E, "routertop: bad sizes H=%d E=%d K=%d", H,
              E, K);
  if (batch < 1) batch = 1;
  const int slices = (H + kRtK - 1) / kRtK;
  const size_t part_bytes = (size_t)slices * batch * E * 4;
  if (c->ws && c->ws_bytes >= e4b::kWsCounterBytes + part_bytes && (size_t)E * 4 <= 48 * 1024) {
    // the split-K partial area of the workspace (free between launches)
    float* part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(c->ws) + e4b::kWsCounterBytes);
    if (int r = e4b_launch(c, "router_part", k_router_part,
                           dim3((batch + kRtTok - 1) / kRtTok, (E + kRtExp - 1) / kRtExp, slices), dim3(256), 0, x,
                           wr, part, batch, H, E))
      return r;
    return e4b_launch(c, "router_topk", k_router_topk, dim3(batch), dim3(E < 256 ? ((E + 31) / 32) * 32 : 256),
                      (size_t)E * 4, (const float*)part, pes, topk_idx, topk_w, batch, E, K, slices);
  }
  return e4b_launch(c, "routertop", k_routertop, dim3(batch), dim3(256), (size_t)E * 4, x, wr, pes, topk_idx, topk_w,
                    H, E, K);
}

E4B_API int e4b_route_zipf(e4b_ctx* c, const uint32_t* params, uint32_t* topk_idx, float* topk_w, int n_tok, int K,
                           int E, float s, uint32_t seed, int salt, int tok0) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, params && topk_idx && topk_w && n_tok > 0 && K > 0 && K <= 32 && K <= E && E <= 4096 && s > 0.f,
              "route_zipf: bad args");
  return e4b_launch(c, "route_zipf", k_route_zipf, dim3((n_tok + 7) / 8), dim3(256), (size_t)E * 8, params, topk_idx,
                    topk_w, n_tok, K, E, s, seed, salt, tok0, n_tok);
}

E4B_API int e4b_zipf_table(e4b_ctx* c, float* table, int E, float s, uint32_t seed) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, table && E > 0 && E <= 4096 && s > 0.f, "zipf_table: bad args");
  return e4b_launch(c, "zipf_table", k_zipf_table, dim3(1), dim3(256), (size_t)E * 8, table, E, s, seed);
}

E4B_API int e4b_route_zipf_layers(e4b_ctx* c, const uint32_t* params, const float* table, uint32_t* topk_idx,
                                  float* topk_w, int n_tok, int n_layers, int K, int E, uint32_t seed, int salt0,
                                  int tok0) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, params && table && topk_idx && topk_w && n_tok > 0 && n_layers > 0 && K > 0 && K <= 32 && K <= E &&
                     E <= 4096,
              "route_zipf_layers: bad args");
  const long long rows = (long long)n_tok * n_layers;
  return e4b_launch(c, "route_zipf_layers", k_route_zipf_layers, dim3((unsigned)((rows + 7) / 8)), dim3(256),
                    (size_t)E * 8, params, table, topk_idx, topk_w, n_tok, n_layers, K, E, seed, salt0, tok0);
}

E4B_API int e4b_route_zipf_rows(e4b_ctx* c, const uint32_t* params, uint32_t* topk_idx, float* topk_w, int nseq,
                                int npos, int K, int E, float s, uint32_t seed, int salt, int tok0) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, params && topk_idx && topk_w && nseq > 0 && npos > 0 && K > 0 && K <= 32 && K <= E && E <= 4096 &&
                     s > 0.f,
              "route_zipf_rows: bad args");
  // every CTA builds the popularity table itself, then routes its rows (a warp per row)
  return e4b_launch(c, "route_zipf", k_route_zipf, dim3((nseq * npos + 7) / 8), dim3(256), (size_t)E * 8, params,
                    topk_idx, topk_w, nseq * npos, K, E, s, seed, salt, tok0, nseq);
}

E4B_API int e4b_router(e4b_ctx* c, const float* h, const float* scale, const float* wr, const float* pes,
                       uint32_t* topk_idx, float* topk_w, int H, int E, int K, float eps) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, h && scale && wr && pes && topk_idx && topk_w, "router: null buffer");
  E4B_REQUIRE(c, H > 0 && E > 0 && E <= 4096 && K > 0 && K <= 32 && K <= E, "router: bad sizes");
  return e4b_launch(c, "router", k_router, dim3(1), dim3(256), (size_t)E * 4, h, scale, wr, pes, topk_idx, topk_w, H,
                    E, K, eps);
}

E4B_API int e4b_top8(e4b_ctx* c, const float* scores, const float* pes, uint32_t* topk_idx, float* topk_w, int E,
                     int K) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, scores && pes && topk_idx && topk_w && E > 0 && E <= 4096 && K > 0 && K <= 32 && K <= E,
              "top8: bad args");
  return e4b_launch(c, "top8", k_top8, dim3(1), dim3(32), (size_t)E * 4, scores, pes, topk_idx, topk_w, E, K);
}

E4B_API int e4b_argmax(e4b_ctx* c, const float* x, uint32_t* part, uint32_t* out, int N, int parts) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, x && part && out && N > 0 && parts > 0 && parts <= 4096, "argmax: bad args");
  if (int r = e4b_launch(c, "argmax0", k_argmax0, dim3(parts), dim3(256), 0, x, part, N, parts)) return r;
  return e4b_launch(c, "argmax1", k_argmax1, dim3(1), dim3(256), 0, (const uint32_t*)part, out, parts);
}

}  // extern "C"

// ---- argmax without caller scratch.
// Some hosts may not allocate device memory once they are serving: a runtime
// that handed all free HBM to its KV cache at start-up, or one that must not
// call cudaMalloc on the decode path because it synchronises the device and can
// fail under memory pressure in the middle of a request.  For them the stage-0
// partials of the argmax live in this fixed module-level array instead of a
// caller-provided buffer.  Its address is looked up once per device (with that
// device current) and cached; nothing in it needs to start at zero, because
// stage 0 writes every partial stage 1 reads.  All callers on a device share
// it, so two such argmax calls in flight at the same time race.
namespace {
constexpr int kStaticArgmaxParts = 4096;
__device__ __align__(256) uint32_t g_argmax_part[2 * kStaticArgmaxParts];
constexpr int kMaxDevices = 64;
std::mutex g_argmax_mu;
uint32_t* g_argmax_addr[kMaxDevices] = {};

int static_part_addr(e4b_ctx* c, uint32_t** out) {
  E4B_REQUIRE(c, c->device >= 0 && c->device < kMaxDevices, "argmax_static: device %d out of range", c->device);
  std::lock_guard<std::mutex> lock(g_argmax_mu);
  if (!g_argmax_addr[c->device]) {
    E4B_CUDA(c, cudaSetDevice(c->device));
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_argmax_part);
    if (e != cudaSuccess || !p)
      return e4b_fail(c, E4B_ECUDA, "argmax_static: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_argmax_addr[c->device] = static_cast<uint32_t*>(p);
  }
  *out = g_argmax_addr[c->device];
  return E4B_OK;
}
}  // namespace

extern "C" {

E4B_API int e4b_argmax_static(e4b_ctx* c, const float* x, uint32_t* out, int N, int parts) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, x && out && N > 0, "argmax_static: bad args");
  E4B_REQUIRE(c, parts > 0 && parts <= kStaticArgmaxParts, "argmax_static: parts %d outside 1..%d", parts,
              kStaticArgmaxParts);
  uint32_t* part = nullptr;
  if (int r = static_part_addr(c, &part)) return r;
  if (int r = e4b_launch(c, "argmax0", k_argmax0, dim3(parts), dim3(256), 0, x, part, N, parts)) return r;
  return e4b_launch(c, "argmax1", k_argmax1, dim3(1), dim3(256), 0, (const uint32_t*)part, out, parts);
}

E4B_API int e4b_argmax_rows(e4b_ctx* c, const float* x, uint32_t* part, uint32_t* out, int N, int parts, int rows) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, x && part && out && N > 0 && parts > 0 && parts <= 4096 && rows > 0, "argmax_rows: bad args");
  if (int r = e4b_launch(c, "argmax0", k_argmax0, dim3(parts, rows), dim3(256), 0, x, part, N, parts)) return r;
  return e4b_launch(c, "argmax1", k_argmax1, dim3(rows), dim3(256), 0, (const uint32_t*)part, out, parts);
}

E4B_API int e4b_feedtok_rows(e4b_ctx* c, const uint32_t* amax, uint32_t* params, uint32_t* ring, int ring_cap,
                             uint32_t* tok, int rows) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, amax && params && tok && rows > 0 && (!ring || ring_cap > 0), "feedtok_rows: bad args");
  return e4b_launch(c, "feedtok_rows", k_feedtok_rows, dim3(1), dim3(256), 0, amax, params, ring, ring_cap, tok, rows);
}

E4B_API int e4b_feedtok(e4b_ctx* c, const uint32_t* amax, uint32_t* params, uint32_t* ring, int ring_cap) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, amax && params && (!ring || ring_cap > 0), "feedtok: bad args");
  return e4b_launch(c, "feedtok", k_feedtok, dim3(1), dim3(1), 0, amax, params, ring, ring_cap);
}

}  // extern "C"
