// Decode attention: head prep (q/k RMSNorm + RoPE, v norm, f16 KV write),
// RoPE, KV write, and split-KV flash-decode (phase A partials + phase B LSE merge)
// over the f16 KV cache with GQA, sliding ring and global (linear) layers.
#include "attn.cuh"

namespace {
using e4b::SlotRule;

E4B_DEV float rope_theta(uint32_t pos, int p, int HD, float theta) {
  // pos * THETA^(-2p/HD), in f32 (kernels/headprep.wgsl:55)
  const float ex = (-2.0f * (float)p) / (float)HD;
  return (float)pos * powf(theta, ex);
}

__global__ void k_headprep(const float* __restrict__ qkv, const float* __restrict__ qw, const float* __restrict__ kw,
                           const uint32_t* __restrict__ params, uint16_t* __restrict__ kcache,
                           uint16_t* __restrict__ vcache, float* __restrict__ q_out, int QH, int KVH, int HD,
                           int angles, float theta, float eps, int keqv, int cachemode, int ring, int cache_slots,
                           uint32_t* status, size_t seq_stride, int nparts, size_t part_stride, int nseq) {
  pdl_wait();
  __shared__ float sh[32];
  __shared__ float xv[512];                      // this head's qkv row (the sum of nparts K-part partials)
  const int head = blockIdx.x, b = blockIdx.y;
  // seq_stride > 0: row b is sequence b % nseq at position params[0] + b / nseq
  // (position-major rows of nseq sequences; one position when there are nseq
  // rows), with its own cache at kcache / vcache + (b % nseq) * seq_stride; else
  // rows are consecutive positions of one sequence
  if (seq_stride) {
    kcache += (size_t)(b % nseq) * seq_stride;
    vcache += (size_t)(b % nseq) * seq_stride;
  }
  const uint32_t pb = seq_stride ? (uint32_t)(b / nseq) : (uint32_t)b;
  int src = head;
  if (keqv && head >= QH + KVH) src = head - KVH;  // v reads the k slice
  const size_t qkvS = (size_t)(QH + KVH * (2 - keqv)) * HD;
  const size_t base = (size_t)b * qkvS + (size_t)src * HD;
  // up to four elements per thread (HD <= 4 * blockDim), all their partial
  // loads in flight together
  float s = 0.f, v4[4];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const int d = threadIdx.x + j * blockDim.x;
    v4[j] = d < HD ? sum_parts(qkv + base + d, part_stride, nparts) : 0.f;
  }
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const int d = threadIdx.x + j * blockDim.x;
    if (d < HD) {
      xv[d] = v4[j];
      s = fmaf(v4[j], v4[j], s);
    }
  }
  const float inv = rms_scale(block_sum(s, sh), HD, eps);
  const int half = HD / 2;
  const uint32_t pos = params[0] + pb;
  uint32_t slot = pos;
  if (cachemode == 1) slot = pos % (uint32_t)ring;
  if (cachemode == 2) slot = params[4] + pb;
  if (head >= QH && slot >= (uint32_t)cache_slots) {
    if (threadIdx.x == 0) set_status(status, E4B_ST_BADINDEX);
    return;
  }
  if (head < QH) {
    float* qo = q_out + ((size_t)b * QH + head) * HD;
    for (int p = threadIdx.x; p < half; p += blockDim.x) {
      const float x0 = xv[p] * inv * qw[p];
      const float x1 = xv[p + half] * inv * qw[p + half];
      if (p < angles) {
        float sn, cs;
        sincosf(rope_theta(pos, p, HD, theta), &sn, &cs);
        qo[p] = x0 * cs - x1 * sn;
        qo[p + half] = x0 * sn + x1 * cs;
      } else {
        qo[p] = x0;
        qo[p + half] = x1;
      }
    }
  } else if (head < QH + KVH) {
    const int h = head - QH;
    uint16_t* kc = kcache + ((size_t)slot * KVH + h) * HD;
    for (int p = threadIdx.x; p < half; p += blockDim.x) {
      const float x0 = xv[p] * inv * kw[p];
      const float x1 = xv[p + half] * inv * kw[p + half];
      if (p < angles) {
        float sn, cs;
        sincosf(rope_theta(pos, p, HD, theta), &sn, &cs);
        kc[p] = f2h(x0 * cs - x1 * sn);
        kc[p + half] = f2h(x0 * sn + x1 * cs);
      } else {
        kc[p] = f2h(x0);
        kc[p + half] = f2h(x1);
      }
    }
  } else {
    const int h = head - QH - KVH;
    uint16_t* vc = vcache + ((size_t)slot * KVH + h) * HD;
    for (int d = threadIdx.x; d < HD; d += blockDim.x) vc[d] = f2h(xv[d] * inv);
  }
}

__global__ void k_rope(float* __restrict__ x, const uint32_t* __restrict__ params, int heads, int HD, int angles,
                       float theta) {
  pdl_wait();
  const int half = HD / 2;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= heads * half) return;
  const int h = idx / half, p = idx % half;
  if (p >= angles) return;
  float sn, cs;
  sincosf(rope_theta(params[0], p, HD, theta), &sn, &cs);
  const size_t i0 = (size_t)h * HD + p, i1 = i0 + half;
  const float x0 = x[i0], x1 = x[i1];
  x[i0] = x0 * cs - x1 * sn;
  x[i1] = x0 * sn + x1 * cs;
}

__global__ void k_kvwrite(const float* __restrict__ src, const uint32_t* __restrict__ params, float* __restrict__ dst,
                          int N) {
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < N) dst[(size_t)params[0] * N + i] = src[i];
}

// Number of addressable slots and whether slot t is attended, for the query at
// position qp (kernels/attnf32.wgsl:28-53, attsplit.wgsl:21-23).


// Phase A: CTA (head h, chunk c) scores `chunk` slots (one per thread), then
// accumulates p_t * v_t over its dims.  Output unnormalised with local (m, l).
__global__ void k_attsplit(const float* __restrict__ q, const uint16_t* __restrict__ kcache,
                           const uint16_t* __restrict__ vcache, const uint32_t* __restrict__ params,
                           float* __restrict__ part_o, float* __restrict__ part_ml, int QH, int KVH, int HD,
                           int window, int cachemode, int ring, int max_chunks, float scale, size_t seq_stride) {
  pdl_wait();
  {   // sequence blockIdx.z: its q rows, cache and partials
    const size_t z = blockIdx.z;
    q += z * QH * HD;
    kcache += z * seq_stride;
    vcache += z * seq_stride;
    part_o += z * QH * max_chunks * HD;
    part_ml += z * QH * max_chunks * 2;
  }
  extern __shared__ float smem[];
  float* qs = smem;            // [HD]
  float* ps = smem + HD;       // [chunk]
  __shared__ float sh[32];
  const int h = blockIdx.x, c = blockIdx.y, chunk = blockDim.x;
  const int kvh = h / (QH / KVH);
  SlotRule rule{cachemode, ring, window, 0, 0};
  rule.qp = params[0];
  rule.len = cachemode == 2 ? params[5] : params[1];
  const uint32_t n = rule.nslots();
  const uint32_t t0 = (uint32_t)c * chunk;
  const size_t pi = (size_t)h * max_chunks + c;
  for (int d = threadIdx.x; d < HD; d += chunk) qs[d] = q[(size_t)h * HD + d];
  __syncthreads();
  const uint32_t t = t0 + threadIdx.x;
  const bool ok = t < n && rule.valid(t);
  float s = -INFINITY;
  if (ok) {
    const uint16_t* kr = kcache + ((size_t)t * KVH + kvh) * HD;
    float acc = 0.f;
    for (int d = 0; d < HD; d += 2) {
      const __half2 kv = *reinterpret_cast<const __half2*>(kr + d);
      const float2 kf = __half22float2(kv);
      acc = fmaf(qs[d], kf.x, acc);
      acc = fmaf(qs[d + 1], kf.y, acc);
    }
    s = acc * scale;
  }
  const float m = block_max(s, sh);
  const float p = ok ? expf(s - m) : 0.f;
  ps[threadIdx.x] = p;
  const float l = block_sum(p, sh);
  if (threadIdx.x == 0) {
    part_ml[2 * pi] = l > 0.f ? m : -INFINITY;
    part_ml[2 * pi + 1] = l;
  }
  const uint32_t hi = min(t0 + (uint32_t)chunk, n);
  for (int d = threadIdx.x; d < HD; d += chunk) {
    float acc = 0.f;
    for (uint32_t tt = t0; tt < hi; tt++) {
      const float pp = ps[tt - t0];
      if (pp != 0.f) acc = fmaf(pp, h2f(vcache[((size_t)tt * KVH + kvh) * HD + d]), acc);
    }
    part_o[pi * HD + d] = acc;
  }
}

__global__ void k_attcomb(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                          uint16_t* __restrict__ out_h, float* __restrict__ out_f, float* __restrict__ lse, int HD,
                          int max_chunks, int xfo) {
  pdl_wait();
  {   // sequence blockIdx.y
    const size_t z = blockIdx.y, QH = gridDim.x;
    part_o += z * QH * max_chunks * HD;
    part_ml += z * QH * max_chunks * 2;
    if (out_h) out_h += z * QH * HD;
    if (out_f) out_f += z * QH * HD;
    if (lse) lse += z * QH;
  }
  const int h = blockIdx.x;
  const float* ml = part_ml + (size_t)h * max_chunks * 2;
  float M = -INFINITY;
  for (int c = 0; c < max_chunks; c++)
    if (ml[2 * c + 1] > 0.f) M = fmaxf(M, ml[2 * c]);
  float den = 0.f;
  for (int c = 0; c < max_chunks; c++)
    if (ml[2 * c + 1] > 0.f) den += ml[2 * c + 1] * expf(ml[2 * c] - M);
  for (int d = threadIdx.x; d < HD; d += blockDim.x) {
    float acc = 0.f;
    for (int c = 0; c < max_chunks; c++)
      if (ml[2 * c + 1] > 0.f) acc = fmaf(part_o[((size_t)h * max_chunks + c) * HD + d], expf(ml[2 * c] - M), acc);
    const float v = den > 0.f ? acc / den : 0.f;
    if (out_h) out_h[xfo ? xfo_pos(h * HD + d) : h * HD + d] = f2h(v);
    if (out_f) out_f[(size_t)h * HD + d] = v;
  }
  if (lse && threadIdx.x == 0) lse[h] = den > 0.f ? M + logf(den) : -INFINITY;
}


// Attention-mass score pass of a counted (linear) cache (the SCORE=1 pass of
// kernels/attnos.wgsl:82-97): for every live slot t < len (len = params[5]) and
// query head h, score[h][t] += exp(scale * q_h . k_t - lse_h), the head's
// normalised attention probability of slot t, accumulated across decode steps.
// One thread per slot; the G query heads of its KV head share the K row.
__global__ void k_attn_score(const float* __restrict__ q, const uint16_t* __restrict__ kcache,
                             const float* __restrict__ lse, const uint32_t* __restrict__ params,
                             float* __restrict__ score, int QH, int KVH, int HD, float scale, int scap) {
  pdl_wait();
  extern __shared__ float qs[];                 // [G][HD]
  const int kvh = blockIdx.y, G = QH / KVH;
  for (int i = threadIdx.x; i < G * HD; i += blockDim.x) qs[i] = q[(size_t)kvh * G * HD + i];
  __syncthreads();
  const uint32_t len = params[5];
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if ((uint32_t)t >= len || t >= scap) return;
  const uint16_t* k = kcache + ((size_t)t * KVH + kvh) * HD;
  float acc[8];
#pragma unroll
  for (int g = 0; g < 8; g++) acc[g] = 0.f;
  for (int d = 0; d < HD; d += 8) {
    const uint4 kv = *reinterpret_cast<const uint4*>(k + d);
    const uint32_t w[4] = {kv.x, kv.y, kv.z, kv.w};
    float kf[8];
#pragma unroll
    for (int e = 0; e < 4; e++) {
      kf[2 * e] = h2f((uint16_t)(w[e] & 0xFFFFu));
      kf[2 * e + 1] = h2f((uint16_t)(w[e] >> 16));
    }
#pragma unroll
    for (int g = 0; g < 8; g++) {
      if (g >= G) break;
#pragma unroll
      for (int e = 0; e < 8; e++) acc[g] = fmaf(qs[g * HD + d + e], kf[e], acc[g]);
    }
  }
#pragma unroll
  for (int g = 0; g < 8; g++) {
    if (g >= G) break;
    const int h = kvh * G + g;
    score[(size_t)h * scap + t] += expf(acc[g] * scale - lse[h]);
  }
}

// kernels/kvgather.wgsl:9-18: dst slot i <- src slot keep[i], K and V.
__global__ void k_kvgather(const uint32_t* __restrict__ keep, const uint16_t* __restrict__ src_k,
                           const uint16_t* __restrict__ src_v, uint16_t* __restrict__ dst_k,
                           uint16_t* __restrict__ dst_v, int row, int src_slots) {
  pdl_wait();
  const int i = blockIdx.x;
  const uint32_t s = keep[i];
  if (s >= (uint32_t)src_slots) return;
  const uint4* sk = reinterpret_cast<const uint4*>(src_k + (size_t)s * row);
  const uint4* sv = reinterpret_cast<const uint4*>(src_v + (size_t)s * row);
  uint4* dk = reinterpret_cast<uint4*>(dst_k + (size_t)i * row);
  uint4* dv = reinterpret_cast<uint4*>(dst_v + (size_t)i * row);
  for (int e = threadIdx.x; e < row / 8; e += blockDim.x) {
    dk[e] = sk[e];
    dv[e] = sv[e];
  }
}
}  // namespace

extern "C" {

E4B_API int e4b_headprep(e4b_ctx* c, const float* qkv, const float* qw, const float* kw, const uint32_t* params,
                         uint16_t* kcache, uint16_t* vcache, float* q_out, int QH, int KVH, int HD, int rope_angles,
                         float theta, float eps, int keqv, int cachemode, int ring, int cache_slots, int batch) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, qkv && qw && kw && params && kcache && vcache && q_out, "headprep: null buffer");
  E4B_REQUIRE(c, QH > 0 && KVH > 0 && QH % KVH == 0 && HD > 0 && HD <= 512 && HD % 2 == 0 && rope_angles >= 0 &&
                     rope_angles <= HD / 2 && cache_slots > 0,
              "headprep: bad geometry QH=%d KVH=%d HD=%d angles=%d", QH, KVH, HD, rope_angles);
  E4B_REQUIRE(c, cachemode >= 0 && cachemode <= 2 && (cachemode != 1 || (ring > 0 && ring <= cache_slots)),
              "headprep: bad cache mode %d / ring %d", cachemode, ring);
  if (batch < 1) batch = 1;
  return e4b_launch(c, "headprep", k_headprep, dim3(QH + 2 * KVH, batch), dim3(128), 0, qkv, qw, kw, params, kcache,
                    vcache, q_out, QH, KVH, HD, rope_angles, theta, eps, keqv ? 1 : 0, cachemode, ring, cache_slots,
                    c->status, (size_t)0, 1, (size_t)0, 1);
}

E4B_API int e4b_headprep_seq(e4b_ctx* c, const float* qkv, const float* qw, const float* kw, const uint32_t* params,
                             uint16_t* kcache, uint16_t* vcache, float* q_out, int QH, int KVH, int HD,
                             int rope_angles, float theta, float eps, int keqv, int cachemode, int ring,
                             int cache_slots, int nseq, int nparts) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, qkv && qw && kw && params && kcache && vcache && q_out && nseq > 0, "headprep_seq: bad args");
  E4B_REQUIRE(c, nparts >= 1 && HD <= 512, "headprep_seq: nparts=%d, HD=%d (<= 512)", nparts, HD);
  E4B_REQUIRE(c, QH > 0 && KVH > 0 && QH % KVH == 0 && HD > 0 && HD % 2 == 0 && rope_angles >= 0 &&
                     rope_angles <= HD / 2 && cache_slots > 0,
              "headprep_seq: bad geometry QH=%d KVH=%d HD=%d angles=%d", QH, KVH, HD, rope_angles);
  E4B_REQUIRE(c, cachemode >= 0 && cachemode <= 2 && (cachemode != 1 || (ring > 0 && ring <= cache_slots)),
              "headprep_seq: bad cache mode %d / ring %d", cachemode, ring);
  const size_t stride = (size_t)cache_slots * KVH * HD;
  return e4b_launch(c, "headprep_seq", k_headprep, dim3(QH + 2 * KVH, nseq), dim3(128), 0, qkv, qw, kw, params,
                    kcache, vcache, q_out, QH, KVH, HD, rope_angles, theta, eps, keqv ? 1 : 0, cachemode, ring,
                    cache_slots, c->status, stride, nparts,
                    (size_t)nseq * (QH + KVH * (2 - (keqv ? 1 : 0))) * HD, nseq);
}

E4B_API int e4b_headprep_rows(e4b_ctx* c, const float* qkv, const float* qw, const float* kw, const uint32_t* params,
                              uint16_t* kcache, uint16_t* vcache, float* q_out, int QH, int KVH, int HD,
                              int rope_angles, float theta, float eps, int keqv, int cachemode, int ring,
                              int cache_slots, int nseq, int npos) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, qkv && qw && kw && params && kcache && vcache && q_out && nseq > 0 && npos > 0,
              "headprep_rows: bad args");
  E4B_REQUIRE(c, HD <= 512 && (long long)nseq * npos <= 65535, "headprep_rows: HD=%d (<= 512), %d rows (<= 65535)",
              HD, nseq * npos);
  E4B_REQUIRE(c, QH > 0 && KVH > 0 && QH % KVH == 0 && HD > 0 && HD % 2 == 0 && rope_angles >= 0 &&
                     rope_angles <= HD / 2 && cache_slots > 0,
              "headprep_rows: bad geometry QH=%d KVH=%d HD=%d angles=%d", QH, KVH, HD, rope_angles);
  E4B_REQUIRE(c, cachemode >= 0 && cachemode <= 2 && (cachemode != 1 || (ring > 0 && ring <= cache_slots)),
              "headprep_rows: bad cache mode %d / ring %d", cachemode, ring);
  const size_t stride = (size_t)cache_slots * KVH * HD;
  return e4b_launch(c, "headprep_rows", k_headprep, dim3(QH + 2 * KVH, nseq * npos), dim3(128), 0, qkv, qw, kw,
                    params, kcache, vcache, q_out, QH, KVH, HD, rope_angles, theta, eps, keqv ? 1 : 0, cachemode, ring,
                    cache_slots, c->status, stride, 1, (size_t)0, nseq);
}

E4B_API int e4b_rope(e4b_ctx* c, float* x, const uint32_t* params, int heads, int HD, int rope_angles, float theta) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, x && params && heads > 0 && HD > 0 && HD % 2 == 0 && rope_angles <= HD / 2, "rope: bad args");
  const int n = heads * HD / 2;
  return e4b_launch(c, "rope", k_rope, dim3((n + 127) / 128), dim3(128), 0, x, params, heads, HD, rope_angles, theta);
}

E4B_API int e4b_kvwrite(e4b_ctx* c, const float* src, const uint32_t* params, float* dst, int N) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, src && params && dst && N > 0, "kvwrite: bad args");
  return e4b_launch(c, "kvwrite", k_kvwrite, dim3((N + 127) / 128), dim3(128), 0, src, params, dst, N);
}

E4B_API int e4b_attsplit(e4b_ctx* c, const float* q, const uint16_t* kcache, const uint16_t* vcache,
                         const uint32_t* params, float* part_o, float* part_ml, int QH, int KVH, int HD, int window,
                         int cachemode, int ring, int chunk, int max_chunks, float scale) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, q && kcache && vcache && params && part_o && part_ml, "attsplit: null buffer");
  E4B_REQUIRE(c, QH > 0 && KVH > 0 && QH % KVH == 0 && HD > 0 && HD % 2 == 0 && max_chunks > 0,
              "attsplit: bad geometry");
  E4B_REQUIRE(c, chunk >= 32 && chunk <= 1024 && (chunk & 31) == 0, "attsplit: chunk %d must be 32..1024, x32",
              chunk);
  E4B_REQUIRE(c, cachemode >= 0 && cachemode <= 2 && (cachemode != 1 || (ring > 0 && window > 0)),
              "attsplit: bad cache mode");
  const size_t sm = (size_t)(HD + chunk) * 4;
  return e4b_launch(c, "attsplit", k_attsplit, dim3(QH, max_chunks), dim3(chunk), sm, q, kcache, vcache, params,
                    part_o, part_ml, QH, KVH, HD, window, cachemode, ring, max_chunks, scale, (size_t)0);
}

E4B_API int e4b_attsplit_seq(e4b_ctx* c, const float* q, const uint16_t* kcache, const uint16_t* vcache,
                             const uint32_t* params, float* part_o, float* part_ml, int QH, int KVH, int HD,
                             int window, int cachemode, int ring, int chunk, int max_chunks, float scale,
                             int cache_slots, int nseq) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, q && kcache && vcache && params && part_o && part_ml && nseq > 0 && cache_slots > 0,
              "attsplit_seq: bad args");
  E4B_REQUIRE(c, QH > 0 && KVH > 0 && QH % KVH == 0 && HD > 0 && HD % 2 == 0 && max_chunks > 0,
              "attsplit_seq: bad geometry");
  E4B_REQUIRE(c, chunk >= 32 && chunk <= 1024 && (chunk & 31) == 0, "attsplit_seq: chunk %d must be 32..1024, x32",
              chunk);
  E4B_REQUIRE(c, cachemode >= 0 && cachemode <= 2 && (cachemode != 1 || (ring > 0 && window > 0)),
              "attsplit_seq: bad cache mode");
  const size_t sm = (size_t)(HD + chunk) * 4;
  const size_t stride = (size_t)cache_slots * KVH * HD;
  return e4b_launch(c, "attsplit_seq", k_attsplit, dim3(QH, max_chunks, nseq), dim3(chunk), sm, q, kcache, vcache,
                    params, part_o, part_ml, QH, KVH, HD, window, cachemode, ring, max_chunks, scale, stride);
}

E4B_API int e4b_attcomb(e4b_ctx* c, const float* part_o, const float* part_ml, uint16_t* out_h, float* out_f,
                        float* lse, int QH, int HD, int max_chunks) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, part_o && part_ml && (out_h || out_f) && QH > 0 && HD > 0 && max_chunks > 0, "attcomb: bad args");
  return e4b_launch(c, "attcomb", k_attcomb, dim3(QH), dim3(128), 0, part_o, part_ml, out_h, out_f, lse, HD,
                    max_chunks, 0);
}

E4B_API int e4b_attcomb_seq(e4b_ctx* c, const float* part_o, const float* part_ml, uint16_t* out_h, float* out_f,
                            float* lse, int QH, int HD, int max_chunks, int nseq, int xfo) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, part_o && part_ml && (out_h || out_f) && QH > 0 && HD > 0 && max_chunks > 0 && nseq > 0,
              "attcomb_seq: bad args");
  E4B_REQUIRE(c, !xfo || (QH * HD) % 32 == 0, "attcomb_seq: fragment order needs QH*HD %% 32 == 0");
  return e4b_launch(c, "attcomb_seq", k_attcomb, dim3(QH, nseq), dim3(128), 0, part_o, part_ml, out_h, out_f, lse,
                    HD, max_chunks, xfo);
}


E4B_API int e4b_attn_score(e4b_ctx* c, const float* q, const uint16_t* kcache, const float* lse,
                           const uint32_t* params, float* score, int QH, int KVH, int HD, float scale, int scap) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, q && kcache && lse && params && score && scap > 0, "attn_score: bad args");
  E4B_REQUIRE(c, QH > 0 && KVH > 0 && QH % KVH == 0 && QH / KVH <= 8 && HD > 0 && HD % 8 == 0,
              "attn_score: QH=%d KVH=%d HD=%d (<= 8 query heads per KV head, HD %% 8 == 0)", QH, KVH, HD);
  E4B_REQUIRE(c, reinterpret_cast<uintptr_t>(kcache) % 16 == 0, "attn_score: cache must be 16-byte aligned");
  return e4b_launch(c, "attn_score", k_attn_score, dim3((scap + 127) / 128, KVH), dim3(128),
                    (size_t)(QH / KVH) * HD * 4, q, kcache, lse, params, score, QH, KVH, HD, scale, scap);
}

E4B_API int e4b_kvgather(e4b_ctx* c, const uint32_t* keep, int n, const uint16_t* src_k, const uint16_t* src_v,
                         uint16_t* dst_k, uint16_t* dst_v, int KVH, int HD, int src_slots) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, keep && src_k && src_v && dst_k && dst_v && n > 0 && src_slots > 0, "kvgather: bad args");
  E4B_REQUIRE(c, KVH > 0 && HD > 0 && (KVH * HD) % 8 == 0, "kvgather: KVH*HD must be a multiple of 8");
  return e4b_launch(c, "kvgather", k_kvgather, dim3(n), dim3(128), 0, keep, src_k, src_v, dst_k, dst_v, KVH * HD,
                    src_slots);
}

}  // extern "C"
