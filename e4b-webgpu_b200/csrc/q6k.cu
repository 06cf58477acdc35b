// q6_K operators over raw GGUF blocks: token-embedding row (q6k MODE 0), LM head
// (q6k MODE 1, softcap) and the per-layer-embedding input prep (pleprep).
#include "common.cuh"
#include "q40_stream.cuh"

namespace {

// sum over the 16 elements of sub-block s of a q6_K block of (q-32)*x.
// The sub-block's ql bytes are 16 consecutive bytes at h*64 + 32*(j&1) + 16*(s&1)
// (nibble j>>1) and its qh bytes 16 consecutive bytes at 128 + h*32 + 16*(s&1)
// (bit pair j), with h = s/8, j = (s%8)/2   (kernels/q6k.wgsl:44-68).
E4B_DEV float q6k_sub_dot(const uint8_t* __restrict__ blk, int s, const float* __restrict__ x) {
  const int h = s >> 3, j = (s & 7) >> 1, half = s & 1;
  const unsigned short* ql = reinterpret_cast<const unsigned short*>(blk + h * 64 + 32 * (j & 1) + 16 * half);
  const unsigned short* qh = reinterpret_cast<const unsigned short*>(blk + 128 + h * 32 + 16 * half);
  const int nsh = (j >> 1) * 4, hsh = 2 * j;
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const uint32_t a = __ldg(ql + i), b = __ldg(qh + i);
    const int q0 = (int)(((a >> nsh) & 0xF) | (((b >> hsh) & 3) << 4)) - 32;
    const int q1 = (int)(((a >> (8 + nsh)) & 0xF) | (((b >> (8 + hsh)) & 3) << 4)) - 32;
    acc = fmaf((float)q0, x[2 * i], acc);
    acc = fmaf((float)q1, x[2 * i + 1], acc);
  }
  return acc;
}

__global__ void k_q6k_embed(const uint8_t* __restrict__ w, const uint32_t* __restrict__ params,
                            const uint32_t* __restrict__ tok, float* __restrict__ y, int N, int rows, float mult,
                            int toksrc, int batch, uint32_t* status) {
  pdl_wait();
  const int b = blockIdx.x;
  const uint32_t row = batch > 0 ? tok[b] : (toksrc ? tok[0] : params[2]);
  float* out = y + (size_t)b * N;
  if (row >= (uint32_t)rows) {
    if (threadIdx.x == 0) set_status(status, E4B_ST_BADINDEX);
    for (int i = threadIdx.x; i < N; i += blockDim.x) out[i] = 0.f;
    return;
  }
  const uint8_t* r = w + (size_t)row * (N / 256) * 210;
  for (int i = threadIdx.x; i < N; i += blockDim.x) out[i] = q6k_elem(r + (size_t)(i >> 8) * 210, i & 255) * mult;
}

// One warp per vocabulary row; lane handles sub-blocks lane, lane+32, ... of the row.
__global__ void __launch_bounds__(256) k_q6k_lmhead(const uint8_t* __restrict__ w, const float* __restrict__ x,
                                                    float* __restrict__ y, int N, int OUT, float softcap) {
  pdl_wait();
  const int o = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int b = blockIdx.y;
  if (o >= OUT) return;
  const int nb = N >> 8;
  const uint8_t* row = w + (size_t)o * nb * 210;
  const float* xr = x + (size_t)b * N;
  float acc = 0.f;
  for (int t = threadIdx.x & 31; t < nb * 16; t += 32) {
    const int blk = t >> 4, s = t & 15;
    const uint8_t* bp = row + (size_t)blk * 210;
    const float ds = q6k_d(bp) * (float)(int8_t)__ldg(bp + 192 + s);
    acc = fmaf(ds, q6k_sub_dot(bp, s, xr + blk * 256 + s * 16), acc);
  }
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) {
    float out = acc;
    if (softcap != 0.f) out = softcap * tanhf(out / softcap);
    y[(size_t)b * OUT + o] = out;
  }
}

__global__ void k_pleprep(const uint8_t* __restrict__ table, const uint32_t* __restrict__ params,
                          const uint32_t* __restrict__ tok, const float* __restrict__ proj,
                          const float* __restrict__ norm_w, float* __restrict__ ple_in, int PD, int LAYERS, int rows,
                          float mult, float proj_scale, float eps, int toksrc, uint32_t* status) {
  pdl_wait();
  __shared__ float sh[32];
  const int blk = blockIdx.x;
  const int base = blk * PD;
  float ss = 0.f;
  for (int i = threadIdx.x; i < PD; i += blockDim.x) {
    const float v = proj[base + i] * proj_scale;
    ss = fmaf(v, v, ss);
  }
  const float inv = rms_scale(block_sum(ss, sh), PD, eps);
  const uint32_t row = toksrc ? tok[0] : params[2];
  if (row >= (uint32_t)rows) {
    if (threadIdx.x == 0) set_status(status, E4B_ST_BADINDEX);
    return;
  }
  const int width = LAYERS * PD;
  const uint8_t* r = table + (size_t)row * (width / 256) * 210;
  for (int i = threadIdx.x; i < PD; i += blockDim.x) {
    const int gi = base + i;
    const float idv = q6k_elem(r + (size_t)(gi >> 8) * 210, gi & 255) * mult;
    const float p = proj[gi] * proj_scale;
    ple_in[gi] = (p * inv * norm_w[i] + idv) * 0.70710678118654752f;
  }
}

}  // namespace

extern "C" {

E4B_API int e4b_q6k_embed(e4b_ctx* c, const uint8_t* w, const uint32_t* params, const uint32_t* tok, float* y,
                          int N, int rows, float mult, int toksrc, int batch) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, w && y && N > 0 && N % 256 == 0 && rows > 0, "q6k_embed: bad args (N=%d must be a multiple of 256)",
              N);
  E4B_REQUIRE(c, (batch > 0 || toksrc) ? tok != nullptr : params != nullptr, "q6k_embed: missing token source");
  return e4b_launch(c, "q6k_embed", k_q6k_embed, dim3(batch > 0 ? batch : 1), dim3(256), 0, w, params, tok, y, N,
                    rows, mult, toksrc, batch, c->status);
}

E4B_API int e4b_q6k_lmhead(e4b_ctx* c, const uint8_t* w, const float* x, float* y, int N, int OUT, float softcap,
                           int batch) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, w && x && y && N > 0 && N % 256 == 0 && OUT > 0, "q6k_lmhead: bad args");
  if (batch < 1) batch = 1;
  if (batch == 1 && e4b::lmhead_stream_supported(w, x, N)) return e4b::lmhead_stream(c, w, x, y, N, OUT, softcap);
  return e4b_launch(c, "q6k_lmhead", k_q6k_lmhead, dim3((OUT + 7) / 8, batch), dim3(256), 0, w, x, y, N, OUT,
                    softcap);
}

E4B_API int e4b_pleprep(e4b_ctx* c, const uint8_t* table, const uint32_t* params, const uint32_t* tok,
                        const float* proj, const float* norm_w, float* ple_in, int PD, int LAYERS, int rows,
                        float mult, float proj_scale, float eps, int toksrc) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, table && proj && norm_w && ple_in && PD > 0 && LAYERS > 0 && rows > 0, "pleprep: bad args");
  E4B_REQUIRE(c, (PD * LAYERS) % 256 == 0, "pleprep: table row LAYERS*PD=%d must be a multiple of 256", PD * LAYERS);
  E4B_REQUIRE(c, toksrc ? tok != nullptr : params != nullptr, "pleprep: missing token source");
  return e4b_launch(c, "pleprep", k_pleprep, dim3(LAYERS), dim3(128), 0, table, params, tok, proj, norm_w, ple_in,
                    PD, LAYERS, rows, mult, proj_scale, eps, toksrc, c->status);
}

}  // extern "C"
