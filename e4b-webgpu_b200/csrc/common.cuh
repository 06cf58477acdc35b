// Shared definitions for the e4b_b200 kernels and runtime (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>

#include <vector>

#include "e4b_b200.h"

#define E4B_DEV __device__ __forceinline__

// ------------------------------------------------------------------ context
struct e4b_ctx {
  int device = 0;
  int sm_count = 0;
  cudaStream_t stream = nullptr;
  bool pdl = true;
  bool capturing = false;
  uint32_t* status = nullptr;       // device status word (bounded waits / checks)
  void* ws = nullptr;               // caller-provided workspace (split-K partials, counters)
  size_t ws_bytes = 0;
  int stream_ctas_per_sm = 1;       // tuning knobs (e4b_set_option)
  int stream_stages = 4;
  int stream_variant = 0;           // GEMV warps x piece size: 0 = 8x32, 1 = 16x16, 2 = 16x8
  int attn_grid_cap = 0;            // batched attention: at most this many CTAs (0 = one per SM)
  uint64_t wait_ns = 1000000000ull; // bound of the batched attention's and ep_wait's device waits
  int lmhead_tc_min = 1;             // batched LM head: tcgen05 kernel for n >= this (<= 64)
  int lmhead_tiles_tc = 0;           // packed LM head, 2..64 rows: 0 = by row count, 1 = tcgen05, 2 = warp-MMA
  cudaStream_t main_stream = nullptr;  // e4b_side_begin .. e4b_side_end: launches go to `side`
  cudaStream_t side = nullptr;
  cudaEvent_t fork_ev = nullptr, join_ev = nullptr;
  bool forked = false, side_pending = false;
  cudaEvent_t ev[64] = {};
  std::vector<cudaGraphExec_t> plans;
  cudaGraph_t cap_graph = nullptr;
  char err[1024] = {0};
};

int e4b_fail(e4b_ctx* c, int code, const char* fmt, ...);
namespace e4b {
void dense_plans_release(e4b_ctx* c);   // frees a context's fused token plans
void nccl_release(e4b_ctx* c);          // destroys a context's NCCL communicator
}

#define E4B_CHECK_CTX(c) \
  do {                   \
    if (!(c)) return E4B_EINVAL; \
  } while (0)
#define E4B_REQUIRE(c, cond, ...) \
  do {                            \
    if (!(cond)) return e4b_fail((c), E4B_EINVAL, __VA_ARGS__); \
  } while (0)
#define E4B_CUDA(c, call)                                                              \
  do {                                                                                 \
    cudaError_t _e = (call);                                                           \
    if (_e != cudaSuccess) return e4b_fail((c), E4B_ECUDA, "%s: %s", #call, cudaGetErrorString(_e)); \
  } while (0)

// Launch on the context stream; with PDL enabled the kernel may start while its
// predecessor drains, so every kernel calls pdl_wait() before touching data a
// predecessor produced.
template <typename... KArgs, typename... Args>
static inline int e4b_launch(e4b_ctx* c, const char* name, void (*kern)(KArgs...), dim3 grid, dim3 block,
                             size_t smem, Args... args) {
  if (grid.x == 0 || grid.y == 0 || grid.z == 0) return E4B_OK;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = c->stream;
  cudaLaunchAttribute attr[1];
  cfg.numAttrs = 0;
  if (c->pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) return e4b_fail(c, E4B_ECUDA, "%s launch: %s", name, cudaGetErrorString(e));
  return E4B_OK;
}

// ------------------------------------------------------------------ device helpers
// Programmatic dependent launch: wait for the previous grid's results, and let
// the next grid get scheduled early.
E4B_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
E4B_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" :::); }

E4B_DEV float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
E4B_DEV uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

// p[0] + p[stride] + ... + p[(n - 1) stride], added in that order (the K-split
// GEMMs' partials); the loads are issued eight at a time, not one per add.
E4B_DEV float sum_parts(const float* __restrict__ p, size_t stride, int n) {
  float v = 0.f;
  for (int k0 = 0; k0 < n; k0 += 8) {
    float x[8];
#pragma unroll
    for (int k = 0; k < 8; k++) x[k] = k0 + k < n ? p[(size_t)(k0 + k) * stride] : 0.f;
#pragma unroll
    for (int k = 0; k < 8; k++)
      if (k0 + k < n) v = (k0 + k == 0) ? x[k] : v + x[k];
  }
  return v;
}

E4B_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
E4B_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum; `sh` is >= 32 floats of shared memory; all threads get the result.
E4B_DEV float block_sum(float v, float* sh) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) sh[wid] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; i++) t += sh[i];
  return t;
}
E4B_DEV float block_max(float v, float* sh) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) sh[wid] = v;
  __syncthreads();
  float t = -INFINITY;
  for (int i = 0; i < nw; i++) t = fmaxf(t, sh[i]);
  return t;
}

// (mean(x^2) + eps)^-1/2 as the reference writes it: pow(ms + eps, -0.5).
E4B_DEV float rms_scale(float sumsq, int n, float eps) { return 1.0f / sqrtf(sumsq / (float)n + eps); }

// gelu_pytorch_tanh with the reference's inner clamp (kernels/q40gu.wgsl:114).
E4B_DEV float gelu_tanh(float g) {
  float t = 0.7978845608028654f * (g + 0.044715f * (g * g * g));
  t = fminf(fmaxf(t, -20.0f), 20.0f);
  return (0.5f * g) * (1.0f + tanhf(t));
}

// ---- fragment order ("xfo") of an f16 activation row that feeds a multi-token
// q4_0 GEMM: inside each 32-element block, the 8 values lane t of an
// m16n8k16 B fragment needs (the k order the q4_0 nibble bytes give its A
// fragment) sit contiguously at halves 8t..8t+7, so one 16-byte load fetches
// them.  Lane t's indices j0..j3 (low half; +16 for the high half) are
// 4t..4t+3 in odd blocks, 2+4t..5+4t (t < 3) or {0, 1, 14, 15} (t = 3) in even
// blocks, stored as [j0, j2, j1, j3, j0+16, j2+16, j1+16, j3+16].
E4B_DEV int xfo_pos(int i) {
  const int b = i >> 5, j = i & 31, hi = j >> 4, jj = j & 15;
  int t, r;
  if (b & 1) {
    t = jj >> 2;
    r = jj & 3;
  } else if (jj >= 2 && jj < 14) {
    t = (jj - 2) >> 2;
    r = (jj - 2) & 3;
  } else {
    t = 3;
    r = jj < 2 ? jj : jj - 12;
  }
  const int slot = r == 1 ? 2 : (r == 2 ? 1 : r);
  return (b << 5) + (t << 3) + (hi << 2) + slot;
}

// ---- q4_0: 18-byte block = f16 d, 16 bytes of nibbles (byte j: elem j | elem j+16 << 4)
struct Q40Block {
  float d;
  uint32_t qs[4];
};
// Blocks start on 2-byte boundaries (18 * b), so load them as 9 halfwords.
E4B_DEV Q40Block q40_load(const uint8_t* blk) {
  const unsigned short* p = reinterpret_cast<const unsigned short*>(blk);
  Q40Block b;
  b.d = h2f(__ldg(p));
#pragma unroll
  for (int i = 0; i < 4; i++) b.qs[i] = (uint32_t)__ldg(p + 1 + 2 * i) | ((uint32_t)__ldg(p + 2 + 2 * i) << 16);
  return b;
}
// sum_j (n_j - 8) * x_j for one block; x points at the block's 32 activations.
template <typename XT>
E4B_DEV float q40_dot(const Q40Block& b, const XT* x);
template <>
E4B_DEV float q40_dot<float>(const Q40Block& b, const float* x) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; i++) {
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const uint32_t byte = (b.qs[i] >> (8 * k)) & 0xFFu;
      const int j = 4 * i + k;
      s = fmaf((float)((int)(byte & 15u) - 8), x[j], s);
      s = fmaf((float)((int)(byte >> 4) - 8), x[j + 16], s);
    }
  }
  return s;
}
template <>
E4B_DEV float q40_dot<uint16_t>(const Q40Block& b, const uint16_t* x) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; i++) {
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const uint32_t byte = (b.qs[i] >> (8 * k)) & 0xFFu;
      const int j = 4 * i + k;
      s = fmaf((float)((int)(byte & 15u) - 8), h2f(x[j]), s);
      s = fmaf((float)((int)(byte >> 4) - 8), h2f(x[j + 16]), s);
    }
  }
  return s;
}

// ---- q6_K: 210-byte block = ql[128] qh[64] int8 sc[16] f16 d; element e of the
// block is q = lo | hi << 4 with lo from ql[h*64 + l + 32*(j&1)] nibble (j>>1),
// hi from qh[h*32 + l] bits 2j..2j+1 (h = e/128, j = (e%128)/32, l = e%32), and
// sub-block scale sc[e/16]  (kernels/q6k.wgsl:44-68).
E4B_DEV int q6k_q(const uint8_t* blk, int e) {
  const int h = e >> 7, r = e & 127, j = r >> 5, l = r & 31;
  const int lo = (blk[h * 64 + l + 32 * (j & 1)] >> ((j >> 1) * 4)) & 0xF;
  const int hi = (blk[128 + h * 32 + l] >> (2 * j)) & 3;
  return (lo | (hi << 4)) - 32;
}
E4B_DEV float q6k_d(const uint8_t* blk) {
  return h2f(*reinterpret_cast<const unsigned short*>(blk + 208));
}
E4B_DEV float q6k_elem(const uint8_t* blk, int e) {
  const float ds = q6k_d(blk) * (float)(int8_t)blk[192 + (e >> 4)];  // exact
  return ds * (float)q6k_q(blk, e);                                    // exact
}

// Device status word codes.
enum : uint32_t { E4B_ST_BADINDEX = 1u, E4B_ST_TIMEOUT = 2u };
E4B_DEV void set_status(uint32_t* st, uint32_t code) {
  if (st) atomicOr(st, code);
}
