// Context, memory, timing, status word and plan (CUDA graph) management.
// Replaces the reference's WebGPU runtime helpers (src/gpu.js:4-50) and its
// per-token plan record/replay (src/engine-a4b.js:800-818).
#include <string.h>

#include "common.cuh"

int e4b_fail(e4b_ctx* c, int code, const char* fmt, ...) {
  if (c) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(c->err, sizeof(c->err), fmt, ap);
    va_end(ap);
  }
  return code;
}

extern "C" {

E4B_API int e4b_create(int device, e4b_ctx** out) {
  if (!out) return E4B_EINVAL;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return E4B_ECUDA;
  e4b_ctx* c = new e4b_ctx();
  c->device = device;
  if (cudaSetDevice(device) != cudaSuccess) { delete c; return E4B_ECUDA; }
  cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, device);
  if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) { delete c; return E4B_ECUDA; }
  for (auto& e : c->ev) cudaEventCreate(&e);
  if (cudaMalloc(&c->status, 256) != cudaSuccess) { delete c; return E4B_ENOMEM; }
  cudaMemset(c->status, 0, 256);
  cudaDeviceSynchronize();
  *out = c;
  return E4B_OK;
}

E4B_API int e4b_destroy(e4b_ctx* c) {
  E4B_CHECK_CTX(c);
  cudaSetDevice(c->device);
  cudaStreamSynchronize(c->stream);
  for (auto& g : c->plans)
    if (g) cudaGraphExecDestroy(g);
  e4b::dense_plans_release(c);
  e4b::nccl_release(c);
  if (c->forked) c->stream = c->main_stream;
  if (c->side) {
    cudaStreamSynchronize(c->side);
    cudaStreamDestroy(c->side);
  }
  if (c->fork_ev) cudaEventDestroy(c->fork_ev);
  if (c->join_ev) cudaEventDestroy(c->join_ev);
  for (auto& e : c->ev) cudaEventDestroy(e);
  cudaFree(c->status);
  cudaStreamDestroy(c->stream);
  delete c;
  return E4B_OK;
}

E4B_API const char* e4b_last_error(const e4b_ctx* c) { return c ? c->err : "null context"; }

E4B_API int e4b_device_info(e4b_ctx* c, int* sm_count, int* cc_major, int* cc_minor, size_t* total_mem) {
  E4B_CHECK_CTX(c);
  cudaDeviceProp p;
  E4B_CUDA(c, cudaGetDeviceProperties(&p, c->device));
  if (sm_count) *sm_count = p.multiProcessorCount;
  if (cc_major) *cc_major = p.major;
  if (cc_minor) *cc_minor = p.minor;
  if (total_mem) *total_mem = p.totalGlobalMem;
  return E4B_OK;
}

E4B_API int e4b_alloc(e4b_ctx* c, size_t bytes, void** out) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, out, "e4b_alloc: null out");
  *out = nullptr;
  cudaError_t e = cudaMalloc(out, bytes ? bytes : 16);
  if (e != cudaSuccess) return e4b_fail(c, E4B_ENOMEM, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
  return E4B_OK;
}
E4B_API int e4b_free(e4b_ctx* c, void* p) {
  E4B_CHECK_CTX(c);
  E4B_CUDA(c, cudaFree(p));
  return E4B_OK;
}
E4B_API int e4b_host_alloc(e4b_ctx* c, size_t bytes, void** out) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, out, "e4b_host_alloc: null out");
  cudaError_t e = cudaMallocHost(out, bytes ? bytes : 16);
  if (e != cudaSuccess) return e4b_fail(c, E4B_ENOMEM, "cudaMallocHost(%zu): %s", bytes, cudaGetErrorString(e));
  return E4B_OK;
}
E4B_API int e4b_host_free(e4b_ctx* c, void* p) {
  E4B_CHECK_CTX(c);
  E4B_CUDA(c, cudaFreeHost(p));
  return E4B_OK;
}
E4B_API int e4b_upload(e4b_ctx* c, void* dst, const void* src, size_t n) {
  E4B_CHECK_CTX(c);
  E4B_CUDA(c, cudaMemcpyAsync(dst, src, n, cudaMemcpyHostToDevice, c->stream));
  E4B_CUDA(c, cudaStreamSynchronize(c->stream));
  return E4B_OK;
}
E4B_API int e4b_download(e4b_ctx* c, void* dst, const void* src, size_t n) {
  E4B_CHECK_CTX(c);
  E4B_CUDA(c, cudaMemcpyAsync(dst, src, n, cudaMemcpyDeviceToHost, c->stream));
  E4B_CUDA(c, cudaStreamSynchronize(c->stream));
  return E4B_OK;
}
E4B_API int e4b_upload_async(e4b_ctx* c, void* dst, const void* src, size_t n) {
  E4B_CHECK_CTX(c);
  E4B_CUDA(c, cudaMemcpyAsync(dst, src, n, cudaMemcpyHostToDevice, c->stream));
  return E4B_OK;
}
E4B_API int e4b_download_async(e4b_ctx* c, void* dst, const void* src, size_t n) {
  E4B_CHECK_CTX(c);
  E4B_CUDA(c, cudaMemcpyAsync(dst, src, n, cudaMemcpyDeviceToHost, c->stream));
  return E4B_OK;
}
E4B_API int e4b_memset(e4b_ctx* c, void* dst, int v, size_t n) {
  E4B_CHECK_CTX(c);
  E4B_CUDA(c, cudaMemsetAsync(dst, v, n, c->stream));
  return E4B_OK;
}
E4B_API int e4b_copy(e4b_ctx* c, void* dst, const void* src, size_t n) {
  E4B_CHECK_CTX(c);
  E4B_CUDA(c, cudaMemcpyAsync(dst, src, n, cudaMemcpyDeviceToDevice, c->stream));
  return E4B_OK;
}
E4B_API int e4b_sync(e4b_ctx* c) {
  E4B_CHECK_CTX(c);
  E4B_CUDA(c, cudaStreamSynchronize(c->stream));
  return E4B_OK;
}
E4B_API int e4b_event_record(e4b_ctx* c, int slot) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, slot >= 0 && slot < 64, "event slot %d out of range", slot);
  E4B_CUDA(c, cudaEventRecord(c->ev[slot], c->stream));
  return E4B_OK;
}
E4B_API int e4b_event_elapsed(e4b_ctx* c, int a, int b, float* ms) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, a >= 0 && a < 64 && b >= 0 && b < 64 && ms, "bad event args");
  E4B_CUDA(c, cudaEventSynchronize(c->ev[b]));
  E4B_CUDA(c, cudaEventElapsedTime(ms, c->ev[a], c->ev[b]));
  return E4B_OK;
}
E4B_API int e4b_set_pdl(e4b_ctx* c, int enable) {
  E4B_CHECK_CTX(c);
  c->pdl = enable != 0;
  return E4B_OK;
}
E4B_API size_t e4b_workspace_bytes(void) { return (size_t)96 << 20; }
E4B_API int e4b_set_option(e4b_ctx* c, const char* name, int value) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, name, "null option name");
  if (!strcmp(name, "stream_ctas_per_sm")) {
    E4B_REQUIRE(c, value >= 1 && value <= 2, "stream_ctas_per_sm must be 1 or 2");
    c->stream_ctas_per_sm = value;
  } else if (!strcmp(name, "stream_variant")) {
    E4B_REQUIRE(c, value >= 0 && value <= 2, "stream_variant must be 0..2");
    c->stream_variant = value;
  } else if (!strcmp(name, "stream_stages")) {
    E4B_REQUIRE(c, value >= 2 && value <= 4, "stream_stages must be 2..4");
    c->stream_stages = value;
  } else if (!strcmp(name, "attn_grid_cap")) {
    E4B_REQUIRE(c, value >= 0, "attn_grid_cap must be >= 0 (0 = one CTA per SM)");
    c->attn_grid_cap = value;
  } else if (!strcmp(name, "lmhead_tiles_tc")) {
    E4B_REQUIRE(c, value >= 0 && value <= 2, "lmhead_tiles_tc must be 0, 1 or 2");
    c->lmhead_tiles_tc = value;
  } else if (!strcmp(name, "lmhead_tc_min")) {
    E4B_REQUIRE(c, value >= 1 && value <= 65, "lmhead_tc_min must be 1..65 (65 = never)");
    c->lmhead_tc_min = value;
  } else if (!strcmp(name, "wait_limit_us")) {
    E4B_REQUIRE(c, value >= 1000 && value <= 10000000, "wait_limit_us must be 1000..10000000");
    c->wait_ns = (uint64_t)value * 1000ull;
  } else {
    return e4b_fail(c, E4B_EINVAL, "unknown option %s", name);
  }
  return E4B_OK;
}
E4B_API int e4b_set_workspace(e4b_ctx* c, void* ws, size_t bytes) {
  E4B_CHECK_CTX(c);
  if (!ws && bytes == 0) {
    c->ws = nullptr;
    c->ws_bytes = 0;
    return E4B_OK;
  }
  E4B_REQUIRE(c, ws && bytes >= (size_t)(1 << 20), "workspace must be at least 1 MiB");
  E4B_CUDA(c, cudaMemsetAsync(ws, 0, bytes, c->stream));
  E4B_CUDA(c, cudaStreamSynchronize(c->stream));
  c->ws = ws;
  c->ws_bytes = bytes;
  return E4B_OK;
}
E4B_API int e4b_device_status(e4b_ctx* c, uint32_t* st) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, st, "null status out");
  E4B_CUDA(c, cudaMemcpyAsync(st, c->status, 4, cudaMemcpyDeviceToHost, c->stream));
  E4B_CUDA(c, cudaMemsetAsync(c->status, 0, 4, c->stream));
  E4B_CUDA(c, cudaStreamSynchronize(c->stream));
  return E4B_OK;
}

E4B_API int e4b_side_begin(e4b_ctx* c) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, !c->forked && !c->side_pending, "side_begin: side work already open or not joined");
  if (!c->side) {
    E4B_CUDA(c, cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking));
    E4B_CUDA(c, cudaEventCreateWithFlags(&c->fork_ev, cudaEventDisableTiming));
    E4B_CUDA(c, cudaEventCreateWithFlags(&c->join_ev, cudaEventDisableTiming));
  }
  E4B_CUDA(c, cudaEventRecord(c->fork_ev, c->stream));
  E4B_CUDA(c, cudaStreamWaitEvent(c->side, c->fork_ev, 0));
  c->main_stream = c->stream;
  c->stream = c->side;
  c->forked = true;
  return E4B_OK;
}
E4B_API int e4b_side_end(e4b_ctx* c) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, c->forked, "side_end without side_begin");
  E4B_CUDA(c, cudaEventRecord(c->join_ev, c->side));
  c->stream = c->main_stream;
  c->forked = false;
  c->side_pending = true;
  return E4B_OK;
}
E4B_API int e4b_join(e4b_ctx* c) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, !c->forked && c->side_pending, "join without side_begin / side_end");
  E4B_CUDA(c, cudaStreamWaitEvent(c->stream, c->join_ev, 0));
  c->side_pending = false;
  return E4B_OK;
}

E4B_API int e4b_plan_begin(e4b_ctx* c) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, !c->capturing, "plan already being recorded");
  E4B_REQUIRE(c, !c->forked && !c->side_pending, "plan_begin with side work open");
  E4B_CUDA(c, cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
  c->capturing = true;
  return E4B_OK;
}
E4B_API int e4b_plan_end(e4b_ctx* c, int* plan) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, c->capturing && plan, "no plan being recorded");
  E4B_REQUIRE(c, !c->forked && !c->side_pending, "plan_end before e4b_join");
  c->capturing = false;
  cudaGraph_t g = nullptr;
  E4B_CUDA(c, cudaStreamEndCapture(c->stream, &g));
  cudaGraphExec_t ex = nullptr;
  cudaError_t e = cudaGraphInstantiate(&ex, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return e4b_fail(c, E4B_ECUDA, "cudaGraphInstantiate: %s", cudaGetErrorString(e));
  c->plans.push_back(ex);
  *plan = (int)c->plans.size() - 1;
  return E4B_OK;
}
E4B_API int e4b_plan_launch(e4b_ctx* c, int plan, int count) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, plan >= 0 && plan < (int)c->plans.size() && c->plans[plan], "bad plan %d", plan);
  for (int i = 0; i < count; i++) E4B_CUDA(c, cudaGraphLaunch(c->plans[plan], c->stream));
  return E4B_OK;
}
E4B_API int e4b_plan_destroy(e4b_ctx* c, int plan) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, plan >= 0 && plan < (int)c->plans.size() && c->plans[plan], "bad plan %d", plan);
  E4B_CUDA(c, cudaGraphExecDestroy(c->plans[plan]));
  c->plans[plan] = nullptr;
  return E4B_OK;
}

}  // extern "C"

// ------------------------------------------------------------------ dequant
__global__ void k_dequant_q40(const uint8_t* __restrict__ w, float* __restrict__ out, int64_t nblocks) {
  pdl_wait();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nblocks * 32) return;
  const int64_t b = i >> 5;
  const int e = (int)(i & 31);
  const uint8_t* blk = w + b * 18;
  const float d = h2f(*reinterpret_cast<const unsigned short*>(blk));
  const int byte = blk[2 + (e & 15)];
  const int n = e < 16 ? (byte & 15) : (byte >> 4);
  out[i] = d * (float)(n - 8);
}
__global__ void k_dequant_q6k(const uint8_t* __restrict__ w, float* __restrict__ out, int64_t nblocks) {
  pdl_wait();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nblocks * 256) return;
  out[i] = q6k_elem(w + (i >> 8) * 210, (int)(i & 255));
}

extern "C" {
E4B_API int e4b_dequant_q40(e4b_ctx* c, const uint8_t* w, float* out, int64_t nblocks) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, w && out && nblocks >= 0, "dequant_q40: bad args");
  const int64_t n = nblocks * 32;
  return e4b_launch(c, "dequant_q40", k_dequant_q40, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, w, out,
                    nblocks);
}
E4B_API int e4b_dequant_q6k(e4b_ctx* c, const uint8_t* w, float* out, int64_t nblocks) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, w && out && nblocks >= 0, "dequant_q6k: bad args");
  const int64_t n = nblocks * 256;
  return e4b_launch(c, "dequant_q6k", k_dequant_q6k, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, w, out,
                    nblocks);
}
}
