// Expert parallelism for the batched MoE decode (benchmark config 5): experts
// sharded in contiguous blocks over the ranks of one node, every rank decoding
// its own sequences (attention and dense layers replicated).  Per MoE layer:
//   dispatch   each (token, slot) entry's f16 activation row and local expert
//              id go to the expert's owner, packed per peer in arrival order
//              into fixed-capacity slabs (no host round trip for counts);
//   exchange   grouped ncclSend / ncclRecv with every rank (NVLink / NVSwitch);
//   experts    the owner groups what it received by local expert and runs the
//              grouped GEMMs on those rows;
//   return     each result row goes back into the slab slot it came from, so
//              the source finds entry (t, k) at slot[t*K+k] and combines in
//              slot order exactly as the single-GPU path does.
// The reference's engine-a4b.js has no multi-GPU path; the per-entry math is
// the single-GPU kernels', so results are bit-identical for any rank count.
//
// Two transports move the slabs.  NCCL: grouped send/recv of the whole slabs.
// Peer memory: every rank's receive slabs are mapped into the other ranks'
// address spaces (CUDA IPC), ep_push stores each row straight into its owner's
// slab (same layout: source rank x cap rows) and publishes an epoch flag in
// every peer; ep_wait holds the stream until every peer's flag for this rank
// has reached the same epoch (bounded, status word on time-out).  Epochs count
// the pushes of each direction on every rank, which all ranks issue in the same
// order, so no host value is needed and CUDA-graph replays stay valid.
#include <dlfcn.h>
#include <nccl.h>
#include <stdlib.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "stream.cuh"

namespace {

// NCCL is opened at run time (E4B_NCCL_LIB, else libnccl.so.2) with local
// symbols, so the process can also hold another framework's NCCL build.
struct Nccl {
  bool tried = false;
  void* h = nullptr;
  ncclResult_t (*getUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*commInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*groupStart)() = nullptr;
  ncclResult_t (*groupEnd)() = nullptr;
  ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*allGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*errorString)(ncclResult_t) = nullptr;
};
Nccl g_nccl;

template <class F>
bool sym(void* h, const char* name, F& f) {
  f = reinterpret_cast<F>(dlsym(h, name));
  return f != nullptr;
}
// Under g_mu.
Nccl* nccl() {
  if (!g_nccl.tried) {
    g_nccl.tried = true;
    const char* path = getenv("E4B_NCCL_LIB");
    void* h = dlopen(path && *path ? path : "libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (h && sym(h, "ncclGetUniqueId", g_nccl.getUniqueId) && sym(h, "ncclCommInitRank", g_nccl.commInitRank) &&
        sym(h, "ncclCommDestroy", g_nccl.commDestroy) && sym(h, "ncclGroupStart", g_nccl.groupStart) &&
        sym(h, "ncclGroupEnd", g_nccl.groupEnd) && sym(h, "ncclSend", g_nccl.send) &&
        sym(h, "ncclRecv", g_nccl.recv) && sym(h, "ncclAllGather", g_nccl.allGather) &&
        sym(h, "ncclGetErrorString", g_nccl.errorString))
      g_nccl.h = h;
  }
  return g_nccl.h ? &g_nccl : nullptr;
}

constexpr uint32_t kNone = 0xffffffffu;

struct NcclState {
  ncclComm_t comm = nullptr;
  int nranks = 0, rank = 0;
  cudaStream_t side = nullptr;          // exchanges that overlap the main stream's work
  cudaEvent_t fork = nullptr, done = nullptr;
};
std::mutex g_mu;
std::vector<std::pair<e4b_ctx*, NcclState>> g_comms;

NcclState* state_of(e4b_ctx* c) {
  for (auto& kv : g_comms)
    if (kv.first == c) return &kv.second;
  return nullptr;
}

// One CTA: entry i = t*K + k in order; its destination rank is the owner of
// expert topk[i]; its position among the entries bound there is the number of
// earlier entries with the same destination (stable, deterministic).
__global__ void __launch_bounds__(1024) k_ep_dispatch(const uint32_t* __restrict__ topk, int n, int per_rank,
                                                      int nranks, int cap, const uint16_t* __restrict__ x, int K,
                                                      int H, uint16_t* __restrict__ send_x,
                                                      uint32_t* __restrict__ send_ids, uint32_t* __restrict__ slot,
                                                      uint32_t* status) {
  pdl_wait();
  __shared__ uint32_t base[64];
  __shared__ uint32_t wcnt[32][64];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < nranks * cap; i += 1024) send_ids[i] = kNone;
  if (tid < 64) base[tid] = 0;
  __syncthreads();
  for (int r0 = 0; r0 < n; r0 += 1024) {
    const int i = r0 + tid;
    uint32_t d = kNone;
    if (i < n) {
      const uint32_t e = topk[i];
      d = e / (uint32_t)per_rank;
      if (d >= (uint32_t)nranks) {
        set_status(status, E4B_ST_BADINDEX);
        slot[i] = kNone;
        d = kNone;
      }
    }
    const uint32_t peers = __match_any_sync(0xffffffffu, d);
    const uint32_t rank_in = __popc(peers & ((1u << lane) - 1u));
    for (int k = tid; k < 32 * 64; k += 1024) wcnt[k >> 6][k & 63] = 0;
    __syncthreads();
    if (d != kNone && rank_in == 0) wcnt[warp][d] = __popc(peers);
    __syncthreads();
    if (d != kNone) {
      uint32_t pos = base[d] + rank_in;
      for (int w = 0; w < warp; w++) pos += wcnt[w][d];
      if (pos < (uint32_t)cap) {
        slot[i] = d * cap + pos;
        send_ids[d * cap + pos] = topk[i] - d * (uint32_t)per_rank;
      } else {
        slot[i] = kNone;
        set_status(status, E4B_ST_BADINDEX);    // capacity exceeded
      }
    }
    __syncthreads();
    if (tid < nranks) {
      uint32_t add = 0;
      for (int w = 0; w < 32; w++) add += wcnt[w][tid];
      base[tid] += add;
    }
    __syncthreads();
  }
  // copy the rows: warp per entry, 16-byte pieces (peer-memory transport: ep_push does it)
  if (!send_x) return;
  for (int i = warp; i < n; i += 32) {
    const uint32_t sl = slot[i];
    if (sl == kNone) continue;
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(i / K) * H);
    uint4* dst = reinterpret_cast<uint4*>(send_x + (size_t)sl * H);
    for (int j = lane; j < H / 8; j += 32) dst[j] = src[j];
  }
}

// Vocabulary-sharded LM head: rank r holds the argmax (index within its slice,
// value) of rows [r*Vs, (r+1)*Vs) for every token; token row0 + b takes the best
// over the ranks, ties to the lowest global index (the single-GPU argmax rule).
__global__ void k_argmax_merge(const uint32_t* __restrict__ all, int nranks, int ntok, uint32_t vs, int row0,
                               int nrows, uint32_t* __restrict__ out) {
  pdl_wait();
  for (int b = blockIdx.x * blockDim.x + threadIdx.x; b < nrows; b += gridDim.x * blockDim.x) {
    float bv = -3.0e38f;
    uint32_t bi = kNone;
    for (int r = 0; r < nranks; r++) {
      const uint32_t* e = all + ((size_t)r * ntok + row0 + b) * 2;
      const float v = __uint_as_float(e[1]);
      const uint32_t i = e[0] == kNone ? kNone : (uint32_t)r * vs + e[0];
      if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
      }
    }
    out[2 * b] = bi;
    out[2 * b + 1] = __float_as_uint(bv);
  }
}

// ---- peer-memory transport
E4B_DEV void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
E4B_DEV uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// After this CTA's stores into peer memory: the last CTA of the grid to get
// here publishes epoch = ctr[0] + 1 to flag[rank] of every rank's flag array
// and keeps it in ctr[0] (ctr[1] counts arrivals, zero at rest).
E4B_DEV void publish_epoch(uint32_t* const* flag, int nranks, int rank, uint32_t* ctr) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t done = atomicAdd(ctr + 1, 1u);
    if (done == gridDim.x - 1) {
      __threadfence_system();
      const uint32_t e = __ldcg(ctr) + 1u;
      for (int d = 0; d < nranks; d++) st_release_sys(flag[d] + rank, e);
      ctr[0] = e;
      ctr[1] = 0u;
    }
  }
}

// Rows of the dispatched entries into their owners' receive slabs: entry i with
// slot d*cap + pos -> rx[d] row rank*cap + pos; block 0 also writes this rank's
// id rows send_ids[d*cap, (d+1)*cap) into rid[d] rows rank*cap ... rank*cap + cap.
__global__ void __launch_bounds__(256) k_ep_push(const uint32_t* __restrict__ slot, int n, int K, int H,
                                                 const uint16_t* __restrict__ x, const uint32_t* __restrict__ send_ids,
                                                 int nranks, int rank, int cap, uint16_t* const* rx,
                                                 uint32_t* const* rid, uint32_t* const* flag, uint32_t* ctr) {
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int i = blockIdx.x * nw + warp; i < n; i += gridDim.x * nw) {
    const uint32_t sl = slot[i];
    if (sl == kNone) continue;
    const uint32_t d = sl / (uint32_t)cap, pos = sl % (uint32_t)cap;
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(i / K) * H);
    uint4* dst = reinterpret_cast<uint4*>(rx[d] + ((size_t)rank * cap + pos) * H);
    for (int j = lane; j < H / 8; j += 32) dst[j] = src[j];
  }
  if (blockIdx.x == 0)
    for (int j = threadIdx.x; j < nranks * cap; j += blockDim.x)
      rid[j / cap][(size_t)rank * cap + j % cap] = send_ids[j];
  publish_epoch(flag, nranks, rank, ctr);
}

// Result rows back to their sources: received row i = p*cap + pos (from rank p)
// holding an entry -> ry[p] row rank*cap + pos = y[inv[i]].
__global__ void __launch_bounds__(256) k_ep_push_back(const uint32_t* __restrict__ ids,
                                                      const uint32_t* __restrict__ inv, const float* __restrict__ y,
                                                      int nranks, int rank, int cap, int H, float* const* ry,
                                                      uint32_t* const* flag, uint32_t* ctr) {
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int i = blockIdx.x * nw + warp; i < nranks * cap; i += gridDim.x * nw) {
    if (ids[i] == kNone) continue;
    const int p = i / cap, pos = i % cap;
    const float4* src = reinterpret_cast<const float4*>(y + (size_t)inv[i] * H);
    float4* dst = reinterpret_cast<float4*>(ry[p] + ((size_t)rank * cap + pos) * H);
    for (int j = lane; j < H / 4; j += 32) dst[j] = src[j];
  }
  publish_epoch(flag, nranks, rank, ctr);
}

// One thread per peer: wait until flag[p] has reached this rank's own epoch
// ctr[0] (wrap-safe), giving up after limit_ns (the context's "wait_limit_us",
// default 1 s) with E4B_ST_TIMEOUT.
__global__ void k_ep_wait(const uint32_t* flag, const uint32_t* ctr, int nranks, uint32_t* status, uint64_t limit_ns) {
  pdl_wait();
  const int p = threadIdx.x;
  if (p >= nranks) return;
  const uint32_t e = __ldcg(ctr);
  const uint64_t t0 = e4b::globaltimer_ns();
  for (uint32_t it = 0;; it++) {
    if ((int32_t)(ld_acquire_sys(flag + p) - e) >= 0) return;
    if ((it & 63u) == 63u && e4b::globaltimer_ns() - t0 > limit_ns) {
      set_status(status, E4B_ST_TIMEOUT);
      return;
    }
    __nanosleep(100);
  }
}

// send_y[i] = y[inv[i]] for every received row i that holds an entry.
__global__ void k_ep_return(const uint32_t* __restrict__ ids, const uint32_t* __restrict__ inv,
                            const float* __restrict__ y, int rows, int H, float* __restrict__ send_y) {
  pdl_wait();
  const int i = blockIdx.x;
  if (i >= rows || ids[i] == kNone) return;
  const float4* src = reinterpret_cast<const float4*>(y + (size_t)inv[i] * H);
  float4* dst = reinterpret_cast<float4*>(send_y + (size_t)i * H);
  for (int j = threadIdx.x; j < H / 4; j += blockDim.x) dst[j] = src[j];
}

}  // namespace

namespace e4b {
void nccl_release(e4b_ctx* c) {
  std::lock_guard<std::mutex> lk(g_mu);
  for (size_t i = 0; i < g_comms.size(); i++)
    if (g_comms[i].first == c) {
      NcclState& st = g_comms[i].second;
      if (st.side) cudaStreamSynchronize(st.side);
      if (st.comm && nccl()) nccl()->commDestroy(st.comm);
      if (st.fork) cudaEventDestroy(st.fork);
      if (st.done) cudaEventDestroy(st.done);
      if (st.side) cudaStreamDestroy(st.side);
      g_comms.erase(g_comms.begin() + i);
      return;
    }
}
}  // namespace e4b

extern "C" {

E4B_API int e4b_nccl_unique_id(uint8_t* out) {
  if (!out) return E4B_EINVAL;
  std::lock_guard<std::mutex> lk(g_mu);
  Nccl* n = nccl();
  if (!n) return E4B_ENCCL;
  ncclUniqueId id;
  if (n->getUniqueId(&id) != ncclSuccess) return E4B_ENCCL;
  static_assert(sizeof(id) == 128, "ncclUniqueId is 128 bytes");
  memcpy(out, &id, sizeof(id));
  return E4B_OK;
}

E4B_API int e4b_nccl_init(e4b_ctx* c, int nranks, int rank, const uint8_t* id) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, id && nranks > 0 && nranks <= 64 && rank >= 0 && rank < nranks, "nccl_init: bad args");
  e4b::nccl_release(c);
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  E4B_CUDA(c, cudaSetDevice(c->device));
  Nccl* n;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    n = nccl();
  }
  E4B_REQUIRE(c, n, "nccl_init: cannot open NCCL (%s)", getenv("E4B_NCCL_LIB") ? getenv("E4B_NCCL_LIB") : "libnccl.so.2");
  // collective over the ranks: not under the lock (ranks may share a process)
  ncclComm_t comm;
  ncclResult_t r = n->commInitRank(&comm, nranks, uid, rank);
  E4B_REQUIRE(c, r == ncclSuccess, "ncclCommInitRank: %s", n->errorString(r));
  NcclState st{comm, nranks, rank};
  if (cudaStreamCreateWithFlags(&st.side, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&st.fork, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&st.done, cudaEventDisableTiming) != cudaSuccess) {
    n->commDestroy(comm);
    return e4b_fail(c, E4B_ECUDA, "nccl_init: side stream / events");
  }
  std::lock_guard<std::mutex> lk(g_mu);
  g_comms.push_back({c, st});
  return E4B_OK;
}

E4B_API int e4b_nccl_destroy(e4b_ctx* c) {
  E4B_CHECK_CTX(c);
  e4b::nccl_release(c);
  return E4B_OK;
}

E4B_API int e4b_ep_dispatch(e4b_ctx* c, const uint32_t* topk, int n_tok, int K, int E, int nranks, int cap,
                            const uint16_t* x, int H, uint16_t* send_x, uint32_t* send_ids, uint32_t* slot) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, topk && x && send_ids && slot && n_tok > 0 && K > 0 && cap > 0, "ep_dispatch: bad args");
  E4B_REQUIRE(c, nranks > 0 && nranks <= 64 && E % nranks == 0, "ep_dispatch: E=%d over %d ranks", E, nranks);
  E4B_REQUIRE(c, H % 8 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(send_x) % 16 == 0,
              "ep_dispatch: rows must be 16-byte aligned");
  return e4b_launch(c, "ep_dispatch", k_ep_dispatch, dim3(1), dim3(1024), 0, topk, n_tok * K, E / nranks, nranks, cap,
                    x, K, H, send_x, send_ids, slot, c->status);
}

namespace {
// One NCCL group: every buffer pair (send_i, recv_i, bytes_i per peer) with every rank.
int exchange(e4b_ctx* c, NcclState* st, Nccl* n, cudaStream_t stream, int nbuf, const void* const* send,
             void* const* recv, const size_t* bytes) {
  ncclResult_t r = n->groupStart();
  for (int b = 0; b < nbuf && r == ncclSuccess; b++)
    for (int p = 0; p < st->nranks && r == ncclSuccess; p++) {
      r = n->send(static_cast<const uint8_t*>(send[b]) + p * bytes[b], bytes[b], ncclUint8, p, st->comm, stream);
      if (r == ncclSuccess)
        r = n->recv(static_cast<uint8_t*>(recv[b]) + p * bytes[b], bytes[b], ncclUint8, p, st->comm, stream);
    }
  const ncclResult_t r2 = n->groupEnd();
  E4B_REQUIRE(c, r == ncclSuccess && r2 == ncclSuccess, "ep_exchange: %s",
              n->errorString(r != ncclSuccess ? r : r2));
  return E4B_OK;
}
int comm_of(e4b_ctx* c, NcclState** st, Nccl** n) {
  {
    std::lock_guard<std::mutex> lk(g_mu);
    *st = state_of(c);
    *n = nccl();
  }
  E4B_REQUIRE(c, *st && (*st)->comm && *n, "ep_exchange: no NCCL communicator (e4b_nccl_init)");
  return E4B_OK;
}
}  // namespace

E4B_API int e4b_ep_exchange(e4b_ctx* c, const void* send, void* recv, size_t bytes_per_peer) {
  E4B_CHECK_CTX(c);
  NcclState* st;
  Nccl* n;
  if (int r = comm_of(c, &st, &n)) return r;
  E4B_REQUIRE(c, send && recv && bytes_per_peer > 0, "ep_exchange: bad args");
  return exchange(c, st, n, c->stream, 1, &send, &recv, &bytes_per_peer);
}

E4B_API int e4b_ep_exchange2_async(e4b_ctx* c, const void* send_a, void* recv_a, size_t bytes_a, const void* send_b,
                                   void* recv_b, size_t bytes_b) {
  E4B_CHECK_CTX(c);
  NcclState* st;
  Nccl* n;
  if (int r = comm_of(c, &st, &n)) return r;
  E4B_REQUIRE(c, send_a && recv_a && bytes_a > 0 && send_b && recv_b && bytes_b > 0, "ep_exchange2_async: bad args");
  E4B_CUDA(c, cudaEventRecord(st->fork, c->stream));
  E4B_CUDA(c, cudaStreamWaitEvent(st->side, st->fork, 0));
  const void* send[2] = {send_a, send_b};
  void* recv[2] = {recv_a, recv_b};
  const size_t bytes[2] = {bytes_a, bytes_b};
  if (int r = exchange(c, st, n, st->side, 2, send, recv, bytes)) return r;
  E4B_CUDA(c, cudaEventRecord(st->done, st->side));
  return E4B_OK;
}

E4B_API int e4b_ep_join(e4b_ctx* c) {
  E4B_CHECK_CTX(c);
  NcclState* st;
  Nccl* n;
  if (int r = comm_of(c, &st, &n)) return r;
  E4B_CUDA(c, cudaStreamWaitEvent(c->stream, st->done, 0));
  return E4B_OK;
}

E4B_API int e4b_ep_allgather(e4b_ctx* c, const void* send, void* recv, size_t bytes_per_rank) {
  E4B_CHECK_CTX(c);
  NcclState* st;
  Nccl* n;
  if (int r = comm_of(c, &st, &n)) return r;
  E4B_REQUIRE(c, send && recv && bytes_per_rank > 0, "ep_allgather: bad args");
  const ncclResult_t r = n->allGather(send, recv, bytes_per_rank, ncclUint8, st->comm, c->stream);
  E4B_REQUIRE(c, r == ncclSuccess, "ep_allgather: %s", n->errorString(r));
  return E4B_OK;
}

E4B_API int e4b_argmax_merge(e4b_ctx* c, const uint32_t* all, int nranks, int ntok, int slice, int row0, int nrows,
                             uint32_t* out) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, all && out && nranks > 0 && ntok > 0 && slice > 0 && row0 >= 0 && nrows > 0 && row0 + nrows <= ntok,
              "argmax_merge: bad args");
  return e4b_launch(c, "argmax_merge", k_argmax_merge, dim3((nrows + 255) / 256), dim3(256), 0, all, nranks, ntok,
                    (uint32_t)slice, row0, nrows, out);
}

E4B_API int e4b_ep_return(e4b_ctx* c, const uint32_t* recv_ids, const uint32_t* inv, const float* y, int rows, int H,
                          float* send_y) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, recv_ids && inv && y && send_y && rows > 0 && H % 4 == 0, "ep_return: bad args");
  return e4b_launch(c, "ep_return", k_ep_return, dim3(rows), dim3(256), 0, recv_ids, inv, y, rows, H, send_y);
}

E4B_API int e4b_ipc_handle(e4b_ctx* c, const void* ptr, uint8_t* out64) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, ptr && out64, "ipc_handle: bad args");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "cudaIpcMemHandle_t is 64 bytes");
  cudaIpcMemHandle_t h;
  E4B_CUDA(c, cudaSetDevice(c->device));
  E4B_CUDA(c, cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)));
  memcpy(out64, &h, sizeof(h));
  return E4B_OK;
}

E4B_API int e4b_ipc_open(e4b_ctx* c, const uint8_t* handle64, void** out) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, handle64 && out, "ipc_open: bad args");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  *out = nullptr;
  E4B_CUDA(c, cudaSetDevice(c->device));
  E4B_CUDA(c, cudaIpcOpenMemHandle(out, h, cudaIpcMemLazyEnablePeerAccess));
  return E4B_OK;
}

E4B_API int e4b_ipc_close(e4b_ctx* c, void* ptr) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, ptr, "ipc_close: null pointer");
  E4B_CUDA(c, cudaSetDevice(c->device));
  E4B_CUDA(c, cudaIpcCloseMemHandle(ptr));
  return E4B_OK;
}

E4B_API int e4b_ep_push(e4b_ctx* c, const uint32_t* slot, int n_tok, int K, const uint16_t* x, int H,
                        const uint32_t* send_ids, int nranks, int rank, int cap, const uint64_t* rx_ptrs,
                        const uint64_t* rid_ptrs, const uint64_t* flag_ptrs, uint32_t* ctr) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, slot && x && send_ids && rx_ptrs && rid_ptrs && flag_ptrs && ctr && n_tok > 0 && K > 0 && cap > 0,
              "ep_push: bad args");
  E4B_REQUIRE(c, nranks > 1 && nranks <= 64 && rank >= 0 && rank < nranks, "ep_push: rank %d of %d", rank, nranks);
  E4B_REQUIRE(c, H % 8 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0, "ep_push: rows must be 16-byte aligned");
  const int n = n_tok * K, grid = std::min(std::max((n + 7) / 8, 1), 4 * c->sm_count);
  return e4b_launch(c, "ep_push", k_ep_push, dim3(grid), dim3(256), 0, slot, n, K, H, x, send_ids, nranks, rank, cap,
                    reinterpret_cast<uint16_t* const*>(rx_ptrs), reinterpret_cast<uint32_t* const*>(rid_ptrs),
                    reinterpret_cast<uint32_t* const*>(flag_ptrs), ctr);
}

E4B_API int e4b_ep_push_back(e4b_ctx* c, const uint32_t* recv_ids, const uint32_t* inv, const float* y, int H,
                             int nranks, int rank, int cap, const uint64_t* ry_ptrs, const uint64_t* flag_ptrs,
                             uint32_t* ctr) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, recv_ids && inv && y && ry_ptrs && flag_ptrs && ctr && cap > 0 && H % 4 == 0,
              "ep_push_back: bad args");
  E4B_REQUIRE(c, nranks > 1 && nranks <= 64 && rank >= 0 && rank < nranks, "ep_push_back: rank %d of %d", rank,
              nranks);
  const int rows = nranks * cap, grid = std::min(std::max((rows + 7) / 8, 1), 4 * c->sm_count);
  return e4b_launch(c, "ep_push_back", k_ep_push_back, dim3(grid), dim3(256), 0, recv_ids, inv, y, nranks, rank, cap,
                    H, reinterpret_cast<float* const*>(ry_ptrs), reinterpret_cast<uint32_t* const*>(flag_ptrs), ctr);
}

E4B_API int e4b_ep_wait(e4b_ctx* c, const uint32_t* flag, const uint32_t* ctr, int nranks) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, flag && ctr && nranks > 1 && nranks <= 64, "ep_wait: bad args");
  return e4b_launch(c, "ep_wait", k_ep_wait, dim3(1), dim3(64), 0, flag, ctr, nranks, c->status, c->wait_ns);
}

}  // extern "C"
