// Grouped MoE and multi-token q4_0 GEMMs for batched decode (kernels/expgroup.wgsl,
// q40gugrp.wgsl, q40downgrp.wgsl, wacc.wgsl): the B x K (token, slot) routing
// entries are sorted by expert, each expert's weights are streamed once for all
// the tokens routed to it, and the per-entry outputs are combined per token in
// slot order.  The dense batched GEMMs of the same step (q|k|v, o, shared FFN)
// run through the same kernel with one matrix and the batch's tokens.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "q40_frag.cuh"
#include "q40_stream.cuh"

namespace {
using namespace e4b;


// ---- routing entries sorted by expert (stable: increasing token * K + slot)
__global__ void k_expgroup(const uint32_t* __restrict__ topk, int n, int E, uint32_t* __restrict__ offsets,
                           uint32_t* __restrict__ entries, uint32_t* __restrict__ inv, uint32_t* status) {
  pdl_wait();
  extern __shared__ uint32_t cnt[];   // [E + 1]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int e = warp; e < E; e += nw) {
    uint32_t c = 0;
    for (int i0 = 0; i0 < n; i0 += 32) {
      const int i = i0 + lane;
      c += __popc(__ballot_sync(0xffffffffu, i < n && topk[i] == (uint32_t)e));
    }
    if (lane == 0) cnt[e] = c;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t s = 0;
    for (int e = 0; e < E; e++) {
      const uint32_t c = cnt[e];
      cnt[e] = s;
      offsets[e] = s;
      s += c;
    }
    offsets[E] = s;
    cnt[E] = s;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x)   // expert id out of range (0xffffffff: an empty slot)
    if (topk[i] >= (uint32_t)E && topk[i] != 0xffffffffu) set_status(status, E4B_ST_BADINDEX);
  for (int e = warp; e < E; e += nw) {
    uint32_t base = cnt[e];
    for (int i0 = 0; i0 < n; i0 += 32) {
      const int i = i0 + lane;
      const bool mine = i < n && topk[i] == (uint32_t)e;
      const uint32_t m = __ballot_sync(0xffffffffu, mine);
      if (mine) {
        const uint32_t pos = base + __popc(m & ((1u << lane) - 1u));
        entries[pos] = (uint32_t)i;
        inv[i] = pos;
      }
      base += __popc(m);
    }
  }
}

// Stable counting sort for small E (<= kSortE): one entry per thread per round
// of 1024; equal experts inside a warp found with match.any, warps ordered by a
// per-round count table, rounds in order -> positions ascend with the entry
// index inside every expert, exactly as the ballot version above.
constexpr int kSortE = 256;
__global__ void __launch_bounds__(1024) k_expsort(const uint32_t* __restrict__ topk, int n, int E,
                                                  uint32_t* __restrict__ offsets, uint32_t* __restrict__ entries,
                                                  uint32_t* __restrict__ inv, uint32_t* status) {
  pdl_wait();
  __shared__ uint32_t base[kSortE + 1];
  __shared__ uint16_t wcnt[32][kSortE];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int e = tid; e <= E; e += 1024) base[e] = 0;
  __syncthreads();
  bool bad = false;
  for (int i = tid; i < n; i += 1024) {
    const uint32_t e = topk[i];
    if (e < (uint32_t)E) atomicAdd(&base[e], 1u);
    else if (e != 0xffffffffu) bad = true;        // 0xffffffff: an empty slot, skipped
  }
  if (bad) set_status(status, E4B_ST_BADINDEX);
  __syncthreads();
  if (warp == 0) {      // exclusive scan of the counts -> offsets and running bases
    uint32_t run = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      const uint32_t c = e < E ? base[e] : 0u;
      uint32_t inc = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += v;
      }
      if (e < E) {
        base[e] = run + inc - c;
        offsets[e] = run + inc - c;
      }
      run += __shfl_sync(0xffffffffu, inc, 31);
    }
    if (lane == 0) offsets[E] = run;
  }
  __syncthreads();
  for (int r0 = 0; r0 < n; r0 += 1024) {
    const int i = r0 + tid;
    const uint32_t e = i < n ? topk[i] : 0xffffffffu;
    const bool live = e < (uint32_t)E;
    const uint32_t peers = __match_any_sync(0xffffffffu, e);
    const uint32_t rank = __popc(peers & ((1u << lane) - 1u));
    for (int k = tid; k < 32 * E; k += 1024) wcnt[k / E][k % E] = 0;
    __syncthreads();
    if (live && rank == 0) wcnt[warp][e] = (uint16_t)__popc(peers);
    __syncthreads();
    if (live) {
      uint32_t pos = base[e] + rank;
      for (int w = 0; w < warp; w++) pos += wcnt[w][e];
      entries[pos] = (uint32_t)i;
      inv[i] = pos;
    }
    __syncthreads();
    for (int e2 = tid; e2 < E; e2 += 1024) {
      uint32_t add = 0;
      for (int w = 0; w < 32; w++) add += wcnt[w][e2];
      base[e2] += add;
    }
    __syncthreads();
  }
}

// ---- multi-token q4_0 GEMM (grouped experts or one dense matrix).
//
// Work: a chunk is up to TOKC (8 or 16) tokens of one matrix (an expert's sorted
// entries, or consecutive tokens of the dense batch); an item is a chunk x W
// consecutive row tiles, one tile per warp.  Every CTA of a persistent grid owns
// a contiguous range of items (chunk-major, so consecutive items share their
// activations).  Per chunk the CTA stages the tokens' activation rows, already
// in fragment order, into shared memory once (one bulk copy per token); each
// warp streams its tile's weights through its own mbarrier ring:
//   MODE 0: 2-D TMA boxes of 16 rows x 8 blocks (144 B per row, conflict-free
//           nibble reads); a quantum is two boxes (32 rows x 8 blocks).  Needs
//           16-byte row strides (IN % 256 == 0).
//   MODE 1: one 1-D bulk copy of 16 whole rows (any IN with 4-byte rows); a
//           tile is 16 rows and one quantum holds all of K.
// Math: per q4_0 block and 16-row subtile, two m16n8k16 MMAs (A = nibbles - 8,
// exact in f16; B = 8 tokens' activations) give sum (n-8) x for the block; its
// f16 scale multiplies that in f32 (the single-token kernels' arithmetic).
// Epilogues: EPI 0 y[pos][row] (f32); EPI 1 tiles pair 16 gate rows with the
// matching 16 up rows and write yh[pos][o] = f16(gelu(gate) * up) in fragment
// order, ready to be the next GEMM's activations.
constexpr int kMaxChunks = 512;  // chunk list capacity (shared memory)

struct Chunk {
  uint32_t e, p0, n;             // matrix, first position (sorted entry or token), tokens
};

struct QmmP {
  const uint16_t* x;             // activation rows in fragment order, IN wide
  const uint8_t* w;              // weights (MODE 1 addressing)
  const uint32_t* offsets;       // [E+1] sorted-entry offsets; null: dense over n_dense tokens
  const uint32_t* entries;       // non-null: x row of position p = entries[p] / K; null: x row = p
  float* y;
  uint16_t* yh;
  uint32_t* status;
  int IN, nb, rowbytes, ROWS, FF, K, E, n_dense;
  int tiles;                     // tiles per matrix
  int nq;                        // quanta per tile
  int RR;                        // items per chunk = ceil(tiles / W)
  int xpitch;                    // staged activation row pitch (halves)
};

E4B_DEV uint4 lds128(const uint16_t* p) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(smem_u32(p)));
  return v;
}

// ---- tile-packed q4_0 (IN % 256 == 0): per 16-row group and 256-k quantum one
// 2304-byte piece, [16 rows][8 blocks] f16 scales (256 B) then the nibble words
// as [k half][row][lane t] uint4 (2048 B): word j of (h, r, t) is the 32-bit
// A-operand source lane t of row r uses for block 4h + j (nib_odd / nib_even of
// the GGUF block).  A warp reads a row's 8 scales and 4 blocks' nibble words
// with one 16-byte load each, conflict-free; the decoded A registers equal the
// row-major path's, so results are bit-identical.
E4B_DEV uint4 lds128b(const uint8_t* p) { return lds128(reinterpret_cast<const uint16_t*>(p)); }
E4B_DEV float half_of(const uint4& v, int k) {
  const uint32_t w = u32w(v, k >> 1);
  const __half2 h = *reinterpret_cast<const __half2*>(&w);     // the conversion reads either half in place
  return (k & 1) ? __high2float(h) : __low2float(h);
}
// One quantum of the gate|up tile from a packed stage (two 16-row pieces).
template <int TWO>
E4B_DEV void qmm_quantum_pk(const uint8_t* st, int g, int t, const uint16_t* xq, int xstep, bool two,
                            float (&acc)[2][2][4]) {
  uint4 S[2][2];
#pragma unroll
  for (int sb = 0; sb < 2; sb++) {
    S[sb][0] = lds128b(st + sb * kPkSub + 16 * g);
    S[sb][1] = lds128b(st + sb * kPkSub + 16 * (g + 8));
  }
#pragma unroll
  for (int kh = 0; kh < 2; kh++) {
    uint4 N[2][2];
#pragma unroll
    for (int sb = 0; sb < 2; sb++)
#pragma unroll
      for (int h = 0; h < 2; h++) N[sb][h] = lds128b(st + sb * kPkSub + 256 + ((kh * 16 + g + 8 * h) * 4 + t) * 16);
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int k = 4 * kh + j;
      uint32_t A[2][8];
      float d[2][2];
#pragma unroll
      for (int sb = 0; sb < 2; sb++) {
        dq_row(u32w(N[sb][0], j), A[sb][0], A[sb][1], A[sb][2], A[sb][3]);
        dq_row(u32w(N[sb][1], j), A[sb][4], A[sb][5], A[sb][6], A[sb][7]);
        d[sb][0] = half_of(S[sb][0], k);
        d[sb][1] = half_of(S[sb][1], k);
      }
#pragma unroll
      for (int q = 0; q < (TWO ? 2 : 1); q++) {
        if (q == 1 && !two) break;
        const uint4 xb = lds128(xq + 32 * k + q * xstep);
#pragma unroll
        for (int sb = 0; sb < 2; sb++) {
          float c[4] = {0.f, 0.f, 0.f, 0.f};
          mma16816(c, A[sb][0], A[sb][4], A[sb][1], A[sb][5], xb.x, xb.y);
          mma16816(c, A[sb][2], A[sb][6], A[sb][3], A[sb][7], xb.z, xb.w);
          acc[q][sb][0] = fmaf(d[sb][0], c[0], acc[q][sb][0]);
          acc[q][sb][1] = fmaf(d[sb][0], c[1], acc[q][sb][1]);
          acc[q][sb][2] = fmaf(d[sb][1], c[2], acc[q][sb][2]);
          acc[q][sb][3] = fmaf(d[sb][1], c[3], acc[q][sb][3]);
        }
      }
    }
  }
}

// Pack rows x IN q4_0 (GGUF blocks) into the tile-packed layout: one CTA of
// 128 threads per (16-row group, quantum); thread (h, r, t) writes one uint4.
__global__ void k_q40_pack(const uint8_t* __restrict__ w, uint8_t* __restrict__ wt, int IN) {
  pdl_wait();
  const int nq = IN / 256, rowbytes = IN / 32 * 18;
  const int r16 = blockIdx.y, kq = blockIdx.x;
  uint8_t* out = wt + ((size_t)r16 * nq + kq) * kPkSub;
  const int i = threadIdx.x, kh = i >> 6, r = (i >> 2) & 15, t = i & 3;
  const uint8_t* row = w + (size_t)(16 * r16 + r) * rowbytes;
  uint32_t wd[4];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const int b = 8 * kq + 4 * kh + j;
    const uint8_t* blk = row + 18 * b;
    uint32_t v;
    if (b & 1) {
      v = blk[2 + 4 * t] | (uint32_t)blk[3 + 4 * t] << 8 | (uint32_t)blk[4 + 4 * t] << 16 | (uint32_t)blk[5 + 4 * t] << 24;
    } else if (t < 3) {
      v = blk[4 + 4 * t] | (uint32_t)blk[5 + 4 * t] << 8 | (uint32_t)blk[6 + 4 * t] << 16 | (uint32_t)blk[7 + 4 * t] << 24;
    } else {
      v = blk[2] | (uint32_t)blk[3] << 8 | (uint32_t)blk[16] << 16 | (uint32_t)blk[17] << 24;
    }
    wd[j] = v;
  }
  *reinterpret_cast<uint4*>(out + 256 + 16 * i) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
  if (i < 16) {
    const uint8_t* ri = w + (size_t)(16 * r16 + i) * rowbytes + (size_t)18 * 8 * kq;
    uint32_t sc[4];
#pragma unroll
    for (int k = 0; k < 4; k++)
      sc[k] = ri[36 * k] | (uint32_t)ri[36 * k + 1] << 8 | (uint32_t)ri[36 * k + 18] << 16 |
              (uint32_t)ri[36 * k + 19] << 24;
    *reinterpret_cast<uint4*>(out + 16 * i) = make_uint4(sc[0], sc[1], sc[2], sc[3]);
  }
}

// Chunk list of this launch (warp 0; dense: arithmetic, grouped: a warp scan of
// the experts' entry counts).  Returns the number of chunks.
template <int kTokC>
E4B_DEV int build_chunks(const QmmP& p, Chunk* ch, int lane) {
  if (!p.offsets) {
    const int n = (p.n_dense + kTokC - 1) / kTokC;
    for (int c = lane; c < n && c < kMaxChunks; c += 32)
      ch[c] = Chunk{0u, (uint32_t)(kTokC * c), (uint32_t)min(kTokC, p.n_dense - kTokC * c)};
    return min(n, kMaxChunks);
  }
  int base = 0;
  for (int e0 = 0; e0 < p.E; e0 += 32) {
    const int e = e0 + lane;
    const uint32_t a = e < p.E ? p.offsets[e] : 0u, b = e < p.E ? p.offsets[e + 1] : 0u;
    const int n = (int)(b - a), c = (n + kTokC - 1) / kTokC;
    int inc = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += v;
    }
    const int ex = base + inc - c;
    for (int j = 0; j < c; j++)
      if (ex + j < kMaxChunks) ch[ex + j] = Chunk{(uint32_t)e, a + (uint32_t)(kTokC * j), (uint32_t)min(kTokC, n - kTokC * j)};
    base += __shfl_sync(0xffffffffu, inc, 31);
  }
  if (base > kMaxChunks) {
    if (lane == 0) set_status(p.status, E4B_ST_BADINDEX);
    base = kMaxChunks;
  }
  return base;
}

// One block (32 k) of NS 16-row subtiles: a/b point at rows g and g+8 of
// subtile 0 (subtile 1 sub_bytes further), xq at this lane's fragment of the
// block for token group 0 (group 1 xstep halves further).
template <int NS, int TWO, int PAR>
E4B_DEV void qmm_block(const uint8_t* a, const uint8_t* b, int sub_bytes, const uint16_t* xq, int xstep, bool two,
                       const Lane& L, float (&acc)[2][2][4]) {
  uint32_t A[NS][8];
  float d[NS][2];
#pragma unroll
  for (int s = 0; s < NS; s++) {
    const uint8_t* ra = a + s * sub_bytes;
    const uint8_t* rb = b + s * sub_bytes;
    dq_row(PAR ? nib_odd(ra, L) : nib_even(ra, L), A[s][0], A[s][1], A[s][2], A[s][3]);
    dq_row(PAR ? nib_odd(rb, L) : nib_even(rb, L), A[s][4], A[s][5], A[s][6], A[s][7]);
    d[s][0] = h2f(*reinterpret_cast<const uint16_t*>(ra));
    d[s][1] = h2f(*reinterpret_cast<const uint16_t*>(rb));
  }
#pragma unroll
  for (int q = 0; q < (TWO ? 2 : 1); q++) {
    if (q == 1 && !two) break;
    const uint4 xb = lds128(xq + q * xstep);
#pragma unroll
    for (int s = 0; s < NS; s++) {
      float c[4] = {0.f, 0.f, 0.f, 0.f};
      mma16816(c, A[s][0], A[s][4], A[s][1], A[s][5], xb.x, xb.y);
      mma16816(c, A[s][2], A[s][6], A[s][3], A[s][7], xb.z, xb.w);
      acc[q][s][0] = fmaf(d[s][0], c[0], acc[q][s][0]);
      acc[q][s][1] = fmaf(d[s][0], c[1], acc[q][s][1]);
      acc[q][s][2] = fmaf(d[s][1], c[2], acc[q][s][2]);
      acc[q][s][3] = fmaf(d[s][1], c[3], acc[q][s][3]);
    }
  }
}

// KS > 1 (dense batches): the KS warps of a tile group split its quanta and sum
// their partials through shared memory in a fixed order (deterministic), so a
// small matrix still spreads over every SM.
template <int MODE, int EPI, int W, int S, int TOKC, int KS, int PK = 0>
__global__ void __launch_bounds__(32 * W, 1) k_qmm(const QmmP p, const __grid_constant__ CUtensorMap map) {
  constexpr int NS = MODE == 0 ? 2 : 1;
  constexpr int TPI = W / KS;            // tiles per item
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[W][S];
  __shared__ __align__(8) uint64_t xbar;
  __shared__ Chunk chunks[kMaxChunks];
  __shared__ int s_nch;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const uint32_t stage_bytes = MODE == 0 ? (uint32_t)kQuantumBytes : 16u * (uint32_t)p.rowbytes;
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem);
  uint8_t* stages = smem + (size_t)TOKC * p.xpitch * 2 + (size_t)warp * S * stage_bytes;
  float* red = reinterpret_cast<float*>(smem + (size_t)TOKC * p.xpitch * 2 + (size_t)W * S * stage_bytes);
  // this warp's tile slot and quantum range
  const int wt = warp / KS, kp = warp % KS;
  const int kq0 = p.nq * kp / KS, kq1 = p.nq * (kp + 1) / KS;

  pdl_trigger();
  if (lane == 0) {
    if (MODE == 0) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map)) : "memory");
    for (int s = 0; s < S; s++) mbar_init(&full[warp][s], 1);
    if (warp == 0) mbar_init(&xbar, 1);
    fence_barrier_init();
  }
  // a dense batch's chunk list needs no device data: its first weight quanta
  // are requested before the wait on the previous kernel
  if (p.offsets) pdl_wait();
  if (warp == 0) {
    const int n = build_chunks<TOKC>(p, chunks, lane);
    if (lane == 0) s_nch = n;
  }
  __syncthreads();
  const int T = s_nch * p.RR;
  const int i0 = (int)((int64_t)T * blockIdx.x / gridDim.x);
  const int i1 = (int)((int64_t)T * (blockIdx.x + 1) / gridDim.x);

  // producer cursor over (item, quantum) of this warp's tiles; every lane keeps
  // it.  Item it = chunk pci, tile slot prr (it = pci * RR + prr), advanced
  // incrementally (no division per quantum).
  int pit = i0, pkq = kq0, pci = i0 / p.RR, prr = i0 - pci * p.RR;
  auto has_slot = [&](int rr) { return rr * TPI + wt < p.tiles && kq0 < kq1; };
  auto next_item = [&]() {
    pit++;
    if (++prr == p.RR) {
      prr = 0;
      pci++;
    }
  };
  while (pit < i1 && !has_slot(prr)) next_item();
  auto issue = [&](int s) {
    const Chunk c = chunks[pci];
    const int tile = prr * TPI + wt;
    uint8_t* st = stages + s * stage_bytes;
    if (MODE == 0 && PK) {
      // two 16-row pieces of the packed copy (rows of expert c.e)
      if (lane == 0) {
        const size_t r0 = ((size_t)c.e * p.ROWS + (EPI == 1 ? 16 * tile : 32 * tile)) / 16;
        const size_t r1 = ((size_t)c.e * p.ROWS + (EPI == 1 ? p.FF + 16 * tile : 32 * tile + 16)) / 16;
        mbar_expect_tx(&full[warp][s], 2u * kPkSub);
        bulk_g2s(st, p.w + (r0 * p.nq + pkq) * kPkSub, kPkSub, &full[warp][s]);
        bulk_g2s(st + kPkSub, p.w + (r1 * p.nq + pkq) * kPkSub, kPkSub, &full[warp][s]);
      }
    } else if (MODE == 0) {
      if (lane == 0) mbar_expect_tx(&full[warp][s], (uint32_t)kQuantumBytes);
      __syncwarp();
      if (lane < 2) {
        const int row = (int)c.e * p.ROWS + (EPI == 1 ? (lane == 0 ? 16 * tile : p.FF + 16 * tile) : 32 * tile + 16 * lane);
        tma_load_2d(st + lane * kSubBytes, &map, pkq * 18, row, &full[warp][s]);
      }
    } else if (lane == 0) {
      mbar_expect_tx(&full[warp][s], stage_bytes);
      bulk_g2s(st, p.w + ((size_t)c.e * p.ROWS + 16 * (size_t)tile) * p.rowbytes, stage_bytes, &full[warp][s]);
    }
    if (++pkq == kq1) {
      pkq = kq0;
      do next_item(); while (pit < i1 && !has_slot(prr));
    }
  };
#pragma unroll
  for (int s = 0; s < S; s++)
    if (pit < i1) issue(s);
  if (!p.offsets) pdl_wait();        // before the activations (produced by the previous kernel) are read

  Lane L;
  L.o_odd = 2 + 4 * t;
  L.o_e1 = t < 3 ? 4 + 4 * t : 0;
  L.sel = t < 3 ? 0x3210u : 0x5432u;
  bool ok = true;
  int cur = -1, restage = 0, used = 0;
  int ci = i0 / p.RR, rr = i0 - ci * p.RR;          // item it = ci * RR + rr
  for (int it = i0; it < i1; it++, rr = rr + 1 == p.RR ? 0 : rr + 1, ci = rr == 0 ? ci + 1 : ci) {
    const Chunk c = chunks[ci];
    if (ci != cur) {
      // every warp is done with the previous chunk's activations
      __syncthreads();
      if (warp == 0) {
        if (lane == 0) mbar_expect_tx(&xbar, c.n * (uint32_t)p.IN * 2u);
        __syncwarp();
        if (lane < (int)c.n) {
          const uint32_t pos = c.p0 + lane;
          const uint32_t row = !p.offsets ? pos : (p.entries ? p.entries[pos] / (uint32_t)p.K : pos);
          bulk_g2s(xs + (size_t)lane * p.xpitch, p.x + (size_t)row * p.IN, (uint32_t)p.IN * 2u, &xbar);
        }
      }
      if (ok) ok = mbar_wait(&xbar, (uint32_t)(restage & 1), p.status);
      restage++;
      cur = ci;
    }
    const bool mine = has_slot(rr);
    if (KS == 1 && !mine) continue;
    const int tile = rr * TPI + wt;
    const bool two = TOKC > 8 && c.n > 8;
    const uint16_t* xr0 = xs + (size_t)g * p.xpitch + 8 * t;
    float acc[2][2][4];
#pragma unroll
    for (int q = 0; q < 2; q++)
#pragma unroll
      for (int s = 0; s < 2; s++)
#pragma unroll
        for (int r = 0; r < 4; r++) acc[q][s][r] = 0.f;
    for (int kq = kq0; kq < (mine ? kq1 : kq0); kq++, used++) {
      const int s = used % S;
      if (ok) ok = mbar_wait(&full[warp][s], (uint32_t)((used / S) & 1), p.status);
      if (ok) {
        constexpr int TWO = TOKC > 8;
        const int xstep = 8 * p.xpitch;
        if (MODE == 0 && PK) {
          qmm_quantum_pk<TWO>(stages + s * stage_bytes, g, t, xr0 + 256 * kq, xstep, two, acc);
        } else if (MODE == 0) {
          // IN % 256 == 0: always 8 whole blocks, fully unrolled (immediate offsets)
          const uint8_t* a = stages + s * stage_bytes + g * kRowPitch;
          const uint16_t* xq = xr0 + 256 * kq;
#pragma unroll
          for (int k = 0; k < 8; k += 2) {
            qmm_block<NS, TWO, 0>(a + 18 * k, a + 8 * kRowPitch + 18 * k, kSubBytes, xq + 32 * k, xstep, two, L, acc);
            qmm_block<NS, TWO, 1>(a + 18 * k + 18, a + 8 * kRowPitch + 18 * k + 18, kSubBytes, xq + 32 * k + 32,
                                  xstep, two, L, acc);
          }
        } else {
          const uint8_t* a = stages + s * stage_bytes + (size_t)g * p.rowbytes;
          const uint8_t* b = a + 8 * (size_t)p.rowbytes;
          const uint16_t* xq = xr0;
#pragma unroll 2
          for (int k = 0; k < p.nb; k += 2) {
            qmm_block<NS, TWO, 0>(a, b, 0, xq, xstep, two, L, acc);
            qmm_block<NS, TWO, 1>(a + 18, b + 18, 0, xq + 32, xstep, two, L, acc);
            a += 36;
            b += 36;
            xq += 64;
          }
        }
      }
      // this lane's reads of the stage fed the MMAs above; refill it
      __syncwarp();
      if (ok && pit < i1) issue(s);
    }
    if (KS > 1) {
      // partials of the KS warps of each tile, summed in k order by its first warp
      float* mine_red = red + ((size_t)warp * 32 + lane) * 16;
#pragma unroll
      for (int q = 0; q < 2; q++)
#pragma unroll
        for (int s2 = 0; s2 < 2; s2++)
#pragma unroll
          for (int r = 0; r < 4; r++) mine_red[q * 8 + s2 * 4 + r] = acc[q][s2][r];
      __syncthreads();
      if (kp == 0 && mine) {
#pragma unroll
        for (int q = 0; q < 2; q++)
#pragma unroll
          for (int s2 = 0; s2 < 2; s2++)
#pragma unroll
            for (int r = 0; r < 4; r++) {
              float v = 0.f;
              for (int k = 0; k < KS; k++) v += red[((size_t)(warp + k) * 32 + lane) * 16 + q * 8 + s2 * 4 + r];
              acc[q][s2][r] = v;
            }
      }
      __syncthreads();
      if (kp != 0 || !mine) continue;
    }
    if (!ok) continue;
    // C fragment: [q][s][0..1] row g, tokens 8q+2t, +1; [2..3] row g+8
#pragma unroll
    for (int q = 0; q < 2; q++)
#pragma unroll
      for (int col = 0; col < 2; col++) {
        const int j = 8 * q + 2 * t + col;
        if (j >= (int)c.n) continue;
        const size_t pos = c.p0 + j;
#pragma unroll
        for (int h = 0; h < 2; h++) {
          if (EPI == 1) {
            const int o = 16 * tile + g + 8 * h;
            if (o < p.FF) p.yh[pos * p.FF + xfo_pos(o)] = f2h(gelu_tanh(acc[q][0][2 * h + col]) * acc[q][1][2 * h + col]);
          } else {
#pragma unroll
            for (int s = 0; s < NS; s++) {
              const int r = (MODE == 0 ? 32 : 16) * tile + 16 * s + g + 8 * h;
              if (r < p.ROWS) p.y[pos * p.ROWS + r] = acc[q][s][2 * h + col];
            }
          }
        }
      }
  }
}

// out[t][o] = sum_k w[t][k] * y[inv[t K + k]][o], slots in order (kernels/wacc.wgsl).
__global__ void k_wacc(const float* __restrict__ y, const uint32_t* __restrict__ inv, const float* __restrict__ tkw,
                       float* __restrict__ out, int n, int K, int OUT) {
  pdl_wait();
  const int tok = blockIdx.y;
  const int o = blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= OUT || tok >= n) return;
  float acc = 0.f;
  for (int k = 0; k < K; k++) acc += tkw[tok * K + k] * y[(size_t)inv[tok * K + k] * OUT + o];
  out[(size_t)tok * OUT + o] = acc;
}

// ---- dense batch, K split across CTAs: y_parts[kp][t][row] = W[row][K-part kp] x_t.
// Item = (K-part, group of kKW 32-row tiles, one per warp); items are K-part
// major, so a CTA restages its activations (all <= 64 tokens, only the part's
// k-range) once per part it visits, as 2-D TMA boxes of [64 tokens x 64 halves]
// under the 128-byte swizzle (four per 256-k quantum; conflict-free reads).  Every weight is decoded once for all the
// tokens (8 MMA column groups); the consumer sums the parts in order.
constexpr int kKW = 8, kKS = 3;

struct QkpP {
  const uint16_t* x;             // [n][IN] fragment order
  float* y;                      // [kparts][n][ROWS]
  uint32_t* status;
  int IN, nb, ROWS, n, tiles, nq, kparts, groups, xpitch;   // groups = tile groups; xpitch = staged quanta
};

E4B_DEV int kq_begin(const QkpP& p, int kp) { return p.nq * kp / p.kparts; }

__global__ void __launch_bounds__(32 * kKW, 1) k_qkp(const QkpP p, const __grid_constant__ CUtensorMap map,
                                                     const __grid_constant__ CUtensorMap xmap) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kKW][kKS];
  __shared__ __align__(8) uint64_t xbar;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  // xpitch: staged quanta per part; each quantum is 4 swizzled boxes of 8 KB
  uint8_t* xs = smem + ((1024u - (smem_u32(smem) & 1023u)) & 1023u);
  uint8_t* stages = xs + (size_t)p.xpitch * 32768 + (size_t)warp * kKS * kQuantumBytes;
  const int T = p.kparts * p.groups;
  const int i0 = (int)((int64_t)T * blockIdx.x / gridDim.x), i1 = (int)((int64_t)T * (blockIdx.x + 1) / gridDim.x);
  pdl_trigger();
  if (lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map)) : "memory");
    if (warp == 0) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&xmap)) : "memory");
    for (int s = 0; s < kKS; s++) mbar_init(&full[warp][s], 1);
    if (warp == 0) mbar_init(&xbar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  // producer cursor over this warp's (item, quantum) sequence; weights only, so
  // the first quanta are requested before the wait on the previous kernel
  auto has_tile = [&](int it) { return (it % p.groups) * kKW + warp < p.tiles; };
  int pit = i0;
  while (pit < i1 && !has_tile(pit)) pit++;
  int pkq = pit < i1 ? kq_begin(p, pit / p.groups) : 0;
  auto issue = [&](int s) {
    const int tile = (pit % p.groups) * kKW + warp, kp = pit / p.groups;
    if (lane == 0) mbar_expect_tx(&full[warp][s], (uint32_t)kQuantumBytes);
    __syncwarp();
    if (lane < 2) tma_load_2d(stages + s * kQuantumBytes + lane * kSubBytes, &map, pkq * 18, 32 * tile + 16 * lane,
                              &full[warp][s]);
    if (++pkq == kq_begin(p, kp + 1)) {
      do pit++; while (pit < i1 && !has_tile(pit));
      if (pit < i1) pkq = kq_begin(p, pit / p.groups);
    }
  };
#pragma unroll
  for (int s = 0; s < kKS; s++)
    if (pit < i1) issue(s);
  pdl_wait();

  Lane L;
  L.o_odd = 2 + 4 * t;
  L.o_e1 = t < 3 ? 4 + 4 * t : 0;
  L.sel = t < 3 ? 0x3210u : 0x5432u;
  const int ng = (p.n + 7) >> 3;
  bool ok = true;
  int cur = -1, restage = 0, used = 0;
  for (int it = i0; it < i1; it++) {
    const int kp = it / p.groups, q0 = kq_begin(p, kp), q1 = kq_begin(p, kp + 1);
    if (kp != cur) {
      __syncthreads();          // every warp is done with the previous part's activations
      if (threadIdx.x == 0) {
        mbar_expect_tx(&xbar, (uint32_t)(q1 - q0) * 32768u);
        for (int b = 0; b < 4 * (q1 - q0); b++) tma_load_2d(xs + (size_t)b * 8192, &xmap, 256 * q0 + 64 * b, 0, &xbar);
      }
      if (ok) ok = mbar_wait(&xbar, (uint32_t)(restage & 1), p.status);
      restage++;
      cur = kp;
    }
    if (!has_tile(it)) continue;
    const int tile = (it % p.groups) * kKW + warp;
    float acc[8][2][4];
#pragma unroll
    for (int q = 0; q < 8; q++)
#pragma unroll
      for (int s = 0; s < 2; s++)
#pragma unroll
        for (int r = 0; r < 4; r++) acc[q][s][r] = 0.f;
    // token 8q + g, block k of quantum kq: box 4 (kq - q0) + k / 2, row 8q + g,
    // 16-byte chunk (4 (k & 1) + t) ^ g
    uint32_t xoff[2];
#pragma unroll
    for (int h = 0; h < 2; h++) xoff[h] = (uint32_t)(g * 128 + (((4 * h + t) ^ g) << 4));
    for (int kq = q0; kq < q1; kq++, used++) {
      const int s = used % kKS;
      if (ok) ok = mbar_wait(&full[warp][s], (uint32_t)((used / kKS) & 1), p.status);
      if (ok) {
        const uint8_t* a = stages + s * kQuantumBytes + g * kRowPitch;
        const uint8_t* xq = xs + (size_t)(kq - q0) * 32768;
#pragma unroll 2
        for (int k = 0; k < 8; k++) {
          const int par = k & 1;
          uint32_t A[2][8];
          float d[2][2];
#pragma unroll
          for (int sb = 0; sb < 2; sb++) {
            const uint8_t* ra = a + sb * kSubBytes + 18 * k;
            const uint8_t* rb = ra + 8 * kRowPitch;
            dq_row(par ? nib_odd(ra, L) : nib_even(ra, L), A[sb][0], A[sb][1], A[sb][2], A[sb][3]);
            dq_row(par ? nib_odd(rb, L) : nib_even(rb, L), A[sb][4], A[sb][5], A[sb][6], A[sb][7]);
            d[sb][0] = h2f(*reinterpret_cast<const uint16_t*>(ra));
            d[sb][1] = h2f(*reinterpret_cast<const uint16_t*>(rb));
          }
#pragma unroll
          for (int q = 0; q < 8; q++) {
            if (q >= ng) break;
            const uint4 xb = *reinterpret_cast<const uint4*>(xq + (k >> 1) * 8192 + q * 1024 + xoff[k & 1]);
#pragma unroll
            for (int sb = 0; sb < 2; sb++) {
              float c[4] = {0.f, 0.f, 0.f, 0.f};
              mma16816(c, A[sb][0], A[sb][4], A[sb][1], A[sb][5], xb.x, xb.y);
              mma16816(c, A[sb][2], A[sb][6], A[sb][3], A[sb][7], xb.z, xb.w);
              acc[q][sb][0] = fmaf(d[sb][0], c[0], acc[q][sb][0]);
              acc[q][sb][1] = fmaf(d[sb][0], c[1], acc[q][sb][1]);
              acc[q][sb][2] = fmaf(d[sb][1], c[2], acc[q][sb][2]);
              acc[q][sb][3] = fmaf(d[sb][1], c[3], acc[q][sb][3]);
            }
          }
        }
      }
      __syncwarp();
      if (ok && pit < i1) issue(s);
    }
    if (!ok) continue;
    float* yp = p.y + (size_t)kp * p.n * p.ROWS;
#pragma unroll
    for (int q = 0; q < 8; q++) {
      if (q >= ng) break;
#pragma unroll
      for (int col = 0; col < 2; col++) {
        const int j = 8 * q + 2 * t + col;
        if (j >= p.n) continue;
#pragma unroll
        for (int h = 0; h < 2; h++)
#pragma unroll
          for (int sb = 0; sb < 2; sb++) {
            const int r = 32 * tile + 16 * sb + g + 8 * h;
            if (r < p.ROWS) yp[(size_t)j * p.ROWS + r] = acc[q][sb][2 * h + col];
          }
      }
    }
  }
}

template <int MODE, int EPI, int W, int S, int TOKC, int KS, int PK = 0>
int qmm_launch(e4b_ctx* c, const char* name, const QmmP& p, const CUtensorMap& map, size_t smem, int grid) {
  auto kern = k_qmm<MODE, EPI, W, S, TOKC, KS, PK>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e4b_fail(c, E4B_ECUDA, "%s smem attr: %s", name, cudaGetErrorString(e));
  return e4b_launch(c, name, kern, dim3((unsigned)grid), dim3(32 * W), smem, p, map);
}

// Shared memory a variant needs: staged activations + the warps' rings.
size_t qmm_smem(const QmmP& p, int mode, int W, int S, int tokc, int ks) {
  const size_t stage = mode == 0 ? (size_t)kQuantumBytes : 16 * (size_t)p.rowbytes;
  return (size_t)tokc * p.xpitch * 2 + (size_t)W * S * stage + (ks > 1 ? (size_t)W * 32 * 16 * 4 : 0);
}
constexpr size_t kQmmSmemCap = 227 * 1024 - 8 * 1024;   // dynamic budget beside the static chunk list

// x: activations in fragment order; grouped when offsets != null.
int qmm(e4b_ctx* c, const char* name, const uint16_t* x, const uint8_t* w, const uint32_t* offsets,
        const uint32_t* entries, float* y, uint16_t* yh, int IN, int ROWS, int FF, int K, int E, int n_dense,
        int epi, bool packed = false) {
  E4B_REQUIRE(c, reinterpret_cast<uintptr_t>(w) % 16 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0,
              "%s: weights and activations must be 16-byte aligned", name);
  E4B_REQUIRE(c, IN > 0 && IN % 64 == 0 && IN <= 16384, "%s: IN=%d must be a multiple of 64 (<= 16384)", name, IN);
  QmmP p = {};
  p.x = x; p.w = w; p.offsets = offsets; p.entries = entries; p.y = y; p.yh = yh; p.status = c->status;
  p.IN = IN; p.nb = IN / 32; p.rowbytes = p.nb * 18; p.ROWS = ROWS; p.FF = FF; p.K = K; p.E = E;
  p.n_dense = n_dense;
  p.xpitch = IN + 32;
  const int mode = (IN % 256 == 0 && tensor_map_encoder() != nullptr) ? 0 : 1;
  E4B_REQUIRE(c, mode == 0 || epi == 0, "%s: the gate|up GEMM needs IN %% 256 == 0 (IN=%d)", name, IN);
  E4B_REQUIRE(c, mode == 0 || ROWS % 16 == 0, "%s: ROWS=%d must be a multiple of 16 for IN=%d", name, ROWS, IN);
  p.tiles = epi == 1 ? (FF + 15) / 16 : (mode == 0 ? (ROWS + 31) / 32 : ROWS / 16);
  p.nq = mode == 0 ? (p.nb + 7) / 8 : 1;
  CUtensorMap map;
  memset(&map, 0, sizeof(map));
  if (mode == 0) {
    const cuuint64_t gdim[2] = {(cuuint64_t)(p.rowbytes / 8), (cuuint64_t)E * (cuuint64_t)ROWS};
    const cuuint64_t gstride[1] = {(cuuint64_t)p.rowbytes};
    const cuuint32_t box[2] = {kRowPitch / 8, 16};
    const cuuint32_t estride[2] = {1, 1};
    CUresult r = tensor_map_encoder()(&map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<uint8_t*>(w), gdim, gstride,
                                      box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    E4B_REQUIRE(c, r == CUDA_SUCCESS, "%s: cuTensorMapEncodeTiled failed (%d)", name, (int)r);
  }
  // variants (warps, stages, tokens per chunk), first that fits the shared
  // memory: grouped experts hold few tokens each, so 8-token chunks and 16
  // warps (more warps hide the dequant's latencies); a dense batch reuses each
  // dequantised weight for 16 tokens.
  struct V { int W, S, T, KS; };
  static const V cand[7] = {{16, 2, 8, 1}, {8, 3, 16, 4}, {8, 2, 16, 4}, {8, 3, 16, 1}, {8, 2, 16, 1},
                            {4, 2, 16, 1}, {4, 2, 8, 1}};
  int vi = -1;
  for (int i = offsets ? 0 : 1; i < 7 && vi < 0; i++) {
    if (cand[i].KS > 1 && p.nq < cand[i].KS) continue;      // nothing to split (whole-row stages)
    if (qmm_smem(p, mode, cand[i].W, cand[i].S, cand[i].T, cand[i].KS) <= kQmmSmemCap) vi = i;
  }
  E4B_REQUIRE(c, vi >= 0, "%s: IN=%d needs more shared memory than a CTA has", name, IN);
  const V v = cand[vi];
  const int tpi = v.W / v.KS;
  p.RR = (p.tiles + tpi - 1) / tpi;
  int grid = c->sm_count;
  if (!offsets) {
    E4B_REQUIRE(c, (n_dense + v.T - 1) / v.T <= kMaxChunks, "%s: n=%d tokens exceed %d", name, n_dense,
                v.T * kMaxChunks);
    const int items = (n_dense + v.T - 1) / v.T * p.RR;
    if (grid > items) grid = items;
  }
  if (grid < 1) grid = 1;
  const size_t sm = qmm_smem(p, mode, v.W, v.S, v.T, v.KS);
  if (packed) {
    // the tile-packed weights: grouped gate|up only, on the grouped variant
    E4B_REQUIRE(c, mode == 0 && epi == 1 && offsets && vi == 0 && FF % 16 == 0,
                "%s: the tile-packed path needs IN %% 256 == 0 and the grouped gate|up GEMM (IN=%d)", name, IN);
    return qmm_launch<0, 1, 16, 2, 8, 1, 1>(c, name, p, map, sm, grid);
  }
#define QMM_CASE(M, EP)                                                          \
  if (mode == M && epi == EP) {                                                  \
    switch (vi) {                                                                \
      case 0: return qmm_launch<M, EP, 16, 2, 8, 1>(c, name, p, map, sm, grid);  \
      case 1: return qmm_launch<M, EP, 8, 3, 16, 4>(c, name, p, map, sm, grid);  \
      case 2: return qmm_launch<M, EP, 8, 2, 16, 4>(c, name, p, map, sm, grid);  \
      case 3: return qmm_launch<M, EP, 8, 3, 16, 1>(c, name, p, map, sm, grid);  \
      case 4: return qmm_launch<M, EP, 8, 2, 16, 1>(c, name, p, map, sm, grid);  \
      case 5: return qmm_launch<M, EP, 4, 2, 16, 1>(c, name, p, map, sm, grid);  \
      default: return qmm_launch<M, EP, 4, 2, 8, 1>(c, name, p, map, sm, grid);  \
    }                                                                            \
  }
  QMM_CASE(0, 0)
  QMM_CASE(0, 1)
  QMM_CASE(1, 0)
#undef QMM_CASE
  return e4b_fail(c, E4B_EINVAL, "%s: no kernel variant", name);
}

}  // namespace

extern "C" {

// dst[i] = src[idx[i] / div] (f16 rows of H), a zero row where idx[i] is the
// empty marker: the activation rows of expert-sorted entries, contiguous per
// expert, for the grouped prefill GEMM.
__global__ void k_gather_rows(const uint16_t* __restrict__ src, const uint32_t* __restrict__ idx, int div,
                              uint16_t* __restrict__ dst, int H, int n, int n_src) {
  pdl_wait();
  const int i = blockIdx.x;
  if (i >= n) return;
  const uint32_t e = idx[i];
  const uint32_t r = e == 0xffffffffu ? 0xffffffffu : e / (uint32_t)div;
  uint4* d = reinterpret_cast<uint4*>(dst + (size_t)i * H);
  if (r >= (uint32_t)n_src) {
    for (int j = threadIdx.x; j < H / 8; j += blockDim.x) d[j] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint4* s = reinterpret_cast<const uint4*>(src + (size_t)r * H);
  for (int j = threadIdx.x; j < H / 8; j += blockDim.x) d[j] = s[j];
}

E4B_API int e4b_gather_rows(e4b_ctx* c, const uint16_t* src, const uint32_t* idx, int div, uint16_t* dst, int H,
                            int n, int n_src) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, src && idx && dst && div > 0 && n > 0 && n_src > 0 && H > 0 && H % 8 == 0,
              "gather_rows: bad args (H=%d must be a multiple of 8)", H);
  E4B_REQUIRE(c, reinterpret_cast<uintptr_t>(src) % 16 == 0 && reinterpret_cast<uintptr_t>(dst) % 16 == 0,
              "gather_rows: rows must be 16-byte aligned");
  return e4b_launch(c, "gather_rows", k_gather_rows, dim3(n), dim3(128), 0, src, idx, div, dst, H, n, n_src);
}

E4B_API int e4b_expgroup(e4b_ctx* c, const uint32_t* topk, int n_tok, int K, int E, uint32_t* offsets,
                         uint32_t* entries, uint32_t* inv) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, topk && offsets && entries && inv, "expgroup: null buffer");
  E4B_REQUIRE(c, n_tok > 0 && K > 0 && E > 0 && E <= 4096 && (long long)n_tok * K < (1ll << 24),
              "expgroup: bad sizes n=%d K=%d E=%d", n_tok, K, E);
  if (E <= kSortE)
    return e4b_launch(c, "expgroup", k_expsort, dim3(1), dim3(1024), 0, topk, n_tok * K, E, offsets, entries, inv,
                      c->status);
  return e4b_launch(c, "expgroup", k_expgroup, dim3(1), dim3(1024), (size_t)(E + 1) * 4, topk, n_tok * K, E, offsets,
                    entries, inv, c->status);
}

E4B_API int e4b_q40gugrp(e4b_ctx* c, const uint16_t* x, const uint8_t* w, const uint32_t* offsets,
                         const uint32_t* entries, uint16_t* yh, int IN, int FF, int E, int K) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, x && w && offsets && entries && yh, "q40gugrp: null buffer");
  E4B_REQUIRE(c, FF > 0 && FF % 32 == 0 && E > 0 && E <= 4096 && K > 0, "q40gugrp: bad sizes FF=%d E=%d", FF, E);
  return qmm(c, "q40gugrp", x, w, offsets, entries, nullptr, yh, IN, 2 * FF, FF, K, E, 0, 1);
}

E4B_API int e4b_q40_pack_tiles(e4b_ctx* c, const uint8_t* w, uint8_t* wt, int rows, int IN) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, w && wt && w != wt, "q40_pack_tiles: null or aliased buffers");
  E4B_REQUIRE(c, rows > 0 && rows % 16 == 0 && rows / 16 <= 65535 && IN > 0 && IN % 256 == 0,
              "q40_pack_tiles: rows=%d (a multiple of 16) x IN=%d (a multiple of 256)", rows, IN);
  E4B_REQUIRE(c, reinterpret_cast<uintptr_t>(wt) % 16 == 0, "q40_pack_tiles: packed copy must be 16-byte aligned");
  return e4b_launch(c, "q40_pack_tiles", k_q40_pack, dim3(IN / 256, rows / 16), dim3(128), 0, w, wt, IN);
}

E4B_API int e4b_q40gugrp_tiles(e4b_ctx* c, const uint16_t* x, const uint8_t* wt, const uint32_t* offsets,
                               const uint32_t* entries, uint16_t* yh, int IN, int FF, int E, int K) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, x && wt && offsets && entries && yh, "q40gugrp_tiles: null buffer");
  E4B_REQUIRE(c, FF > 0 && FF % 32 == 0 && E > 0 && E <= 4096 && K > 0, "q40gugrp_tiles: bad sizes FF=%d E=%d", FF,
              E);
  return qmm(c, "q40gugrp_tiles", x, wt, offsets, entries, nullptr, yh, IN, 2 * FF, FF, K, E, 0, 1, true);
}

E4B_API int e4b_q40downgrp(e4b_ctx* c, const uint16_t* x, const uint8_t* w, const uint32_t* offsets,
                           const uint32_t* entries, float* y, int IN, int OUT, int E) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, x && w && offsets && entries && y, "q40downgrp: null buffer");
  E4B_REQUIRE(c, OUT > 0 && E > 0 && E <= 4096, "q40downgrp: bad sizes OUT=%d E=%d", OUT, E);
  return qmm(c, "q40downgrp", x, w, offsets, nullptr, y, nullptr, IN, OUT, 0, 1, E, 0, 0);
}

E4B_API int e4b_q40mm(e4b_ctx* c, const uint16_t* x, const uint8_t* w, float* y, int IN, int OUT, int n) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, x && w && y && n > 0 && OUT > 0, "q40mm: bad args");
  return qmm(c, "q40mm", x, w, nullptr, nullptr, y, nullptr, IN, OUT, 0, 1, 1, n, 0);
}

E4B_API int e4b_q40mm_kparts(e4b_ctx* c, const uint16_t* x, const uint8_t* w, float* y_parts, int IN, int OUT, int n,
                             int kparts) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, x && w && y_parts && n > 0 && n <= 64 && OUT > 0, "q40mm_kparts: bad args (n <= 64)");
  E4B_REQUIRE(c, IN > 0 && IN % 256 == 0 && IN <= 16384 && tensor_map_encoder(), "q40mm_kparts: IN=%d must be a multiple of 256", IN);
  E4B_REQUIRE(c, reinterpret_cast<uintptr_t>(w) % 16 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0,
              "q40mm_kparts: weights and activations must be 16-byte aligned");
  QkpP p = {};
  p.x = x; p.y = y_parts; p.status = c->status;
  p.IN = IN; p.nb = IN / 32; p.ROWS = OUT; p.n = n;
  p.nq = p.nb / 8;
  E4B_REQUIRE(c, kparts >= 1 && kparts <= p.nq, "q40mm_kparts: kparts=%d must be in [1, %d]", kparts, p.nq);
  p.kparts = kparts;
  p.tiles = (OUT + 31) / 32;
  p.groups = (p.tiles + kKW - 1) / kKW;
  const int max_q = (p.nq + kparts - 1) / kparts;
  p.xpitch = max_q;
  const size_t smem = (size_t)max_q * 32768 + (size_t)kKW * kKS * kQuantumBytes + 1024;
  E4B_REQUIRE(c, smem <= kQmmSmemCap, "q40mm_kparts: %d quanta per part need too much shared memory", max_q);
  const int rowbytes = p.nb * 18;
  CUtensorMap map;
  const cuuint64_t gdim[2] = {(cuuint64_t)(rowbytes / 8), (cuuint64_t)OUT};
  const cuuint64_t gstride[1] = {(cuuint64_t)rowbytes};
  const cuuint32_t box[2] = {kRowPitch / 8, 16};
  const cuuint32_t estride[2] = {1, 1};
  CUresult r = tensor_map_encoder()(&map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<uint8_t*>(w), gdim, gstride,
                                    box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  E4B_REQUIRE(c, r == CUDA_SUCCESS, "q40mm_kparts: cuTensorMapEncodeTiled failed (%d)", (int)r);
  // the activations [n][IN] f16 as boxes of 64 halves x 64 rows (rows past n read as zeros)
  CUtensorMap xmap;
  {
    const cuuint64_t xd[2] = {(cuuint64_t)IN, (cuuint64_t)n};
    const cuuint64_t xs[1] = {(cuuint64_t)IN * 2};
    const cuuint32_t xb[2] = {64, 64};
    CUresult rx = tensor_map_encoder()(&xmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint16_t*>(x), xd, xs, xb,
                                       estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    E4B_REQUIRE(c, rx == CUDA_SUCCESS, "q40mm_kparts: activation tensor map failed (%d)", (int)rx);
  }
  cudaError_t e = cudaFuncSetAttribute(k_qkp, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e4b_fail(c, E4B_ECUDA, "q40mm_kparts smem attr: %s", cudaGetErrorString(e));
  const int items = kparts * p.groups;
  const int grid = items < c->sm_count ? items : c->sm_count;
  return e4b_launch(c, "q40mm_kparts", k_qkp, dim3((unsigned)grid), dim3(32 * kKW), smem, p, map, xmap);
}

E4B_API int e4b_q40gumm(e4b_ctx* c, const uint16_t* x, const uint8_t* w, uint16_t* yh, int IN, int FF, int n) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, x && w && yh && n > 0 && FF > 0 && FF % 32 == 0, "q40gumm: bad args");
  return qmm(c, "q40gumm", x, w, nullptr, nullptr, nullptr, yh, IN, 2 * FF, FF, 1, 1, n, 1);
}

E4B_API int e4b_wacc(e4b_ctx* c, const float* y, const uint32_t* inv, const float* topk_w, float* out, int n_tok,
                     int K, int OUT) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, y && inv && topk_w && out && n_tok > 0 && K > 0 && OUT > 0, "wacc: bad args");
  return e4b_launch(c, "wacc", k_wacc, dim3((OUT + 255) / 256, n_tok), dim3(256), 0, y, inv, topk_w, out, n_tok, K,
                    OUT);
}

}  // extern "C"
