// Streaming q4_0 GEMV on the tensor cores (sm_100a).
//
// y[o] = sum_b d[o][b] * sum_{i<32} (n[o][b][i] - 8) * x[32b + i]  over raw GGUF
// q4_0 rows (18-byte blocks), with f16 (or f32) activations.
//
// Data movement: the weight matrix, viewed as rows of 8-byte words, is read by
// 2-D TMA tensor loads (cp.async.bulk.tensor.2d) of [16 rows x 8 blocks] boxes
// (2304 B, one "quantum" per 16-row subtile) straight into shared memory, where
// a box lands as 16 rows of 144 B -- a row pitch of 36 words, so the 8 rows a
// warp reads fall 4 banks apart (conflict-free).  No repacking: the blocks are
// the GGUF bytes.
//
// Work split ("stream-K"): a tile is 32 rows (two 16-row subtiles; for the
// fused gate|up, 16 gate rows + the matching 16 up rows) and a quantum is one
// tile x 8 blocks.  Every warp of a persistent grid is an independent worker
// with a contiguous range of quanta (balanced across all warps of the GPU to
// within one quantum) and its own 2-stage mbarrier ring of pieces (up to PQ
// quanta of one tile).  The first pieces are issued before griddepcontrol.wait:
// weights never depend on the previous kernel.
//
// Math per 8-block group, per 16-row subtile, on the tensor cores (mma.sync
// m16n8k16, f16 x f16 -> f32):
//   A (16 rows x 16 k) = nibbles n-8, exact in f16 (LOP3 magic-number decode);
//   B (16 k x 8 cols)  = x, block-diagonal: column j holds block j's activations;
//   C[row][j]          = sum_i (n-8) x over block j (exact products, f32 sums),
// then d[row][block] (f16) scales column j in f32, so the arithmetic is the
// reference's (kernels/q40mv.wgsl:38-54, 78-84) up to f32 summation order.  A
// tile cut by a worker boundary is merged by its last finishing worker, which
// sums the published partials in k order (deterministic).
#include <cuda.h>
#include <cudaTypedefs.h>

#include "q40_frag.cuh"
#include "q40_stream.cuh"

namespace {
using namespace e4b;


struct Q40P {
  const void* x;
  float* y;
  uint16_t* yh;
  const float* ple;
  float* part;                  // [n_rt][qpr][32] split partials
  uint32_t* ctr;                // [n_rt] arrival counters (zero at rest)
  unsigned long long* starts;   // [n_rt] bit c: a partial was published at slot c (zero at rest)
  uint32_t* status;
  int IN, OUT, nb, ff, off;
  int epi;
  int n_rt;                     // tiles of 32 rows (gate|up: 16 outputs)
  int qpr;                      // quanta per tile = nb / 8
  int Q;                        // total quanta
};

// First tensor row of subtile s of tile rt.
E4B_DEV int sub_row(const Q40P& p, int rt, int s) {
  if (p.epi == 1) return s == 0 ? 16 * rt : p.ff + 16 * rt;
  return 32 * rt + 16 * s;
}

struct Piece {
  int rt, qa, qb;    // tile, quanta [qa, qb) relative to the tile
};
template <int PQ>
E4B_DEV Piece piece_at(const Q40P& p, int q, int q1) {
  Piece pc;
  pc.rt = q / p.qpr;
  pc.qa = q - pc.rt * p.qpr;
  const int end = min(min(q1, (pc.rt + 1) * p.qpr), q + PQ);
  pc.qb = pc.qa + (end - q);
  return pc;
}

// Lane 2*j + s issues quantum j, subtile s of the piece (rows beyond the
// tensor are zero-filled by the TMA unit and still count as transferred bytes).
E4B_DEV void issue_piece(const Q40P& p, const CUtensorMap* map, const Piece& pc, uint8_t* stage, uint64_t* bar,
                         int lane) {
  const int nq = pc.qb - pc.qa;
  if (lane == 0) mbar_expect_tx(bar, (uint32_t)(nq * kQuantumBytes));
  __syncwarp();
  if (lane < 2 * nq) {
    const int j = lane >> 1, s = lane & 1;
    tma_load_2d(stage + j * kQuantumBytes + s * kSubBytes, map, (pc.qa + j) * 18, sub_row(p, pc.rt, s), bar);
  }
}

template <int XF32, int EPI, int kW, int kS, int PQ>
__global__ void __launch_bounds__(32 * kW, 1) k_q40_stream(const Q40P p, const __grid_constant__ CUtensorMap map) {
  constexpr int kStageBytes = PQ * kQuantumBytes;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kW][kS];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int NW = gridDim.x * kW, vw = blockIdx.x * kW + warp;
  const int q0 = (int)part_begin(p.Q, NW, vw), q1 = (int)part_begin(p.Q, NW, vw + 1);
  uint8_t* stages = smem + (size_t)warp * kS * kStageBytes;

  pdl_trigger();
  if (lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map)) : "memory");
    for (int s = 0; s < kS; s++) mbar_init(&full[warp][s], 1);
    fence_barrier_init();
  }
  __syncwarp();
  // first pieces: weights only, so before the dependency wait
  int qn = q0;
  Piece ring[kS];
  int issued = 0;
#pragma unroll
  for (int s = 0; s < kS; s++) {
    ring[s] = Piece{0, 0, 0};
    if (qn < q1) {
      ring[s] = piece_at<PQ>(p, qn, q1);
      issue_piece(p, &map, ring[s], stages + s * kStageBytes, &full[warp][s], lane);
      qn += ring[s].qb - ring[s].qa;
      issued++;
    }
  }

  pdl_wait();

  Lane L;
  L.o_odd = 2 + 4 * t;
  L.o_e1 = t < 3 ? 4 + 4 * t : 0;
  L.sel = t < 3 ? 0x3210u : 0x5432u;
  const XLane X = xlane(g, t);
  // activations of this lane's block of the first quantum (one quantum of lookahead)
  uint4 xh = make_uint4(0, 0, 0, 0), xl = make_uint4(0, 0, 0, 0);
  if (issued) xfrag<XF32>(p.x, (ring[0].qa) * 8 + g, X, xh, xl);

  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  int cover_begin = -1, covered = 0;
  bool ok = true;
  for (int i = 0; i < issued; i++) {
    const int s = i % kS;
    Piece pc = ring[0];
#pragma unroll
    for (int k = 1; k < kS; k++)
      if (s == k) pc = ring[k];
    if (cover_begin < 0) {
      cover_begin = pc.qa;
      covered = 0;
    }
    if (ok) ok = mbar_wait(&full[warp][s], (uint32_t)((i / kS) & 1), p.status);
    if (ok) {
      const uint8_t* st = stages + s * kStageBytes;
      for (int j = 0; j < pc.qb - pc.qa; j++) {
        // prefetch the next quantum's activations (next in this piece, or the next piece)
        uint4 nh = make_uint4(0, 0, 0, 0), nl = make_uint4(0, 0, 0, 0);
        int nq = -1;
        if (j + 1 < pc.qb - pc.qa) {
          nq = pc.qa + j + 1;
        } else if (i + 1 < issued) {
          Piece nx = ring[0];
#pragma unroll
          for (int k = 1; k < kS; k++)
            if ((i + 1) % kS == k) nx = ring[k];
          nq = nx.qa;
        }
        if (nq >= 0) xfrag<XF32>(p.x, nq * 8 + g, X, nh, nl);
        quantum_mma<XF32>(st + j * kQuantumBytes, xh, xl, L, g, t, acc);
        xh = nh;
        xl = nl;
      }
    }
    covered += pc.qb - pc.qa;
    // refill: every lane's shared-memory reads of this stage have returned
    // (their values fed the MMAs above) before the TMA unit overwrites it
    __syncwarp();
    if (qn < q1 && ok) {
      const Piece nx = piece_at<PQ>(p, qn, q1);
      issue_piece(p, &map, nx, stages + s * kStageBytes, &full[warp][s], lane);
#pragma unroll
      for (int k = 0; k < kS; k++)
        if (s == k) ring[k] = nx;
      qn += nx.qb - nx.qa;
      issued++;
    }
    if (!(pc.qb == p.qpr || i + 1 == issued)) continue;   // tile not finished by this worker yet
    float v[4];
#pragma unroll
    for (int r = 0; r < 4; r++) {
      v[r] = acc[r];
      v[r] += __shfl_xor_sync(0xffffffffu, v[r], 1);
      v[r] += __shfl_xor_sync(0xffffffffu, v[r], 2);
      acc[r] = 0.f;
    }
    const int rt = pc.rt;
    const int cb = cover_begin, cov = covered;
    cover_begin = -1;
    if (!(cb == 0 && cov == p.qpr)) {
      // split tile: publish this worker's partial; the last arrival merges in k order
      float* slot = p.part + ((size_t)rt * p.qpr + cb) * 32;
      if (t == 0) {
        slot[g] = v[0];
        slot[8 + g] = v[1];
        slot[16 + g] = v[2];
        slot[24 + g] = v[3];
      }
      __syncwarp();   // the lanes' partial stores happen before lane 0's release
      uint32_t last = 0;
      if (lane == 0) {
        atom_or_release(&p.starts[rt], 1ull << cb);
        last = atom_add_acq_rel(&p.ctr[rt], (uint32_t)cov) + (uint32_t)cov == (uint32_t)p.qpr;
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      if (!last) continue;
      unsigned long long m = 0;
      if (lane == 0) m = atom_or_acquire(&p.starts[rt], 0ull);
      m = __shfl_sync(0xffffffffu, m, 0);
      v[0] = v[1] = v[2] = v[3] = 0.f;
      while (m) {                              // slots in increasing k order
        const int c = __ffsll((long long)m) - 1;
        m &= m - 1;
        const float* sl = p.part + ((size_t)rt * p.qpr + c) * 32;
        v[0] += __ldcg(sl + g);
        v[1] += __ldcg(sl + 8 + g);
        v[2] += __ldcg(sl + 16 + g);
        v[3] += __ldcg(sl + 24 + g);
      }
      if (lane == 0) {
        p.ctr[rt] = 0;
        p.starts[rt] = 0ull;
      }
    }
    if (t == 0) {
      if (EPI == 1) {
        // subtile 0 = gate rows 16rt.., subtile 1 = the matching up rows
        const int e0 = 16 * rt + g, e1 = e0 + 8;
        if (e0 < p.ff) p.yh[e0] = f2h(gelu_tanh(v[0]) * v[2]);
        if (e1 < p.ff) p.yh[e1] = f2h(gelu_tanh(v[1]) * v[3]);
      } else {
        const int o[4] = {32 * rt + g, 32 * rt + 8 + g, 32 * rt + 16 + g, 32 * rt + 24 + g};
#pragma unroll
        for (int r = 0; r < 4; r++) {
          if (o[r] >= p.OUT) continue;
          if (EPI == 0) p.y[o[r]] = v[r];
          else p.yh[o[r]] = f2h(gelu_tanh(v[r]) * p.ple[p.off + o[r]]);
        }
      }
    }
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }
  return fn;
}

template <int XF32, int EPI, int kW, int kS, int PQ>
int launch(e4b_ctx* c, const Q40P& p, const CUtensorMap& map, const char* name) {
  const size_t smem = (size_t)kW * kS * PQ * kQuantumBytes;
  auto kern = k_q40_stream<XF32, EPI, kW, kS, PQ>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e4b_fail(c, E4B_ECUDA, "%s smem attr: %s", name, cudaGetErrorString(e));
  int per_sm = 1;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 32 * kW, smem);
  if (per_sm < 1) per_sm = 1;
  const int want = c->stream_ctas_per_sm;
  int64_t G = (int64_t)c->sm_count * (per_sm < want ? per_sm : want);
  const int64_t need = (p.Q + 2 * kW - 1) / (2 * kW);     // at least 2 quanta per worker
  if (G > need) G = need;
  return e4b_launch(c, name, kern, dim3((unsigned)G), dim3(32 * kW), smem, p, map);
}

// Warps per CTA x stages per warp x quanta per stage.  Shared memory stays at
// ~110 KB so the next kernel's CTA fits beside this one and can prefetch its
// weights under programmatic dependent launch.
template <int XF32, int EPI>
int launch_variant(e4b_ctx* c, const Q40P& p, const CUtensorMap& map, const char* name) {
  switch (c->stream_variant) {
    case 1: return launch<XF32, EPI, 4, 3, 2>(c, p, map, name);     // 110.6 KB
    case 2: return launch<XF32, EPI, 8, 2, 2>(c, p, map, name);     // 147.5 KB
    default: return launch<XF32, EPI, 8, 3, 1>(c, p, map, name);    // 110.6 KB
  }
}

}  // namespace

namespace e4b {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() { return encode_fn(); }

bool q40_stream_supported(const void* w, const void* x, int IN, int rows) {
  (void)rows;
  if (IN <= 0 || IN % 256 || IN > 16384) return false;           // whole 8-block groups, 16-byte rows
  if (reinterpret_cast<uintptr_t>(w) % 16) return false;         // TMA global address alignment
  if (reinterpret_cast<uintptr_t>(x) % 16) return false;         // x is staged with 16-byte loads
  return encode_fn() != nullptr;
}

int q40_stream(e4b_ctx* c, const uint8_t* w, const void* x, int x_f32, float* y, uint16_t* yh, const float* ple,
               int IN, int OUT, int epi, int ff, int off) {
  E4B_REQUIRE(c, c->ws && c->ws_bytes > 0, "q4_0 GEMV needs a workspace (e4b_set_workspace)");
  E4B_REQUIRE(c, q40_stream_supported(w, x, IN, OUT), "q4_0 stream GEMV: unsupported IN=%d", IN);
  Q40P p = {};
  p.x = x; p.y = y; p.yh = yh; p.ple = ple; p.status = c->status;
  p.IN = IN; p.OUT = OUT; p.nb = IN / 32; p.ff = ff; p.off = off; p.epi = epi;
  const int rowbytes = p.nb * 18;
  const int rows_total = epi == 1 ? 2 * ff : OUT;
  p.n_rt = epi == 1 ? (ff + 15) / 16 : (OUT + 31) / 32;
  p.qpr = p.nb / 8;
  const int64_t Q = (int64_t)p.n_rt * p.qpr;
  E4B_REQUIRE(c, Q < (1ll << 30), "q4_0 GEMV: matrix too large");
  p.Q = (int)Q;
  // workspace: [u32 counters | u64 start masks: kWsCounterBytes, zero at rest][split partials]
  const size_t need = kWsCounterBytes + (size_t)p.n_rt * p.qpr * 32 * 4;
  E4B_REQUIRE(c, p.n_rt <= (int)kWsMaxTiles, "q4_0 GEMV: %d tiles exceed the counter area", p.n_rt);
  E4B_REQUIRE(c, need <= c->ws_bytes, "workspace too small: need %zu bytes, have %zu", need, c->ws_bytes);
  p.ctr = reinterpret_cast<uint32_t*>(c->ws);
  p.starts = reinterpret_cast<unsigned long long*>(reinterpret_cast<uint8_t*>(c->ws) + kWsMaxTiles * 4);
  p.part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(c->ws) + kWsCounterBytes);

  // the weight tensor as 8-byte words: [rows_total][rowbytes / 8], boxes of 16 rows x 8 blocks
  CUtensorMap map;
  const cuuint64_t gdim[2] = {(cuuint64_t)(rowbytes / 8), (cuuint64_t)rows_total};
  const cuuint64_t gstride[1] = {(cuuint64_t)rowbytes};
  const cuuint32_t box[2] = {kRowPitch / 8, 16};
  const cuuint32_t estride[2] = {1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<uint8_t*>(w), gdim, gstride, box,
                           estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  E4B_REQUIRE(c, r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (%d) for IN=%d rows=%d", (int)r, IN, rows_total);
  if (x_f32) {
    if (epi == 0) return launch_variant<1, 0>(c, p, map, "q40mv_stream");
    if (epi == 1) return launch_variant<1, 1>(c, p, map, "q40gu_stream");
    return launch_variant<1, 2>(c, p, map, "plegate_stream");
  }
  if (epi == 0) return launch_variant<0, 0>(c, p, map, "q40mv_stream");
  if (epi == 1) return launch_variant<0, 1>(c, p, map, "q40gu_stream");
  return launch_variant<0, 2>(c, p, map, "plegate_stream");
}

}  // namespace e4b
