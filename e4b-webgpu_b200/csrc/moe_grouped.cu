// Grouped MoE for batched decode (kernels/expgroup.wgsl, q40gugrp.wgsl,
// q40downgrp.wgsl, wacc.wgsl): the B x K (token, slot) routing entries are
// sorted by expert, each expert's weights are read once for all the tokens
// routed to it, and the per-entry outputs are combined per token in slot order.
//
// GEMM formulation: an expert's rows x its tokens on the tensor cores
// (mma.sync m16n8k16, f16 x f16 -> f32), tokens as the 8 columns of B.  A q4_0
// block's scale multiplies all of that block's products, so each block is one
// K-step with its own accumulator that is scaled in f32 and added, keeping the
// reference's arithmetic (d * sum (n-8) x per block, f32 sums) exactly as the
// single-token kernels do.  Warps of a CTA split the blocks of the row and
// reduce through shared memory.
#include "q40_frag.cuh"

namespace {
using namespace e4b;

constexpr int kGW = 4;          // warps per CTA
constexpr int kGroups = 8;      // 8-token groups per pass (64 tokens)

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
  if (threadIdx.x == 0 && cnt[E] != (uint32_t)n) set_status(status, E4B_ST_BADINDEX);   // expert id out of range
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

// ---- grouped q4_0 GEMM: rows of expert e x the tokens routed to it.
// EPI 0: y[pos][row] = W_e x_token (f32); EPI 1: rows [gate FF | up FF] ->
// yh[pos][o] = f16(gelu(gate_o) * up_o).  Tile = 32 rows (EPI 1: 16 gate + 16 up).
// XPOS: x row of entry p is x[entries[p] / K] (token rows) or x[p] (entry rows).
template <int EPI, int XPOS>
__global__ void __launch_bounds__(32 * kGW) k_grp(const uint16_t* __restrict__ x, const uint8_t* __restrict__ w,
                                                   const uint32_t* __restrict__ offsets,
                                                   const uint32_t* __restrict__ entries, float* __restrict__ y,
                                                   uint16_t* __restrict__ yh, int IN, int ROWS, int FF, int K,
                                                   int n_direct) {
  pdl_wait();
  __shared__ float red[kGW][32][kGroups * 8];
  const int e = blockIdx.y, tile = blockIdx.x;
  // n_direct > 0: one matrix, tokens 0..n_direct-1 in order (dense batched GEMM)
  const uint32_t p0 = n_direct > 0 ? 0u : offsets[e], ne = n_direct > 0 ? (uint32_t)n_direct : offsets[e + 1] - p0;
  if (ne == 0) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int nb = IN >> 5;
  const size_t rowbytes = (size_t)nb * 18;
  const uint8_t* we = w + (size_t)e * ROWS * rowbytes;
  // this lane's rows: subtile s, row g (+8)
  int rows[2][2];
  for (int s = 0; s < 2; s++) {
    const int base = EPI == 1 ? (s == 0 ? 16 * tile : FF + 16 * tile) : 32 * tile + 16 * s;
    rows[s][0] = base + g;
    rows[s][1] = base + g + 8;
  }
  Lane L;
  L.o_odd = 2 + 4 * t;
  L.o_e1 = t < 3 ? 4 + 4 * t : 0;
  L.sel = t < 3 ? 0x3210u : 0x5432u;
  // B holds tokens as columns, so its element order follows the block's parity
  // (the A nibble layout), not the column index
  const XLane Xe = xlane(0, t), Xo = xlane(1, t);
  for (uint32_t pass = 0; pass < ne; pass += kGroups * 8) {
    const int ng = (int)min((uint32_t)kGroups, (ne - pass + 7) / 8);
    // this lane's token (column g) of every group
    const uint16_t* xr[kGroups];
#pragma unroll
    for (int q = 0; q < kGroups; q++) {
      const uint32_t j = pass + 8 * q + g;
      xr[q] = nullptr;
      if (q < ng && j < ne) xr[q] = x + (size_t)(XPOS ? p0 + j : entries[p0 + j] / (uint32_t)K) * IN;
    }
    float acc[kGroups][2][4];
#pragma unroll
    for (int q = 0; q < kGroups; q++)
#pragma unroll
      for (int s = 0; s < 2; s++)
#pragma unroll
        for (int r = 0; r < 4; r++) acc[q][s][r] = 0.f;
    for (int b = warp; b < nb; b += kGW) {
      uint32_t A[2][8];
      float d[2][2];
#pragma unroll
      for (int s = 0; s < 2; s++)
#pragma unroll
        for (int h = 0; h < 2; h++) {
          const int row = rows[s][h];
          if (row < ROWS) {   // rows beyond the matrix read as zero
            const uint8_t* blk = we + (size_t)row * rowbytes + (size_t)b * 18;
            dq_row(nib(blk, b, L), A[s][4 * h], A[s][4 * h + 1], A[s][4 * h + 2], A[s][4 * h + 3]);
            d[s][h] = h2f(__ldg(reinterpret_cast<const uint16_t*>(we + (size_t)row * rowbytes + (size_t)b * 18)));
          } else {
            A[s][4 * h] = A[s][4 * h + 1] = A[s][4 * h + 2] = A[s][4 * h + 3] = 0u;
            d[s][h] = 0.f;
          }
        }
      // the block's scales of the rows this lane's C fragment holds (rows g, g+8)
#pragma unroll
      for (int q = 0; q < kGroups; q++) {
        if (q >= ng) break;
        const uint4 xb = xr[q] ? xfrag_f16(xr[q], b, (b & 1) ? Xo : Xe) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int s = 0; s < 2; s++) {
          float c[4] = {0.f, 0.f, 0.f, 0.f};
          // A regs: [row g: lo02, lo13, hi02, hi13 | row g+8: ...]
          mma16816(c, A[s][0], A[s][4], A[s][1], A[s][5], xb.x, xb.y);
          mma16816(c, A[s][2], A[s][6], A[s][3], A[s][7], xb.z, xb.w);
          acc[q][s][0] = fmaf(d[s][0], c[0], acc[q][s][0]);
          acc[q][s][1] = fmaf(d[s][0], c[1], acc[q][s][1]);
          acc[q][s][2] = fmaf(d[s][1], c[2], acc[q][s][2]);
          acc[q][s][3] = fmaf(d[s][1], c[3], acc[q][s][3]);
        }
      }
    }
    // reduce the warps' block subsets (fixed order)
#pragma unroll
    for (int q = 0; q < kGroups; q++)
#pragma unroll
      for (int s = 0; s < 2; s++)
#pragma unroll
        for (int r = 0; r < 4; r++) red[warp][lane][q * 8 + s * 4 + r] = acc[q][s][r];
    __syncthreads();
    for (int i = threadIdx.x; i < 32 * ng * 8; i += blockDim.x) {
      const int ln = i / (ng * 8), k = i % (ng * 8);
      float v = 0.f;
      for (int ww = 0; ww < kGW; ww++) v += red[ww][ln][k];
      red[0][ln][k] = v;
    }
    __syncthreads();
    // C layout: c0, c1 = row g, columns 2t, 2t+1; c2, c3 = row g+8
    for (int i = threadIdx.x; i < 32 * ng; i += blockDim.x) {
      const int ln = i % 32, q = i / 32, gg = ln >> 2, tt = ln & 3;
      const float* v = red[0][ln] + q * 8;
      for (int col = 0; col < 2; col++) {
        const uint32_t j = pass + 8 * q + 2 * tt + col;
        if (j >= ne) continue;
        const uint32_t pos = p0 + j;
        for (int h = 0; h < 2; h++) {
          const float a0 = v[0 * 4 + 2 * h + col], a1 = v[1 * 4 + 2 * h + col];
          if (EPI == 1) {
            const int o = 16 * tile + gg + 8 * h;
            if (o < FF) yh[(size_t)pos * FF + o] = f2h(gelu_tanh(a0) * a1);
          } else {
            const int r0 = 32 * tile + gg + 8 * h, r1 = r0 + 16;
            if (r0 < ROWS) y[(size_t)pos * ROWS + r0] = a0;
            if (r1 < ROWS) y[(size_t)pos * ROWS + r1] = a1;
          }
        }
      }
    }
    __syncthreads();
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

}  // namespace

extern "C" {

E4B_API int e4b_expgroup(e4b_ctx* c, const uint32_t* topk, int n_tok, int K, int E, uint32_t* offsets,
                         uint32_t* entries, uint32_t* inv) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, topk && offsets && entries && inv, "expgroup: null buffer");
  E4B_REQUIRE(c, n_tok > 0 && K > 0 && E > 0 && E <= 4096 && (long long)n_tok * K < (1ll << 24),
              "expgroup: bad sizes n=%d K=%d E=%d", n_tok, K, E);
  return e4b_launch(c, "expgroup", k_expgroup, dim3(1), dim3(1024), (size_t)(E + 1) * 4, topk, n_tok * K, E, offsets,
                    entries, inv, c->status);
}

E4B_API int e4b_q40gugrp(e4b_ctx* c, const uint16_t* x, const uint8_t* w, const uint32_t* offsets,
                         const uint32_t* entries, uint16_t* yh, int IN, int FF, int E, int K) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, x && w && offsets && entries && yh, "q40gugrp: null buffer");
  E4B_REQUIRE(c, IN > 0 && IN % 32 == 0 && FF > 0 && E > 0 && K > 0, "q40gugrp: bad sizes IN=%d FF=%d", IN, FF);
  E4B_REQUIRE(c, reinterpret_cast<uintptr_t>(w) % 4 == 0 && (IN / 32) % 2 == 0,
              "q40gugrp: IN/32 must be even (rows on 4-byte boundaries, word reads inside each row)");
  return e4b_launch(c, "q40gugrp", k_grp<1, 0>, dim3((FF + 15) / 16, E), dim3(32 * kGW), 0, x, w, offsets, entries,
                    (float*)nullptr, yh, IN, 2 * FF, FF, K, 0);
}

E4B_API int e4b_q40downgrp(e4b_ctx* c, const uint16_t* x, const uint8_t* w, const uint32_t* offsets,
                           const uint32_t* entries, float* y, int IN, int OUT, int E) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, x && w && offsets && entries && y, "q40downgrp: null buffer");
  E4B_REQUIRE(c, IN > 0 && IN % 32 == 0 && OUT > 0 && E > 0, "q40downgrp: bad sizes IN=%d OUT=%d", IN, OUT);
  E4B_REQUIRE(c, reinterpret_cast<uintptr_t>(w) % 4 == 0 && (IN / 32) % 2 == 0,
              "q40downgrp: IN/32 must be even (rows on 4-byte boundaries, word reads inside each row)");
  return e4b_launch(c, "q40downgrp", k_grp<0, 1>, dim3((OUT + 31) / 32, E), dim3(32 * kGW), 0, x, w, offsets,
                    entries, y, (uint16_t*)nullptr, IN, OUT, 0, 1, 0);
}

E4B_API int e4b_q40mm(e4b_ctx* c, const uint16_t* x, const uint8_t* w, float* y, int IN, int OUT, int n) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, x && w && y && n > 0, "q40mm: bad args");
  E4B_REQUIRE(c, IN > 0 && IN % 64 == 0 && OUT > 0 && reinterpret_cast<uintptr_t>(w) % 4 == 0,
              "q40mm: IN=%d must be a multiple of 64", IN);
  return e4b_launch(c, "q40mm", k_grp<0, 1>, dim3((OUT + 31) / 32, 1), dim3(32 * kGW), 0, x, w,
                    (const uint32_t*)nullptr, (const uint32_t*)nullptr, y, (uint16_t*)nullptr, IN, OUT, 0, 1, n);
}

E4B_API int e4b_q40gumm(e4b_ctx* c, const uint16_t* x, const uint8_t* w, uint16_t* yh, int IN, int FF, int n) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, x && w && yh && n > 0, "q40gumm: bad args");
  E4B_REQUIRE(c, IN > 0 && IN % 64 == 0 && FF > 0 && reinterpret_cast<uintptr_t>(w) % 4 == 0,
              "q40gumm: IN=%d must be a multiple of 64", IN);
  return e4b_launch(c, "q40gumm", k_grp<1, 1>, dim3((FF + 15) / 16, 1), dim3(32 * kGW), 0, x, w,
                    (const uint32_t*)nullptr, (const uint32_t*)nullptr, (float*)nullptr, yh, IN, 2 * FF, FF, 1, n);
}

E4B_API int e4b_wacc(e4b_ctx* c, const float* y, const uint32_t* inv, const float* topk_w, float* out, int n_tok,
                     int K, int OUT) {
  E4B_CHECK_CTX(c);
  E4B_REQUIRE(c, y && inv && topk_w && out && n_tok > 0 && K > 0 && OUT > 0, "wacc: bad args");
  return e4b_launch(c, "wacc", k_wacc, dim3((OUT + 255) / 256, n_tok), dim3(256), 0, y, inv, topk_w, out, n_tok, K,
                    OUT);
}

}  // extern "C"
