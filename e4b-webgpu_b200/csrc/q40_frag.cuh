// q4_0 tensor-core building blocks shared by the streaming GEMV kernel and the
// persistent decode kernel: the staged quantum layout, the A-operand nibble
// decode, the B-operand activation fragments, and one quantum's MMAs.
#pragma once

#include <cuda.h>

#include "stream.cuh"

namespace e4b {

constexpr int kRowPitch = 144;                     // 8 blocks x 18 B per staged row
constexpr int kSubBytes = 16 * kRowPitch;          // one TMA box: 16 rows x 8 blocks
constexpr int kQuantumBytes = 2 * kSubBytes;       // two 16-row subtiles

// ---- A operand: the 4 nibble bytes lane (g, t) owns of one block.
// Odd blocks (18b + 2 word aligned) give lane t the nibble bytes 4t..4t+3;
// even blocks are word aligned at the scale, so t<3 takes nibble bytes
// 2+4t..5+4t and t=3 the edge bytes {0,1,14,15} (PRMT of words 0 and 4).
struct Lane {
  int o_odd, o_e1;
  uint32_t sel;
};
E4B_DEV uint32_t nib_even(const uint8_t* blk, const Lane& L) {
  return __byte_perm(*reinterpret_cast<const uint32_t*>(blk + L.o_e1),
                     *reinterpret_cast<const uint32_t*>(blk + 16), L.sel);
}
E4B_DEV uint32_t nib_odd(const uint8_t* blk, const Lane& L) {
  return *reinterpret_cast<const uint32_t*>(blk + L.o_odd);
}
E4B_DEV uint32_t nib(const uint8_t* blk, int k, const Lane& L) {
  return (k & 1) ? nib_odd(blk, L) : nib_even(blk, L);
}

// A fragments of one row from its nibble bytes v = [B0 B1 B2 B3]:
//   low k-half: (B0, B2) -> k = 2t, 2t+1 ; (B1, B3) -> k = 2t+8, 2t+9
//   high k-half: the same with the high nibbles (elements 16 + j).
// f16 magic: 0x6400|n = 1024+n, minus 1032 -> n-8 ; 0x6400|n<<4 = 1024+16n, /16 - 72 -> n-8.
// (a & m) | c in one LOP3 (truth table 0xEA), whatever the compiler would make
// of the two constants.
E4B_DEV uint32_t and_or(uint32_t a, uint32_t m, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(m), "r"(c));
  return d;
}
E4B_DEV void dq_row(uint32_t v, uint32_t& lo02, uint32_t& lo13, uint32_t& hi02, uint32_t& hi13) {
  const uint32_t v8 = v >> 8;
  const uint32_t k1032 = 0x64086408u, kSixteenth = 0x2C002C00u, kM72 = 0xD480D480u, kMag = 0x64006400u;
  lo02 = hsub2(and_or(v, 0x000F000Fu, kMag), k1032);
  lo13 = hsub2(and_or(v8, 0x000F000Fu, kMag), k1032);
  hi02 = hfma2(and_or(v, 0x00F000F0u, kMag), kSixteenth, kM72);
  hi13 = hfma2(and_or(v8, 0x00F000F0u, kMag), kSixteenth, kM72);
}

// ---- tile-packed q4_0 (e4b_q40_pack_tiles): per 16 rows x 256 k one piece of
// kPkSub bytes, [16 rows][8 blocks] f16 scales then, as [block half][row][lane]
// uint4s, the 32-bit words nib() returns for lane t (word j: block 4 half + j).
constexpr int kPkSub = 2304;
E4B_DEV uint32_t u32w(const uint4& v, int j) { return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w; }

// ---- B operand: lane (g, t) supplies column g of B, i.e. the activations of
// block 8q+g of quantum q at the element indices its A fragments use: low half
// {j0, j2}, {j1, j3}; high half the same + 16.  A block's parity equals g's
// parity, so each lane's word offsets into the block's 32 f16 activations are
// fixed for the whole kernel:
//   odd g:  j = 4t..4t+3       -> words (2t, 2t+1)
//   even g: j = 2+4t..5+4t     -> words (1+2t, 2+2t) (t < 3); j = {0,1,14,15} -> words (0, 7)
// and the high half uses words + 8.
struct XLane {
  int wa, wb;        // word offsets of (j0 j1) and (j2 j3)
};
E4B_DEV XLane xlane(int g, int t) {
  XLane X;
  if (g & 1) {
    X.wa = 2 * t;
    X.wb = 2 * t + 1;
  } else if (t < 3) {
    X.wa = 1 + 2 * t;
    X.wb = 2 + 2 * t;
  } else {
    X.wa = 0;
    X.wb = 7;
  }
  return X;
}
// B registers {b0 lo, b1 lo, b0 hi, b1 hi} from f16 x for block `blk`.
E4B_DEV uint4 xfrag_f16(const uint16_t* x, int blk, const XLane& X) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(x + 32 * blk);
  const uint32_t a = __ldg(w + X.wa), b = __ldg(w + X.wb), ah = __ldg(w + 8 + X.wa), bh = __ldg(w + 8 + X.wb);
  // (j0 j1) (j2 j3) -> (j0 j2) (j1 j3)
  return make_uint4(__byte_perm(a, b, 0x5410), __byte_perm(a, b, 0x7632), __byte_perm(ah, bh, 0x5410),
                    __byte_perm(ah, bh, 0x7632));
}
// f32 x split into f16 hi + f16 lo (x = hi + lo to ~22 bits): two uint4.
E4B_DEV void xfrag_f32(const float* x, int blk, const XLane& X, uint4& hi, uint4& lo) {
  const float* b = x + 32 * blk;
  const int idx[8] = {2 * X.wa, 2 * X.wb, 2 * X.wa + 1, 2 * X.wb + 1,
                      16 + 2 * X.wa, 16 + 2 * X.wb, 16 + 2 * X.wa + 1, 16 + 2 * X.wb + 1};
  uint16_t h[8], l[8];
#pragma unroll
  for (int k = 0; k < 8; k++) {
    const float v = __ldg(b + idx[k]);
    const __half hh = __float2half_rn(v);
    h[k] = __half_as_ushort(hh);
    l[k] = f2h(v - __half2float(hh));
  }
  hi = make_uint4(pack_h2(h[0], h[1]), pack_h2(h[2], h[3]), pack_h2(h[4], h[5]), pack_h2(h[6], h[7]));
  lo = make_uint4(pack_h2(l[0], l[1]), pack_h2(l[2], l[3]), pack_h2(l[4], l[5]), pack_h2(l[6], l[7]));
}
// The same fragments read through a generic pointer (shared or global memory).
E4B_DEV uint4 xfrag_f16_any(const uint16_t* x, int blk, const XLane& X) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(x + 32 * blk);
  const uint32_t a = w[X.wa], b = w[X.wb], ah = w[8 + X.wa], bh = w[8 + X.wb];
  return make_uint4(__byte_perm(a, b, 0x5410), __byte_perm(a, b, 0x7632), __byte_perm(ah, bh, 0x5410),
                    __byte_perm(ah, bh, 0x7632));
}
E4B_DEV void xfrag_f32_any(const float* x, int blk, const XLane& X, uint4& hi, uint4& lo) {
  const float* b = x + 32 * blk;
  const int idx[8] = {2 * X.wa, 2 * X.wb, 2 * X.wa + 1, 2 * X.wb + 1,
                      16 + 2 * X.wa, 16 + 2 * X.wb, 16 + 2 * X.wa + 1, 16 + 2 * X.wb + 1};
  uint16_t h[8], l[8];
#pragma unroll
  for (int k = 0; k < 8; k++) {
    const float v = b[idx[k]];
    const __half hh = __float2half_rn(v);
    h[k] = __half_as_ushort(hh);
    l[k] = f2h(v - __half2float(hh));
  }
  hi = make_uint4(pack_h2(h[0], h[1]), pack_h2(h[2], h[3]), pack_h2(h[4], h[5]), pack_h2(h[6], h[7]));
  lo = make_uint4(pack_h2(l[0], l[1]), pack_h2(l[2], l[3]), pack_h2(l[4], l[5]), pack_h2(l[6], l[7]));
}

template <int XF32>
E4B_DEV void xfrag(const void* x, int blk, const XLane& X, uint4& hi, uint4& lo) {
  if (XF32) {
    xfrag_f32(reinterpret_cast<const float*>(x), blk, X, hi, lo);
  } else {
    hi = xfrag_f16(reinterpret_cast<const uint16_t*>(x), blk, X);
    lo = make_uint4(0, 0, 0, 0);
  }
}

E4B_DEV void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// One quantum (8 blocks x 32 rows) at `q`; xs_g is the lane's x fragment.
template <int XF32>
E4B_DEV void quantum_mma(const uint8_t* q, const uint4 xh, const uint4 xl, const Lane& L, int g, int t,
                         float (&acc)[4]) {
  const uint8_t* r0 = q + g * kRowPitch;            // subtile 0, row g
  const uint8_t* r1 = r0 + 8 * kRowPitch;           // subtile 0, row g+8
  const uint8_t* r2 = r0 + kSubBytes;               // subtile 1, row g
  const uint8_t* r3 = r1 + kSubBytes;               // subtile 1, row g+8
  float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};   // subtile 0: low / high k-half
  float c2[4] = {0.f, 0.f, 0.f, 0.f}, c3[4] = {0.f, 0.f, 0.f, 0.f};   // subtile 1
#pragma unroll
  for (int k = 0; k < 8; k++) {
    uint32_t A[16];
    dq_row(nib(r0 + 18 * k, k, L), A[0], A[1], A[2], A[3]);
    dq_row(nib(r1 + 18 * k, k, L), A[4], A[5], A[6], A[7]);
    dq_row(nib(r2 + 18 * k, k, L), A[8], A[9], A[10], A[11]);
    dq_row(nib(r3 + 18 * k, k, L), A[12], A[13], A[14], A[15]);
    const bool mine = g == k;
    const uint32_t b0 = mine ? xh.x : 0u, b1 = mine ? xh.y : 0u, b2 = mine ? xh.z : 0u, b3 = mine ? xh.w : 0u;
    mma16816(c0, A[0], A[4], A[1], A[5], b0, b1);
    mma16816(c2, A[8], A[12], A[9], A[13], b0, b1);
    mma16816(c1, A[2], A[6], A[3], A[7], b2, b3);
    mma16816(c3, A[10], A[14], A[11], A[15], b2, b3);
    if (XF32) {
      const uint32_t l0 = mine ? xl.x : 0u, l1 = mine ? xl.y : 0u, l2 = mine ? xl.z : 0u, l3 = mine ? xl.w : 0u;
      mma16816(c0, A[0], A[4], A[1], A[5], l0, l1);
      mma16816(c2, A[8], A[12], A[9], A[13], l0, l1);
      mma16816(c1, A[2], A[6], A[3], A[7], l2, l3);
      mma16816(c3, A[10], A[14], A[11], A[15], l2, l3);
    }
  }
  // C cols 2t, 2t+1 = blocks 2t, 2t+1 of the group; c[0], c[1] row g, c[2], c[3] row g+8
  const uint8_t* rr[4] = {r0, r1, r2, r3};
  float d[8];
#pragma unroll
  for (int r = 0; r < 4; r++) {
    d[2 * r] = h2f(*reinterpret_cast<const uint16_t*>(rr[r] + 36 * t));
    d[2 * r + 1] = h2f(*reinterpret_cast<const uint16_t*>(rr[r] + 36 * t + 18));
  }
  acc[0] = fmaf(d[0], c0[0] + c1[0], fmaf(d[1], c0[1] + c1[1], acc[0]));
  acc[1] = fmaf(d[2], c0[2] + c1[2], fmaf(d[3], c0[3] + c1[3], acc[1]));
  acc[2] = fmaf(d[4], c2[0] + c3[0], fmaf(d[5], c2[1] + c3[1], acc[2]));
  acc[3] = fmaf(d[6], c2[2] + c3[2], fmaf(d[7], c2[3] + c3[3], acc[3]));
}

}  // namespace e4b
