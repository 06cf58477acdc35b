/*
 * CPU ORACLE -- TEST INFRASTRUCTURE ONLY.  Scalar C restatement of the
 * reference's quantised matvecs, used by the numpy oracle (oracle/ops.py) as the
 * checker and as the timed CPU baseline.  Never linked into, or called by, the
 * product path.
 *
 *   q4_0 matvec: y[o] = sum_b d_b * sum_i (n_i - 8) * x_i   (kernels/q40mv.wgsl:21-54,
 *                nibble order: byte j low nibble = element j, high = element j+16,
 *                scripts/ternarize_a4b.py:80-87)
 *   q6_K matvec: y[o] = sum_b d * sum_s sc_s * sum_i (q_i - 32) * x_i
 *                (element/scale mapping kernels/q6k.wgsl:44-68, 75-127)
 *
 * Per-block sums are f32 (like the reference's per-lane block dot); the sum
 * over blocks is carried in f64, so the oracle is at least as exact as any
 * f32 GPU summation order it is compared with.
 */
#include <stdint.h>
#include <string.h>
#include <math.h>

static inline float f16_to_f32(uint16_t h) {
  uint32_t s = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu, bits;
  float f;
  if (e == 0) {
    f = (float)m * (1.0f / 16777216.0f);
    return (h & 0x8000u) ? -f : f;
  }
  if (e == 31) bits = s | 0x7F800000u | (m << 13);
  else bits = s | ((e + 112) << 23) | (m << 13);
  memcpy(&f, &bits, 4);
  return f;
}

static inline float q40_block_dot(const uint8_t* blk, const float* x) {
  float s = 0.0f;
  for (int j = 0; j < 16; j++) {
    int lo = blk[2 + j] & 0x0F, hi = blk[2 + j] >> 4;
    s += (float)(lo - 8) * x[j] + (float)(hi - 8) * x[j + 16];
  }
  uint16_t dh = (uint16_t)(blk[0] | (blk[1] << 8));
  return f16_to_f32(dh) * s;
}

void oracle_q40_matvec(const uint8_t* w, const float* x, float* y, int64_t rows, int64_t n_in) {
  int64_t nb = n_in / 32;
#pragma omp parallel for schedule(static)
  for (int64_t o = 0; o < rows; o++) {
    const uint8_t* row = w + o * nb * 18;
    double acc = 0.0;
    for (int64_t b = 0; b < nb; b++) acc += (double)q40_block_dot(row + b * 18, x + b * 32);
    y[o] = (float)acc;
  }
}

/* q6_K element e of a 210-byte block as (q - 32) and its sub-block scale index e/16. */
static inline int q6k_q(const uint8_t* blk, int e) {
  const uint8_t* ql = blk;
  const uint8_t* qh = blk + 128;
  int h = e / 128, r = e % 128, j = r / 32, l = r % 32;
  int lo = (ql[h * 64 + l + (j & 1) * 32] >> ((j >> 1) * 4)) & 0xF;
  int hb = (qh[h * 32 + l] >> (2 * j)) & 3;
  return (lo | (hb << 4)) - 32;
}

void oracle_q6k_matvec(const uint8_t* w, const float* x, float* y, int64_t rows, int64_t n_in) {
  int64_t nb = n_in / 256;
#pragma omp parallel for schedule(static)
  for (int64_t o = 0; o < rows; o++) {
    const uint8_t* row = w + o * nb * 210;
    double acc = 0.0;
    for (int64_t b = 0; b < nb; b++) {
      const uint8_t* blk = row + b * 210;
      const int8_t* sc = (const int8_t*)(blk + 192);
      float d = f16_to_f32((uint16_t)(blk[208] | (blk[209] << 8)));
      float bs = 0.0f;
      for (int s = 0; s < 16; s++) {
        float ss = 0.0f;
        for (int i = 0; i < 16; i++) ss += (float)q6k_q(blk, 16 * s + i) * x[b * 256 + 16 * s + i];
        bs += (float)sc[s] * ss;
      }
      acc += (double)(d * bs);
    }
    y[o] = (float)acc;
  }
}

/* Dequantise rows [r0, r0+n) of a q6_K matrix: v = ((d*sc)*(q-32))*mult (kernels/q6k.wgsl:64-67). */
void oracle_q6k_rows(const uint8_t* w, float* out, int64_t r0, int64_t n, int64_t n_in, float mult) {
  int64_t nb = n_in / 256;
  for (int64_t r = 0; r < n; r++) {
    const uint8_t* row = w + (r0 + r) * nb * 210;
    for (int64_t b = 0; b < nb; b++) {
      const uint8_t* blk = row + b * 210;
      const int8_t* sc = (const int8_t*)(blk + 192);
      float d = f16_to_f32((uint16_t)(blk[208] | (blk[209] << 8)));
      for (int e = 0; e < 256; e++) {
        float v = d * (float)sc[e / 16];
        v = v * (float)q6k_q(blk, e);
        out[r * n_in + b * 256 + e] = v * mult;
      }
    }
  }
}

int oracle_threads(void) {
#ifdef _OPENMP
  extern int omp_get_max_threads(void);
  return omp_get_max_threads();
#else
  return 1;
#endif
}
