/*
 * Synthetic-weight generator and GGUF block quantizers (host code, OpenMP).
 *
 * Builds the seeded synthetic models the decode path is measured on: weights are
 * N(0, std) fp32 drawn from a counter-based generator (element i of stream s
 * depends only on (seed, s, i), so the bytes do not depend on the thread count),
 * then quantised to GGUF block formats:
 *
 *   q4_0: 32 weights per 18-byte block = f16 d + 16 nibble bytes; byte j holds
 *         element j (low nibble) and element j+16 (high nibble); w = d*(n-8).
 *         Quantiser: the ggml reference rule (the published llama.cpp
 *         quantize_row_q4_0_ref; restated by the python `gguf` package as
 *         gguf.quants.Q4_0.quantize_blocks): d = m/-8 with m the element of
 *         largest magnitude, n = min(15, trunc(x/d + 8.5)).  Tests check this
 *         file against that package byte for byte.
 *   q6_K: 256 weights per 210-byte block = ql[128] qh[64] i8 sc[16] f16 d, with
 *         the ggml element order (reference restatement: kernels/q6k.wgsl:44-68,
 *         src/engine-a4b.js:43-73).  Quantiser: a plain max-abs rule per
 *         16-element sub-block (sub-scale = m/-32, super-scale d = max|sub|/127,
 *         int8 sub-scales, q = round(x/(d*sc)) clamped to [-32, 31]).  It is not
 *         llama.cpp's rmse-searching quantiser; any valid block decodes the same
 *         way, and only decoding is on the measured path.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stddef.h>

#ifdef _OPENMP
#include <omp.h>
#endif

static inline uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

/* Normal pair k of stream (seed, stream): Box-Muller on two 53-bit uniforms. */
static inline void normal_pair(uint64_t key, uint64_t k, double* z0, double* z1) {
  uint64_t h1 = splitmix64(key ^ splitmix64(2 * k));
  uint64_t h2 = splitmix64(key ^ splitmix64(2 * k + 1));
  double u1 = ((double)(h1 >> 11) + 1.0) * (1.0 / 9007199254740992.0); /* (0,1] */
  double u2 = (double)(h2 >> 11) * (1.0 / 9007199254740992.0);         /* [0,1) */
  double r = sqrt(-2.0 * log(u1));
  double a = 6.283185307179586 * u2;
  *z0 = r * cos(a);
  *z1 = r * sin(a);
}

static inline uint64_t stream_key(uint64_t seed, uint64_t stream) {
  return splitmix64(seed * 0xD1B54A32D192ED03ull ^ splitmix64(stream + 0x632BE59BD9B4E019ull));
}

static inline float gen_at(uint64_t key, uint64_t i, float std) {
  double z0, z1;
  normal_pair(key, i >> 1, &z0, &z1);
  return (float)((i & 1) ? z1 : z0) * std;
}

/* Elements [i0, i0+n) of a stream, n even and i0 even: one Box-Muller pair per
 * two elements (element 2k is the cosine half of pair k, 2k+1 the sine half). */
static inline void gen_block(uint64_t key, uint64_t i0, int n, float std, float* x) {
  for (int j = 0; j < n; j += 2) {
    double z0, z1;
    normal_pair(key, (i0 + (uint64_t)j) >> 1, &z0, &z1);
    x[j] = (float)z0 * std;
    x[j + 1] = (float)z1 * std;
  }
}

/* IEEE binary16 from binary32, round to nearest even (host side; no CUDA). */
static uint16_t f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) return (uint16_t)(sign | (ax > 0x7F800000u ? 0x7E00u : 0x7C00u));
  if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* rounds to inf */
  if (ax < 0x38800000u) {                                    /* subnormal half */
    if (ax < 0x33000000u) return (uint16_t)sign;             /* < 2^-25: zero */
    uint32_t e = ax >> 23;
    uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
    uint32_t shift = 126 - e; /* 14 + (113 - e) - ... : value = m * 2^(e-150) */
    /* target units of 2^-24: m * 2^(e-150+24) = m >> (126-e) */
    uint32_t q = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1u))) q++;
    return (uint16_t)(sign | q);
  }
  uint32_t e = (ax >> 23) - 112; /* rebias 127 -> 15 */
  uint32_t m = ax & 0x7FFFFFu;
  uint32_t q = (e << 10) | (m >> 13);
  uint32_t rem = m & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
  return (uint16_t)(sign | q);
}

/* ---- q4_0 ---- */
static void quant_q4_0_block(const float* x, uint8_t* out) {
  float amax = 0.0f, m = 0.0f;
  for (int j = 0; j < 32; j++) {
    float a = fabsf(x[j]);
    if (a > amax) { amax = a; m = x[j]; }
  }
  float d = m / -8.0f;
  float id = d != 0.0f ? 1.0f / d : 0.0f;
  uint16_t dh = f32_to_f16(d);
  out[0] = (uint8_t)(dh & 0xFF);
  out[1] = (uint8_t)(dh >> 8);
  for (int j = 0; j < 16; j++) {
    float v0 = truncf(x[j] * id + 8.5f);
    float v1 = truncf(x[j + 16] * id + 8.5f);
    int q0 = (int)v0, q1 = (int)v1;
    /* uint8 cast then clip(0,15), as the gguf package does */
    q0 = (uint8_t)q0; q1 = (uint8_t)q1;
    if (q0 > 15) q0 = 15;
    if (q1 > 15) q1 = 15;
    out[2 + j] = (uint8_t)(q0 | (q1 << 4));
  }
}

/* Quantise nblocks*32 floats into q4_0 blocks. */
void e4b_quant_q4_0(const float* x, uint8_t* out, int64_t nblocks) {
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nblocks; b++) quant_q4_0_block(x + b * 32, out + b * 18);
}

/* ---- q6_K ---- */
static inline int nearest_int(float v) { return (int)lrintf(v); }

static void quant_q6_K_block(const float* x, uint8_t* out) {
  float sub[16];
  float maxsub = 0.0f;
  for (int s = 0; s < 16; s++) {
    float amax = 0.0f, m = 0.0f;
    for (int j = 0; j < 16; j++) {
      float a = fabsf(x[16 * s + j]);
      if (a > amax) { amax = a; m = x[16 * s + j]; }
    }
    sub[s] = m / -32.0f;
    if (fabsf(sub[s]) > maxsub) maxsub = fabsf(sub[s]);
  }
  uint8_t* ql = out;
  uint8_t* qh = out + 128;
  int8_t* sc = (int8_t*)(out + 192);
  memset(out, 0, 210);
  if (maxsub == 0.0f) {
    /* all-zero block: d = 0, every q = 32 (zero point) */
    for (int e = 0; e < 256; e++) {
      int h = e / 128, r = e % 128, j = r / 32, l = r % 32;
      int q = 32;
      uint8_t* qlb = ql + h * 64 + l + (j & 1) * 32;
      *qlb |= (uint8_t)((q & 0xF) << ((j >> 1) * 4));
      qh[h * 32 + l] |= (uint8_t)((q >> 4) << (2 * j));
    }
    return;
  }
  float d = maxsub / 127.0f;
  uint16_t dh = f32_to_f16(d);
  /* decode the stored f16 so element quantisation uses the value kernels see */
  float dq;
  {
    uint32_t s = (dh & 0x8000u) << 16, e = (dh >> 10) & 0x1F, m = dh & 0x3FF, bits;
    if (e == 0) {
      float v = (float)m * (1.0f / 16777216.0f);
      dq = (dh & 0x8000u) ? -v : v;
    } else {
      bits = s | ((e + 112) << 23) | (m << 13);
      memcpy(&dq, &bits, 4);
    }
  }
  for (int s = 0; s < 16; s++) {
    int v = dq != 0.0f ? nearest_int(sub[s] / dq) : 0;
    if (v > 127) v = 127;
    if (v < -128) v = -128;
    sc[s] = (int8_t)v;
  }
  out[208] = (uint8_t)(dh & 0xFF);
  out[209] = (uint8_t)(dh >> 8);
  for (int e = 0; e < 256; e++) {
    int s = e / 16;
    float step = dq * (float)sc[s];
    int q = step != 0.0f ? nearest_int(x[e] / step) : 0;
    if (q > 31) q = 31;
    if (q < -32) q = -32;
    q += 32;
    int h = e / 128, r = e % 128, j = r / 32, l = r % 32;
    /* ql[h*64 + l (+32 for j odd)] holds j<2 in the low nibble, j>=2 in the high */
    uint8_t* qlb = ql + h * 64 + l + (j & 1) * 32;
    *qlb |= (uint8_t)((q & 0xF) << ((j >> 1) * 4));
    qh[h * 32 + l] |= (uint8_t)((q >> 4) << (2 * j));
  }
}

void e4b_quant_q6_K(const float* x, uint8_t* out, int64_t nblocks) {
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nblocks; b++) quant_q6_K_block(x + b * 256, out + b * 210);
}

/* ---- generators ---- */

/* n normals N(0, std) of stream (seed, stream) into out (f32). */
void e4b_synth_normal_f32(float* out, int64_t n, uint64_t seed, uint64_t stream, float std) {
  uint64_t key = stream_key(seed, stream);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; i++) out[i] = gen_at(key, (uint64_t)i, std);
}

/* Generate N(0, std) weights and quantise straight to q4_0 (no f32 buffer). */
void e4b_synth_q4_0(uint8_t* out, int64_t nblocks, uint64_t seed, uint64_t stream, float std) {
  uint64_t key = stream_key(seed, stream);
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nblocks; b++) {
    float x[32];
    gen_block(key, (uint64_t)b * 32, 32, std, x);
    quant_q4_0_block(x, out + b * 18);
  }
}

void e4b_synth_q6_K(uint8_t* out, int64_t nblocks, uint64_t seed, uint64_t stream, float std) {
  uint64_t key = stream_key(seed, stream);
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nblocks; b++) {
    float x[256];
    gen_block(key, (uint64_t)b * 256, 256, std, x);
    quant_q6_K_block(x, out + b * 210);
  }
}

int e4b_synth_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
