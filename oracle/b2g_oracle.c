/*
 * b2g_oracle.c -- TEST INFRASTRUCTURE ONLY.  CPU restatement of the GEMM path,
 * used as the parity checker in tests/ and as the timed CPU baseline in
 * bench.py.  The product library (libb2g) never links, loads or calls it.
 *
 * Parity status: the reference computes no observable GEMM output (its MMA
 * loops never read TMEM back, umma_throughput/umma_tput.cu:491-522) and zero-
 * fills its only real GEMM (cutlass_gemm_mainloop/cutlass_gemm_bench.cu:69-73),
 * so GEMM values are parity unpinned against the reference.  Pinned against the
 * reference: the 2:4 metadata nibble for kept indices {0,1}, 0x4 per group,
 * i.e. the word 0x44444444 (tcgen05_sparse_mma/tcgen05_sparse_mma.cu:331), and
 * the operand layouts (cutlass_gemm_bench.cu:78-80: A row-major, B column-major).
 * Codecs follow the OCP 8-bit floating point spec (E4M3 "fn": max 448, no inf;
 * E5M2: max finite 57344) and the OCP MX v1.0 E2M1 element type; rounding is
 * round-to-nearest-even with saturation to the largest finite value, the
 * semantics of PTX cvt.rn.satfinite.  int8 rounds to nearest even and
 * saturates; tf32 keeps 10 mantissa bits (nearest even) in fp32 storage.
 */
#include "b2g_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ */
/* generator                                                           */
/* ------------------------------------------------------------------ */
uint64_t orc_hash(uint64_t seed, uint64_t counter) {
  uint64_t z = seed + (counter + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

float orc_uniform(uint64_t seed, uint64_t counter) {
  int64_t u = (int64_t)(orc_hash(seed, counter) >> 40); /* 24 bits */
  return (float)(2 * u - (1ll << 24)) * 0x1p-24f;       /* exact */
}

float orc_normal(uint64_t seed, uint64_t counter) {
  int64_t s = 0;
  for (int i = 0; i < 6; ++i) {
    uint64_t h = orc_hash(seed ^ 0x6A09E667F3BCC909ull, counter * 6 + (uint64_t)i);
    s += (int64_t)(h >> 40);
    s += (int64_t)((h >> 16) & 0xFFFFFF);
  }
  return (float)((double)(s - 6 * (1ll << 24)) * 0x1p-24);
}

void orc_fill(float* out, int64_t r0, int64_t nrows, int64_t cols, uint64_t seed, int dist) {
  for (int64_t r = 0; r < nrows; ++r)
    for (int64_t c = 0; c < cols; ++c) {
      uint64_t ctr = (uint64_t)(r0 + r) * (uint64_t)cols + (uint64_t)c;
      out[r * cols + c] = dist ? orc_normal(seed, ctr) : orc_uniform(seed, ctr);
    }
}

/* ------------------------------------------------------------------ */
/* codecs                                                              */
/* ------------------------------------------------------------------ */
static uint32_t f2u(float x) { uint32_t u; memcpy(&u, &x, 4); return u; }
static float u2f(uint32_t u) { float x; memcpy(&x, &u, 4); return x; }

uint16_t orc_f32_to_bf16(float x) {
  uint32_t u = f2u(x);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FC0; /* NaN */
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

float orc_bf16_to_f32(uint16_t b) { return u2f((uint32_t)b << 16); }

/* Generic small-float encoder: e_bits exponent bits, m_bits mantissa bits,
 * exponent bias `bias`, largest finite magnitude `maxv`.  Round to nearest
 * even on the value grid, saturate to maxv.  Returns sign|exp|mant code. */
static uint32_t encode_small(float x, int m_bits, int bias, float maxv, int sign_shift) {
  uint32_t sign = (f2u(x) >> 31) & 1u;
  float a = fabsf(x);
  if (a > maxv) a = maxv;
  const int emin = 1 - bias; /* exponent of the smallest normal */
  int e;
  frexpf(a, &e); /* a = f * 2^e, f in [0.5,1) */
  int exp_unb = e - 1;
  if (a == 0.0f || exp_unb < emin) exp_unb = emin; /* subnormal grid */
  float ulp = ldexpf(1.0f, exp_unb - m_bits);
  float q = nearbyintf(a / ulp); /* exact power-of-two scale, RNE */
  float v = q * ulp;
  if (v > maxv) v = maxv;
  /* re-encode v */
  uint32_t code;
  if (v == 0.0f) {
    code = 0;
  } else {
    int ev;
    frexpf(v, &ev);
    int eu = ev - 1;
    if (eu < emin) { /* subnormal */
      code = (uint32_t)(v / ldexpf(1.0f, emin - m_bits));
    } else {
      uint32_t mant = (uint32_t)(v / ldexpf(1.0f, eu - m_bits)) - (1u << m_bits);
      code = ((uint32_t)(eu + bias) << m_bits) | mant;
    }
  }
  return code | (sign << sign_shift);
}

uint8_t orc_f32_to_e4m3(float x) {
  if (isnan(x)) return 0x7F;
  return (uint8_t)encode_small(x, 3, 7, 448.0f, 7);
}

float orc_e4m3_to_f32(uint8_t b) {
  int s = b >> 7, e = (b >> 3) & 0xF, m = b & 7;
  if (e == 0xF && m == 7) return NAN;
  float v = e ? ldexpf(1.0f + m / 8.0f, e - 7) : ldexpf(m / 8.0f, -6);
  return s ? -v : v;
}

uint8_t orc_f32_to_e2m1(float x) {
  if (isnan(x)) return 0x7; /* e2m1 has no NaN; satfinite maps it to max */
  return (uint8_t)encode_small(x, 1, 1, 6.0f, 3);
}

float orc_e2m1_to_f32(uint8_t code) {
  static const float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
  float v = mag[code & 7];
  return (code & 8) ? -v : v;
}

/* OCP 8-bit E5M2: 1-5-2, bias 15, IEEE-like (inf / NaN at exponent 31); the
 * saturating conversion maps everything above 57344 to 57344. */
uint8_t orc_f32_to_e5m2(float x) {
  if (isnan(x)) return 0x7F;
  return (uint8_t)encode_small(x, 2, 15, 57344.0f, 7);
}

float orc_e5m2_to_f32(uint8_t b) {
  int s = b >> 7, e = (b >> 2) & 0x1F, m = b & 3;
  float v;
  if (e == 0x1F) v = m ? NAN : INFINITY;
  else v = e ? ldexpf(1.0f + m / 4.0f, e - 15) : ldexpf(m / 4.0f, -14);
  return s ? -v : v;
}

/* int8: round to nearest even, saturate to [-128, 127]. */
int8_t orc_f32_to_s8(float x) {
  float r = nearbyintf(x); /* default rounding mode: nearest even */
  if (r < -128.0f) r = -128.0f;
  if (r > 127.0f) r = 127.0f;
  return (int8_t)r;
}

/* uint8: round to nearest even, saturate to [0, 255]. */
uint8_t orc_f32_to_u8(float x) {
  float r = nearbyintf(x);
  if (r < 0.0f) r = 0.0f;
  if (r > 255.0f) r = 255.0f;
  return (uint8_t)r;
}

/* IEEE binary16 from its definition: 1-5-10, bias 15; round to nearest even,
 * overflow to infinity. */
uint16_t orc_f32_to_f16(float x) {
  uint32_t u = f2u(x);
  uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
  float a = fabsf(x);
  if (isnan(x)) return (uint16_t)(sign | 0x7E00u);
  if (a >= 65520.0f) return (uint16_t)(sign | 0x7C00u); /* rounds past 65504 */
  int e;
  frexpf(a, &e);
  int eu = e - 1;
  if (a == 0.0f || eu < -14) eu = -14; /* subnormal grid: ulp 2^-24 */
  float ulp = ldexpf(1.0f, eu - 10);
  float q = nearbyintf(a / ulp);
  float v = q * ulp;
  if (v == 0.0f) return sign;
  frexpf(v, &e);
  eu = e - 1;
  uint16_t code;
  if (eu < -14) code = (uint16_t)(v / ldexpf(1.0f, -24));
  else code = (uint16_t)(((eu + 15) << 10) | ((uint32_t)(v / ldexpf(1.0f, eu - 10)) - 1024u));
  return (uint16_t)(sign | code);
}

float orc_f16_to_f32(uint16_t h) {
  int s = h >> 15, e = (h >> 10) & 0x1F, m = h & 0x3FF;
  float v;
  if (e == 0x1F) v = m ? NAN : INFINITY;
  else v = e ? ldexpf(1.0f + m / 1024.0f, e - 15) : ldexpf((float)m, -24);
  return s ? -v : v;
}

/* tf32 as stored in fp32: 10 mantissa bits, round to nearest even, low 13 bits
 * zero (inf / NaN truncated). */
float orc_f32_to_tf32(float x) {
  uint32_t u = f2u(x);
  if ((u & 0x7F800000u) == 0x7F800000u) return u2f(u & 0xFFFFE000u);
  return u2f((u + 0xFFFu + ((u >> 13) & 1u)) & 0xFFFFE000u);
}

/* OCP MX v1.0 FP6 element types (no inf / NaN): E2M3 = 1-2-3, bias 1, largest
 * 7.5; E3M2 = 1-3-2, bias 3, largest 28.  6-bit codes sign|exp|mant. */
uint8_t orc_f32_to_e2m3(float x) {
  if (isnan(x)) return 0x1F;
  return (uint8_t)encode_small(x, 3, 1, 7.5f, 5);
}

float orc_e2m3_to_f32(uint8_t c) {
  int s = (c >> 5) & 1, e = (c >> 3) & 3, m = c & 7;
  float v = e ? ldexpf(1.0f + m / 8.0f, e - 1) : m / 8.0f;
  return s ? -v : v;
}

uint8_t orc_f32_to_e3m2(float x) {
  if (isnan(x)) return 0x1F;
  return (uint8_t)encode_small(x, 2, 3, 28.0f, 5);
}

float orc_e3m2_to_f32(uint8_t c) {
  int s = (c >> 5) & 1, e = (c >> 2) & 7, m = c & 3;
  float v = e ? ldexpf(1.0f + m / 4.0f, e - 3) : ldexpf(m / 4.0f, -2);
  return s ? -v : v;
}

/* Sub-byte elements of kind::f8f6f4, packed along each row in groups of 16:
 * elem 0 e2m1 (8 bytes per group, element i at bits [4i, 4i+4)), 1 e2m3 and
 * 2 e3m2 (12 bytes per group, element i at bits [6i, 6i+6)), little-endian.
 * n % 16 == 0. */
void orc_quant_sub(const float* in, int64_t n, int elem, uint8_t* out, float* out_deq) {
  const int bits = elem == 0 ? 4 : 6;
  memset(out, 0, (size_t)(n / 16) * (size_t)(2 * bits));
  for (int64_t i = 0; i < n; ++i) {
    uint32_t c;
    float d;
    if (elem == 0) {
      c = orc_f32_to_e2m1(in[i]);
      d = orc_e2m1_to_f32((uint8_t)c);
    } else if (elem == 1) {
      c = orc_f32_to_e2m3(in[i]);
      d = orc_e2m3_to_f32((uint8_t)c);
    } else {
      c = orc_f32_to_e3m2(in[i]);
      d = orc_e3m2_to_f32((uint8_t)c);
    }
    const uint64_t bit = (uint64_t)i * (uint64_t)bits; /* groups of 16 tile the row exactly */
    for (int b = 0; b < bits; ++b)
      if ((c >> b) & 1u) out[(bit + b) >> 3] |= (uint8_t)(1u << ((bit + b) & 7));
    if (out_deq) out_deq[i] = d;
  }
}

/* Element-wise conversion without scale factors: elem 0 int8, 1 tf32 (4-byte
 * fp32 storage), 2 e5m2 (1 byte), 3 uint8, 4 fp16 (2 bytes).  out_deq receives
 * the values the MMA reads. */
void orc_quant_elem(const float* in, int64_t n, int elem, void* out, float* out_deq) {
  for (int64_t i = 0; i < n; ++i) {
    float d;
    if (elem == 0) {
      int8_t q = orc_f32_to_s8(in[i]);
      ((int8_t*)out)[i] = q;
      d = (float)q;
    } else if (elem == 1) {
      d = orc_f32_to_tf32(in[i]);
      ((float*)out)[i] = d;
    } else if (elem == 2) {
      uint8_t q = orc_f32_to_e5m2(in[i]);
      ((uint8_t*)out)[i] = q;
      d = orc_e5m2_to_f32(q);
    } else if (elem == 3) {
      uint8_t q = orc_f32_to_u8(in[i]);
      ((uint8_t*)out)[i] = q;
      d = (float)q;
    } else {
      uint16_t q = orc_f32_to_f16(in[i]);
      ((uint16_t*)out)[i] = q;
      d = orc_f16_to_f32(q);
    }
    if (out_deq) out_deq[i] = d;
  }
}

void orc_quant_bf16(const float* in, int64_t n, uint16_t* out, float* out_deq) {
  for (int64_t i = 0; i < n; ++i) {
    uint16_t b = orc_f32_to_bf16(in[i]);
    if (out) out[i] = b;
    if (out_deq) out_deq[i] = orc_bf16_to_f32(b);
  }
}

void orc_quant_e4m3(const float* in, int64_t n, uint8_t* out, float* out_deq) {
  for (int64_t i = 0; i < n; ++i) {
    uint8_t b = orc_f32_to_e4m3(in[i]);
    if (out) out[i] = b;
    if (out_deq) out_deq[i] = orc_e4m3_to_f32(b);
  }
}

void orc_quant_nvfp4(const float* in, int64_t rows, int64_t cols, uint8_t* out_packed,
                     uint8_t* out_sf, float* out_deq) {
  orc_quant_nvfp4_block(in, rows, cols, 16, out_packed, out_sf, out_deq);
}

/* One ue4m3 scale e4m3(amax / 6) per `block` elements (16, NVFP4; 32, the block of the
 * 4:8-sparse NVFP4 GEMM), each element e2m1(x / scale), packed two per byte with the
 * even index in the low nibble. */
void orc_quant_nvfp4_block(const float* in, int64_t rows, int64_t cols, int block,
                           uint8_t* out_packed, uint8_t* out_sf, float* out_deq) {
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t b = 0; b < cols / block; ++b) {
      const float* x = in + r * cols + b * block;
      float amax = 0.0f;
      for (int i = 0; i < block; ++i) amax = fmaxf(amax, fabsf(x[i]));
      uint8_t sf = orc_f32_to_e4m3(amax / 6.0f);
      float sv = orc_e4m3_to_f32(sf);
      if (out_sf) out_sf[r * (cols / block) + b] = sf;
      for (int i = 0; i < block; ++i) {
        uint8_t q = sv > 0.0f ? orc_f32_to_e2m1(x[i] / sv) : 0;
        if (out_packed) {
          uint8_t* p = out_packed + r * (cols / 2) + b * (block / 2) + i / 2;
          if (i & 1) *p = (uint8_t)((*p & 0x0F) | (q << 4));
          else *p = (uint8_t)((*p & 0xF0) | q);
        }
        if (out_deq) out_deq[r * cols + b * block + i] = orc_e2m1_to_f32(q) * sv;
      }
    }
  }
}

/* OCP MX v1.0 block quantisation (mx spec section 6.3): each block of 32
 * consecutive elements of a row shares the E8M0 scale X = 2^s with
 * s = clamp(floor(log2(amax)) - emax_elem, -127, 127), emax_elem = 8 for e4m3 and
 * 2 for e2m1; the elements are x * 2^-s converted to the element type (round to
 * nearest even, saturating to the largest finite value).  2^-s is exact in fp32
 * for every s in range, so the scaling itself rounds only where x * 2^-s falls in
 * the fp32 subnormal range. */
static int orc_floor_log2(float a) { /* a > 0, finite */
  uint32_t u;
  memcpy(&u, &a, 4);
  const int e = (int)((u >> 23) & 0xFF);
  if (e) return e - 127;
  int top = 22; /* subnormal: the highest set bit of the mantissa */
  while (top > 0 && !((u >> top) & 1u)) --top;
  return top - 149;
}

static float orc_pow2(int e) { /* exact 2^e for e in [-127, 127] */
  uint32_t u = e >= -126 ? (uint32_t)(e + 127) << 23 : 0x00400000u;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

void orc_quant_mx(const float* in, int64_t rows, int64_t cols, int elem, uint8_t* out,
                  uint8_t* out_sf, float* out_deq) {
  orc_quant_mx_block(in, rows, cols, elem, 32, out, out_sf, out_deq);
}

/* One E8M0 scale per `block` elements (32, the OCP MX block; 64, the block the
 * 2:4-sparse kind::mxf8f6f4 MMA applies one scale to): amax over the block, the
 * elements scaled and converted as for block 32, stored in the element layout. */
void orc_quant_mx_block(const float* in, int64_t rows, int64_t cols, int elem, int block,
                        uint8_t* out, uint8_t* out_sf, float* out_deq) {
  /* emax of the element type: e4m3 8, e2m1 2, e5m2 15, e2m3 2, e3m2 4 */
  const int emax = elem == 0 ? 8 : elem == 2 ? 15 : elem == 4 ? 4 : 2;
  if (out && elem >= 3) memset(out, 0, (size_t)(rows * cols * 6 / 8));
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t b = 0; b < cols / block; ++b) {
      const float* x = in + r * cols + b * block;
      float amax = 0.0f;
      for (int i = 0; i < block; ++i) amax = fmaxf(amax, fabsf(x[i]));
      int s = amax > 0.0f ? orc_floor_log2(amax) - emax : -127;
      if (s < -127) s = -127;
      if (s > 127) s = 127;
      if (out_sf) out_sf[r * (cols / block) + b] = (uint8_t)(s + 127);
      const float inv = orc_pow2(-s), sv = orc_pow2(s);
      for (int i = 0; i < block; ++i) {
        const float v = x[i] * inv;
        if (elem == 0) {
          const uint8_t q = orc_f32_to_e4m3(v);
          if (out) out[r * cols + b * block + i] = q;
          if (out_deq) out_deq[r * cols + b * block + i] = orc_e4m3_to_f32(q) * sv;
        } else if (elem == 2) {
          const uint8_t q = orc_f32_to_e5m2(v);
          if (out) out[r * cols + b * block + i] = q;
          if (out_deq) out_deq[r * cols + b * block + i] = orc_e5m2_to_f32(q) * sv;
        } else if (elem >= 3) {
          const uint8_t q = elem == 3 ? orc_f32_to_e2m3(v) : orc_f32_to_e3m2(v);
          if (out) { /* element j of the row at bits [6j, 6j+6) of the packed row */
            const uint64_t bit = (uint64_t)(b * block + i) * 6u;
            uint8_t* row = out + r * (cols * 6 / 8);
            for (int k = 0; k < 6; ++k)
              if ((q >> k) & 1u) row[(bit + k) >> 3] |= (uint8_t)(1u << ((bit + k) & 7));
          }
          if (out_deq)
            out_deq[r * cols + b * block + i] =
                (elem == 3 ? orc_e2m3_to_f32(q) : orc_e3m2_to_f32(q)) * sv;
        } else {
          const uint8_t q = orc_f32_to_e2m1(v);
          if (out) {
            uint8_t* p = out + r * (cols / 2) + b * (block / 2) + i / 2;
            if (i & 1) *p = (uint8_t)((*p & 0x0F) | (q << 4));
            else *p = (uint8_t)((*p & 0xF0) | q);
          }
          if (out_deq) out_deq[r * cols + b * block + i] = orc_e2m1_to_f32(q) * sv;
        }
      }
    }
  }
}

/* ------------------------------------------------------------------ */
/* 2:4                                                                 */
/* ------------------------------------------------------------------ */
static const uint8_t kPairs[6][2] = {{0, 1}, {0, 2}, {0, 3}, {1, 2}, {1, 3}, {2, 3}};

/* The 2:4 operations on elements of eb bytes (2: bf16 / fp16, 1: fp8 / int8), or, for
 * eb < 0, on packed -eb-bit codes (fp4 / fp6 of kind::f8f6f4: element i at bits
 * [-eb * i, -eb * (i + 1)) of a little-endian bit stream, as orc_quant_sub packs). */
static inline uint32_t ld_elem(const void* p, int64_t i, int eb) {
  if (eb < 0) {
    const uint8_t* q = (const uint8_t*)p;
    uint32_t v = 0;
    for (int k = 0; k < -eb; ++k) {
      const int64_t bit = i * (int64_t)(-eb) + k;
      v |= (uint32_t)((q[bit >> 3] >> (bit & 7)) & 1u) << k;
    }
    return v;
  }
  return eb == 2 ? ((const uint16_t*)p)[i] : ((const uint8_t*)p)[i];
}

static inline void st_elem(void* p, int64_t i, int eb, uint32_t v) {
  if (eb < 0) {
    uint8_t* q = (uint8_t*)p;
    for (int k = 0; k < -eb; ++k) {
      const int64_t bit = i * (int64_t)(-eb) + k;
      q[bit >> 3] = (uint8_t)((q[bit >> 3] & ~(1u << (bit & 7))) | (((v >> k) & 1u) << (bit & 7)));
    }
    return;
  }
  if (eb == 2) ((uint16_t*)p)[i] = (uint16_t)v;
  else ((uint8_t*)p)[i] = (uint8_t)v;
}

static void prune_24_e(void* m, int eb, int64_t r0, int64_t nrows, int64_t cols, uint64_t seed) {
  int64_t groups = cols / 4;
  for (int64_t r = 0; r < nrows; ++r)
    for (int64_t g = 0; g < groups; ++g) {
      uint64_t h = orc_hash(seed ^ 0x3C6EF372FE94F82Bull, (uint64_t)(r0 + r) * (uint64_t)groups + (uint64_t)g);
      int p = (int)((h >> 32) % 6u);
      for (int i = 0; i < 4; ++i)
        if (i != kPairs[p][0] && i != kPairs[p][1]) st_elem(m, r * cols + g * 4 + i, eb, 0);
    }
}

static int compress_24_e(const void* dense, int eb, int64_t rows, int64_t K, uint32_t nz_mask,
                         void* comp, uint32_t* meta) {
  int64_t words = K / 32;
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t w = 0; w < words; ++w) {
      uint32_t word = 0;
      for (int g = 0; g < 8; ++g) {
        const int64_t base = r * K + w * 32 + g * 4;
        int idx[2], n = 0;
        for (int i = 0; i < 4; ++i)
          if (ld_elem(dense, base + i, eb) & nz_mask) {
            if (n == 2) return -1;
            idx[n++] = i;
          }
        /* fill with the lowest indices not already chosen */
        for (int i = 0; n < 2 && i < 4; ++i) {
          int used = 0;
          for (int j = 0; j < n; ++j) used |= (idx[j] == i);
          if (!used) idx[n++] = i;
        }
        if (idx[0] > idx[1]) { int t = idx[0]; idx[0] = idx[1]; idx[1] = t; }
        const int64_t out = r * (K / 2) + w * 16 + g * 2;
        st_elem(comp, out, eb, ld_elem(dense, base + idx[0], eb));
        st_elem(comp, out + 1, eb, ld_elem(dense, base + idx[1], eb));
        word |= (uint32_t)(idx[0] | (idx[1] << 2)) << (4 * g);
      }
      meta[r * words + w] = word;
    }
  return 0;
}

static void decompress_24_e(const void* comp, int eb, const uint32_t* meta, int64_t rows, int64_t K,
                            void* dense) {
  int64_t words = K / 32;
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t w = 0; w < words; ++w) {
      uint32_t word = meta[r * words + w];
      for (int g = 0; g < 8; ++g) {
        const int64_t base = r * K + w * 32 + g * 4;
        const int64_t in = r * (K / 2) + w * 16 + g * 2;
        uint32_t nib = (word >> (4 * g)) & 0xF;
        for (int i = 0; i < 4; ++i) st_elem(dense, base + i, eb, 0);
        st_elem(dense, base + (nib & 3), eb, ld_elem(comp, in, eb));
        st_elem(dense, base + ((nib >> 2) & 3), eb, ld_elem(comp, in + 1, eb));
      }
    }
}

void orc_prune_24(uint16_t* m, int64_t r0, int64_t nrows, int64_t cols, uint64_t seed) {
  prune_24_e(m, 2, r0, nrows, cols, seed);
}

int orc_compress_24(const uint16_t* dense, int64_t rows, int64_t K, uint16_t* comp,
                    uint32_t* meta) {
  return compress_24_e(dense, 2, rows, K, 0x7FFFu, comp, meta);
}

void orc_decompress_24(const uint16_t* comp, const uint32_t* meta, int64_t rows, int64_t K,
                       uint16_t* dense) {
  decompress_24_e(comp, 2, meta, rows, K, dense);
}

void orc_prune_12_f32(uint32_t* m, int64_t r0, int64_t nrows, int64_t cols, uint64_t seed) {
  const int64_t pairs = cols / 2;
  for (int64_t r = 0; r < nrows; ++r)
    for (int64_t g = 0; g < pairs; ++g) {
      uint64_t h = orc_hash(seed ^ 0x3C6EF372FE94F82Bull, (uint64_t)(r0 + r) * (uint64_t)pairs + (uint64_t)g);
      const int keep = (int)((h >> 32) & 1u);
      m[r * cols + g * 2 + (1 - keep)] = 0;
    }
}

int orc_compress_12_f32(const uint32_t* dense, int64_t rows, int64_t K, uint32_t* comp,
                        uint32_t* meta) {
  const int64_t words = K / 16;
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t w = 0; w < words; ++w) {
      uint32_t word = 0;
      for (int g = 0; g < 8; ++g) {
        const uint32_t e0 = dense[r * K + w * 16 + 2 * g], e1 = dense[r * K + w * 16 + 2 * g + 1];
        const int nz0 = (e0 & 0x7FFFFFFFu) != 0, nz1 = (e1 & 0x7FFFFFFFu) != 0;
        if (nz0 && nz1) return -1;
        const int keep = nz1 ? 1 : 0;
        comp[r * (K / 2) + w * 8 + g] = keep ? e1 : e0;
        word |= (keep ? 0xEu : 0x4u) << (4 * g);
      }
      meta[r * words + w] = word;
    }
  return 0;
}

void orc_decompress_12_f32(const uint32_t* comp, const uint32_t* meta, int64_t rows, int64_t K,
                           uint32_t* dense) {
  const int64_t words = K / 16;
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t w = 0; w < words; ++w)
      for (int g = 0; g < 8; ++g) {
        const uint32_t nib = (meta[r * words + w] >> (4 * g)) & 0xFu;
        const int keep = nib == 0xEu ? 1 : 0;
        dense[r * K + w * 16 + 2 * g] = keep ? 0u : comp[r * (K / 2) + w * 8 + g];
        dense[r * K + w * 16 + 2 * g + 1] = keep ? comp[r * (K / 2) + w * 8 + g] : 0u;
      }
}

void orc_prune_24_u8(uint8_t* m, int64_t r0, int64_t nrows, int64_t cols, uint64_t seed) {
  prune_24_e(m, 1, r0, nrows, cols, seed);
}

int orc_compress_24_u8(const uint8_t* dense, int64_t rows, int64_t K, uint8_t nz_mask,
                       uint8_t* comp, uint32_t* meta) {
  return compress_24_e(dense, 1, rows, K, nz_mask, comp, meta);
}

void orc_decompress_24_u8(const uint8_t* comp, const uint32_t* meta, int64_t rows, int64_t K,
                          uint8_t* dense) {
  decompress_24_e(comp, 1, meta, rows, K, dense);
}

/* Packed fp4 (bits 4) / fp6 (bits 6) codes: the same 2:4 positions and metadata as
 * the 8-bit codes, element by element; comp holds the kept codes packed the same way
 * ([rows][K/2] elements).  nz_mask leaves the sign bit out (-0 counts as zero). */
void orc_prune_24_sub(uint8_t* m, int64_t r0, int64_t nrows, int64_t cols, uint64_t seed,
                      int bits) {
  prune_24_e(m, -bits, r0, nrows, cols, seed);
}

int orc_compress_24_sub(const uint8_t* dense, int64_t rows, int64_t K, int bits, uint8_t nz_mask,
                        uint8_t* comp, uint32_t* meta) {
  return compress_24_e(dense, -bits, rows, K, nz_mask, comp, meta);
}

/* ------------------------------------------------------------------ */
/* FP32 GEMM (blocked, 8-wide partial sums, pthreads over M)           */
/* ------------------------------------------------------------------ */
typedef float v8f __attribute__((vector_size(32)));

typedef struct {
  const float *A, *B;
  float* C;
  int64_t M, N, K, lda, ldb, ldc, m0, m1, c0, c1; /* rows [m0, m1) x columns [c0, c1) */
  float alpha;
} gemm_job;

static inline float hsum8(v8f v) {
  return ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
}

static inline v8f ld8(const float* p) { v8f v; memcpy(&v, p, 32); return v; }

#define KB 512
#define NB 64

static void* gemm_worker(void* arg) {
  gemm_job* j = (gemm_job*)arg;
  const int64_t K = j->K;
  for (int64_t m = j->m0; m < j->m1; ++m)
    for (int64_t n = j->c0; n < j->c1; ++n) j->C[m * j->ldc + n] = 0.0f;
  for (int64_t k0 = 0; k0 < K; k0 += KB) {
    int64_t kl = (K - k0 < KB) ? K - k0 : KB;
    int64_t kv = kl & ~(int64_t)7;
    for (int64_t n0 = j->c0; n0 < j->c1; n0 += NB) {
      int64_t n1 = (n0 + NB < j->c1) ? n0 + NB : j->c1;
      for (int64_t m = j->m0; m < j->m1; m += 2) {
        int two = (m + 1 < j->m1);
        const float* a0 = j->A + m * j->lda + k0;
        const float* a1 = two ? a0 + j->lda : a0;
        for (int64_t n = n0; n < n1; n += 4) {
          int nc = (n1 - n < 4) ? (int)(n1 - n) : 4;
          const float* b[4];
          for (int c = 0; c < 4; ++c) b[c] = j->B + (n + (c < nc ? c : 0)) * j->ldb + k0;
          v8f acc0[4] = {{0}}, acc1[4] = {{0}};
          for (int64_t k = 0; k < kv; k += 8) {
            v8f x0 = ld8(a0 + k), x1 = ld8(a1 + k);
            for (int c = 0; c < 4; ++c) {
              v8f y = ld8(b[c] + k);
              acc0[c] += x0 * y;
              acc1[c] += x1 * y;
            }
          }
          for (int c = 0; c < nc; ++c) {
            float s0 = hsum8(acc0[c]), s1 = hsum8(acc1[c]);
            for (int64_t k = kv; k < kl; ++k) {
              s0 += a0[k] * b[c][k];
              s1 += a1[k] * b[c][k];
            }
            j->C[m * j->ldc + n + c] += s0;
            if (two) j->C[(m + 1) * j->ldc + n + c] += s1;
          }
        }
      }
    }
  }
  if (j->alpha != 1.0f)
    for (int64_t m = j->m0; m < j->m1; ++m)
      for (int64_t n = j->c0; n < j->c1; ++n) j->C[m * j->ldc + n] *= j->alpha;
  return NULL;
}

/* Threads split the rows of C when each gets at least 64 of them, else the
 * columns (in whole NB blocks): with few rows a row split makes every thread
 * stream all of B for a handful of rows.  Every element of C is computed in the
 * same order either way, so the result does not depend on the split. */
void orc_gemm_f32(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
                  int64_t lda, int64_t ldb, int64_t ldc, float alpha, int nthreads) {
  if (nthreads < 1) nthreads = 1;
  const int by_rows = M >= 64 * (int64_t)nthreads;
  const int64_t extent = by_rows ? M : (N + NB - 1) / NB; /* rows, or column blocks */
  if (nthreads > extent) nthreads = (int)(extent > 0 ? extent : 1);
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)nthreads);
  gemm_job* jobs = (gemm_job*)malloc(sizeof(gemm_job) * (size_t)nthreads);
  int64_t per = (extent + nthreads - 1) / nthreads;
  if (by_rows) per = (per + 1) & ~(int64_t)1;
  int launched = 0;
  for (int t = 0; t < nthreads; ++t) {
    int64_t e0 = t * per, e1 = e0 + per < extent ? e0 + per : extent;
    if (e0 >= extent) break;
    int64_t m0 = 0, m1 = M, c0 = 0, c1 = N;
    if (by_rows) {
      m0 = e0;
      m1 = e1;
    } else {
      c0 = e0 * NB;
      c1 = e1 * NB < N ? e1 * NB : N;
    }
    gemm_job jb = {A, B, C, M, N, K, lda, ldb, ldc, m0, m1, c0, c1, alpha};
    jobs[t] = jb;
    if (t == 0) continue;
    pthread_create(&th[t], NULL, gemm_worker, &jobs[t]);
    launched = t;
  }
  if (M > 0 && N > 0) gemm_worker(&jobs[0]);
  for (int t = 1; t <= launched; ++t) pthread_join(th[t], NULL);
  free(th);
  free(jobs);
}
