// datagen.cu -- seeded synthetic operands, quantisers and the 2:4 compressor.
//
// The reference fills its SMEM tiles with deterministic byte patterns
// (umma_throughput/umma_tput.cu:257-266, tcgen05_sparse_mma/tcgen05_sparse_mma.cu:246-256)
// and writes a constant 2:4 metadata word (tcgen05_sparse_mma.cu:327-332).  A real
// GEMM needs real operands: these kernels generate the seeded inputs of the
// benchmark configurations and quantise them, on the device, bit-identically to
// the CPU test oracle.  All kernels are grid-stride and HBM-bound.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "b2g_gemm.h"
#include "b2g_ptx.cuh"

namespace b2g {

__device__ __forceinline__ uint64_t hash64(uint64_t seed, uint64_t counter) {
  uint64_t z = seed + (counter + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__device__ __forceinline__ float gen_uniform(uint64_t seed, uint64_t ctr) {
  const int64_t u = (int64_t)(hash64(seed, ctr) >> 40);
  return (float)(2 * u - (1ll << 24)) * 0x1p-24f;
}

// Irwin-Hall: 12 uniforms of 24 bits (two per 64-bit hash); exact integer sum,
// one double -> float rounding, so host and device agree bit for bit.
__device__ __forceinline__ float gen_normal(uint64_t seed, uint64_t ctr) {
  int64_t s = 0;
#pragma unroll
  for (int i = 0; i < 6; ++i) {
    const uint64_t h = hash64(seed ^ 0x6A09E667F3BCC909ull, ctr * 6 + (uint64_t)i);
    s += (int64_t)(h >> 40);
    s += (int64_t)((h >> 16) & 0xFFFFFF);
  }
  return (float)((double)(s - 6 * (1ll << 24)) * 0x1p-24);
}

__global__ void fill_f32_kernel(float* out, int64_t n, uint64_t ctr0, uint64_t seed, int dist) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t c = ctr0 + (uint64_t)i;
    out[i] = dist ? gen_normal(seed, c) : gen_uniform(seed, c);
  }
}

__global__ void quant_bf16_kernel(const float* in, int64_t n, uint16_t* out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    __nv_bfloat16 b = __float2bfloat16_rn(in[i]);
    out[i] = *reinterpret_cast<uint16_t*>(&b);
  }
}

// e4m3 via the hardware cvt (round to nearest even, saturate to +-448).
__device__ __forceinline__ uint16_t cvt_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// four e2m1 pairs -> one 32-bit word; byte j = (hi nibble x[2j+1], lo nibble x[2j])
__device__ __forceinline__ uint32_t cvt_e2m1x8(const float* x) {
  uint32_t r;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(r)
      : "f"(x[0]), "f"(x[1]), "f"(x[2]), "f"(x[3]), "f"(x[4]), "f"(x[5]), "f"(x[6]),
        "f"(x[7]));
  return r;
}

__device__ __forceinline__ float e4m3_value(uint32_t b) {
  const uint32_t e = (b >> 3) & 15u, m = b & 7u;
  float v = e ? __uint_as_float(((e + 120u) << 23) | (m << 20)) : (float)m * 0x1p-9f;
  return (b & 0x80u) ? -v : v;
}

__global__ void quant_e4m3_kernel(const float* in, int64_t n, uint8_t* out) {
  const int64_t pairs = n / 2;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < pairs;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float2 v = reinterpret_cast<const float2*>(in)[i];
    reinterpret_cast<uint16_t*>(out)[i] = cvt_e4m3x2(v.x, v.y);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && (n & 1))
    out[n - 1] = (uint8_t)(cvt_e4m3x2(in[n - 1], 0.0f) & 0xFF);
}

// Element-wise conversions without scale factors, one element per thread:
//   QE_S8   int8: round to nearest even, saturate to [-128, 127]
//   QE_TF32 fp32 rounded to tf32 (10 mantissa bits, nearest even), low 13 bits zero
//   QE_E5M2 fp8 e5m2 via the hardware cvt (nearest even, saturate to +-57344)
//   QE_U8   uint8: round to nearest even, saturate to [0, 255]
//   QE_F16  fp16: round to nearest even (overflow to inf)
enum { QE_S8 = 0, QE_TF32 = 1, QE_E5M2 = 2, QE_U8 = 3, QE_F16 = 4 };

__device__ __forceinline__ uint32_t round_tf32_bits(uint32_t u) {
  if ((u & 0x7F800000u) == 0x7F800000u) return u & 0xFFFFE000u;  // inf / nan: truncate
  return (u + 0xFFFu + ((u >> 13) & 1u)) & 0xFFFFE000u;
}

template <int QE>
__global__ void quant_elem_kernel(const float* in, int64_t n, void* out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float x = in[i];
    if constexpr (QE == QE_S8 || QE == QE_U8) {
      int v = __float2int_rn(x);
      const int lo = QE == QE_S8 ? -128 : 0, hi = QE == QE_S8 ? 127 : 255;
      v = v < lo ? lo : (v > hi ? hi : v);
      static_cast<uint8_t*>(out)[i] = (uint8_t)(v & 0xFF);
    } else if constexpr (QE == QE_F16) {
      static_cast<__half*>(out)[i] = __float2half_rn(x);
    } else if constexpr (QE == QE_TF32) {
      static_cast<uint32_t*>(out)[i] = round_tf32_bits(__float_as_uint(x));
    } else {
      uint16_t r;
      asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.0f), "f"(x));
      static_cast<uint8_t*>(out)[i] = (uint8_t)(r & 0xFFu);
    }
  }
}

// Sub-byte elements of kind::f8f6f4 without scale factors, packed along the row
// the way the TMA's unpacking loads read them: each group of 16 consecutive
// elements fills 8 bytes (e2m1, element i in bits [4i, 4i+4)) or 12 bytes (e2m3 /
// e3m2, element i in bits [6i, 6i+6)), little-endian.  One thread per group.
enum { QS_E2M1 = 0, QS_E2M3 = 1, QS_E3M2 = 2 };

template <int QS>
__device__ __forceinline__ uint32_t cvt_fp6x2(float lo, float hi) {
  uint16_t r;
  if constexpr (QS == QS_E2M3)
    asm("cvt.rn.satfinite.e2m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  else
    asm("cvt.rn.satfinite.e3m2x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  // one 6-bit code in the low bits of each byte
  return (uint32_t)(r & 0x3Fu) | ((uint32_t)((r >> 8) & 0x3Fu) << 6);
}

// 16 fp6 values -> 12 bytes, element i at bits [6i, 6i+6), little-endian
template <int QS>
__device__ __forceinline__ void pack_fp6x16(const float* x, uint32_t (&w)[3]) {
  w[0] = w[1] = w[2] = 0u;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t pair = cvt_fp6x2<QS>(x[2 * i], x[2 * i + 1]);  // 12 bits
    const int bit = 12 * i, word = bit >> 5, off = bit & 31;
    w[word] |= pair << off;
    if (off > 20) w[word + 1] |= pair >> (32 - off);
  }
}

template <int QS>
__global__ void quant_sub_kernel(const float* in, int64_t groups, uint8_t* out) {
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < groups;
       g += (int64_t)gridDim.x * blockDim.x) {
    float x[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 v = reinterpret_cast<const float4*>(in + g * 16)[i];
      x[4 * i] = v.x;
      x[4 * i + 1] = v.y;
      x[4 * i + 2] = v.z;
      x[4 * i + 3] = v.w;
    }
    if constexpr (QS == QS_E2M1) {
      uint2 w;
      w.x = cvt_e2m1x8(x);
      w.y = cvt_e2m1x8(x + 8);
      reinterpret_cast<uint2*>(out)[g] = w;
    } else {
      uint32_t w[3];
      pack_fp6x16<QS>(x, w);
      uint32_t* o = reinterpret_cast<uint32_t*>(out + g * 12);
      o[0] = w[0];
      o[1] = w[1];
      o[2] = w[2];
    }
  }
}

// One thread per 16-element block: ue4m3 scale = e4m3(amax / 6), e2m1(x / scale).
template <int HALVES>
__global__ void quant_nvfp4_kernel(const float* in, int64_t blocks, uint8_t* out, uint8_t* sf) {
  // one ue4m3 scale = e4m3(amax / 6) per block of 16 * HALVES elements, each 16-element
  // half converted and stored as a block of 16 is
  for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < blocks;
       b += (int64_t)gridDim.x * blockDim.x) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 4 * HALVES; ++i) {
      const float4 v = reinterpret_cast<const float4*>(in + b * 16 * HALVES)[i];
      amax = fmaxf(fmaxf(amax, fmaxf(fabsf(v.x), fabsf(v.y))), fmaxf(fabsf(v.z), fabsf(v.w)));
    }
    const uint8_t s = (uint8_t)(cvt_e4m3x2(amax / 6.0f, 0.0f) & 0xFF);
    const float sv = e4m3_value(s);
#pragma unroll
    for (int hh = 0; hh < HALVES; ++hh) {
      const int64_t hb = b * HALVES + hh;
      float x[16];
      const float4* src = reinterpret_cast<const float4*>(in + hb * 16);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 v = src[i];
        x[4 * i] = v.x;
        x[4 * i + 1] = v.y;
        x[4 * i + 2] = v.z;
        x[4 * i + 3] = v.w;
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) x[i] = sv > 0.0f ? x[i] / sv : 0.0f;
      uint2 packed;
      packed.x = cvt_e2m1x8(x);
      packed.y = cvt_e2m1x8(x + 8);
      reinterpret_cast<uint2*>(out)[hb] = packed;
    }
    sf[b] = s;
  }
}

// OCP MX block-32 quantisation, one thread per block: E8M0 scale 2^s with
// s = clamp(floor(log2(amax)) - emax, -127, 127) (emax 8 for e4m3, 2 for e2m1),
// elements x * 2^-s converted with round-to-nearest-even and saturation.  2^-s is
// built exactly from its bits, so the result matches the CPU oracle bit for bit.
__device__ __forceinline__ float pow2_exact(int e) {  // e in [-127, 127]
  return __uint_as_float(e >= -126 ? (uint32_t)(e + 127) << 23 : 0x00400000u);
}

__device__ __forceinline__ int floor_log2_pos(float a) {  // a > 0, finite
  const uint32_t u = __float_as_uint(a);
  const int e = (int)((u >> 23) & 0xFF);
  if (e) return e - 127;
  return (31 - __clz((int)(u & 0x7FFFFFu))) - 149;
}

// ELEM: 0 = e4m3 (32 bytes per block), 1 = e2m1 (16 packed bytes), 2 = e5m2 (32 bytes),
// 3 = e2m3, 4 = e3m2 (24 packed bytes); emax of the element type (OCP MX v1.0):
// e4m3 8, e2m1 2, e5m2 15, e2m3 2, e3m2 4
template <int ELEM, int HALVES>
__global__ void quant_mx_kernel(const float* in, int64_t blocks, uint8_t* out, uint8_t* sf) {
  constexpr int kEmax = ELEM == 0 ? 8 : ELEM == 2 ? 15 : ELEM == 4 ? 4 : 2;
  for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < blocks;
       b += (int64_t)gridDim.x * blockDim.x) {
    // one scale per block of 32 * HALVES elements: the amax over the whole block,
    // then each 32-element half converted and stored as a 32-element block is
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8 * HALVES; ++i) {
      const float4 v = reinterpret_cast<const float4*>(in + b * 32 * HALVES)[i];
      amax = fmaxf(fmaxf(amax, fmaxf(fabsf(v.x), fabsf(v.y))), fmaxf(fabsf(v.z), fabsf(v.w)));
    }
    int sc = amax > 0.0f ? floor_log2_pos(amax) - kEmax : -127;
    sc = sc < -127 ? -127 : (sc > 127 ? 127 : sc);
    const float inv = pow2_exact(-sc);
#pragma unroll 1
    for (int hh = 0; hh < HALVES; ++hh) {
      const int64_t hb = b * HALVES + hh;  // 32-element block of the output
      float x[32];
      const float4* src = reinterpret_cast<const float4*>(in + hb * 32);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 v = src[i];
        x[4 * i] = v.x;
        x[4 * i + 1] = v.y;
        x[4 * i + 2] = v.z;
        x[4 * i + 3] = v.w;
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) x[i] = __fmul_rn(x[i], inv);
      if constexpr (ELEM == 0) {
        uint32_t w[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          w[j] = (uint32_t)cvt_e4m3x2(x[4 * j], x[4 * j + 1]) |
                 ((uint32_t)cvt_e4m3x2(x[4 * j + 2], x[4 * j + 3]) << 16);
        uint4* dst = reinterpret_cast<uint4*>(out + hb * 32);
        dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
        dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
      } else if constexpr (ELEM == 1) {
        reinterpret_cast<uint4*>(out)[hb] =
            make_uint4(cvt_e2m1x8(x), cvt_e2m1x8(x + 8), cvt_e2m1x8(x + 16), cvt_e2m1x8(x + 24));
      } else if constexpr (ELEM == 2) {
        uint8_t* dst = out + hb * 32;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          uint16_t r;
          asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.0f), "f"(x[j]));
          dst[j] = (uint8_t)(r & 0xFFu);
        }
      } else {
        uint32_t w[3], v[3];
        pack_fp6x16<ELEM == 3 ? QS_E2M3 : QS_E3M2>(x, w);
        pack_fp6x16<ELEM == 3 ? QS_E2M3 : QS_E3M2>(x + 16, v);
        uint32_t* dst = reinterpret_cast<uint32_t*>(out + hb * 24);
        dst[0] = w[0];
        dst[1] = w[1];
        dst[2] = w[2];
        dst[3] = v[0];
        dst[4] = v[1];
        dst[5] = v[2];
      }
    }
    sf[b] = (uint8_t)(sc + 127);
  }
}

__global__ void prune_24_kernel(uint16_t* m, int64_t groups_total, uint64_t group0,
                                uint64_t seed) {
  const uint8_t pairs[6][2] = {{0, 1}, {0, 2}, {0, 3}, {1, 2}, {1, 3}, {2, 3}};
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < groups_total;
       g += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t h = hash64(seed ^ 0x3C6EF372FE94F82Bull, group0 + (uint64_t)g);
    const int p = (int)((h >> 32) % 6u);
    uint2 v = reinterpret_cast<uint2*>(m)[g];
    uint16_t e[4] = {(uint16_t)(v.x & 0xFFFF), (uint16_t)(v.x >> 16), (uint16_t)(v.y & 0xFFFF),
                     (uint16_t)(v.y >> 16)};
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (i != pairs[p][0] && i != pairs[p][1]) e[i] = 0;
    v.x = (uint32_t)e[0] | ((uint32_t)e[1] << 16);
    v.y = (uint32_t)e[2] | ((uint32_t)e[3] << 16);
    reinterpret_cast<uint2*>(m)[g] = v;
  }
}

// One thread per 32 dense elements (8 groups): 16 kept values + one metadata word.
// 2:4 pruning of 8-bit codes (e4m3, e5m2, s8, u8): the same group counter and
// hash as prune_24_kernel, one 4-byte group per thread.
__global__ void prune_24_u8_kernel(uint32_t* m, int64_t groups_total, uint64_t group0,
                                   uint64_t seed) {
  const uint8_t pairs[6][2] = {{0, 1}, {0, 2}, {0, 3}, {1, 2}, {1, 3}, {2, 3}};
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < groups_total;
       g += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t h = hash64(seed ^ 0x3C6EF372FE94F82Bull, group0 + (uint64_t)g);
    const int p = (int)((h >> 32) % 6u);
    m[g] &= (0xFFu << (8 * pairs[p][0])) | (0xFFu << (8 * pairs[p][1]));
  }
}

// tf32 structured 1:2 pruning: pair g of absolute row r keeps element
// (hash(seed, r * (cols / 2) + g) >> 32) & 1 and zeroes the other; one pair per thread.
__global__ void prune_12_f32_kernel(uint2* m, int64_t pairs_total, uint64_t pair0, uint64_t seed) {
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < pairs_total;
       g += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t h = hash64(seed ^ 0x3C6EF372FE94F82Bull, pair0 + (uint64_t)g);
    uint2 v = m[g];
    if ((h >> 32) & 1u) v.x = 0u;
    else v.y = 0u;
    m[g] = v;
  }
}

// tf32 1:2 compressor: one thread per 16 dense elements (8 pairs) writes 8 kept words
// and one metadata word; the tcgen05 sparse tf32 MMA reads a pair as a group of four
// 16-bit halves, so nibble g is 0x4 (element 2g kept) or 0xE (element 2g + 1 kept).
// A pair with two non-zeros (31 low bits) sets ERRW_BAD_SPARSITY.
__global__ void compress_12_f32_kernel(const uint32_t* dense, int64_t chunks, uint32_t* comp,
                                       uint32_t* meta, uint32_t* err) {
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < chunks;
       c += (int64_t)gridDim.x * blockDim.x) {
    const uint4* src = reinterpret_cast<const uint4*>(dense + c * 16);
    uint32_t e[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 v = src[i];
      e[4 * i] = v.x;
      e[4 * i + 1] = v.y;
      e[4 * i + 2] = v.z;
      e[4 * i + 3] = v.w;
    }
    uint32_t word = 0, out[8];
    bool bad = false;
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      const bool nz0 = (e[2 * g] & 0x7FFFFFFFu) != 0u, nz1 = (e[2 * g + 1] & 0x7FFFFFFFu) != 0u;
      bad |= nz0 && nz1;
      out[g] = nz1 ? e[2 * g + 1] : e[2 * g];
      word |= (nz1 ? 0xEu : 0x4u) << (4 * g);
    }
    if (bad) atomicOr(err, ERRW_BAD_SPARSITY);
    uint4* dst = reinterpret_cast<uint4*>(comp + c * 8);
    dst[0] = make_uint4(out[0], out[1], out[2], out[3]);
    dst[1] = make_uint4(out[4], out[5], out[6], out[7]);
    meta[c] = word;
  }
}

// The two kept indices of a group of 4 from its non-zero flags (bit i: element i
// non-zero): the non-zero ones in ascending order, filled up with the lowest free
// indices.  *bad when more than two are non-zero.
__device__ __forceinline__ void pick_24(uint32_t nz, int& i0, int& i1, bool& bad) {
  i0 = -1;
  i1 = -1;
  int n = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (nz & (1u << i)) {
      if (n == 0) i0 = i;
      else if (n == 1) i1 = i;
      ++n;
    }
  bad |= (n > 2);
  if (n == 0) {
    i0 = 0;
    i1 = 1;
  } else if (n == 1) {
    if (i0 == 0) i1 = 1;
    else {
      i1 = i0;
      i0 = 0;
    }
  }
}

// 2:4 compressor of 8-bit codes: one thread per 32 dense elements reads 32 bytes and
// writes 16 bytes of kept values plus the canonical metadata word.  An element is
// non-zero when (byte & nz_mask) != 0 (0x7F for fp8, whose 0x80 is -0; 0xFF for
// the integers).
__global__ void compress_24_u8_kernel(const uint8_t* dense, int64_t chunks, uint32_t nz_mask,
                                      uint8_t* comp, uint32_t* meta, uint32_t* err) {
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < chunks;
       c += (int64_t)gridDim.x * blockDim.x) {
    const uint4* src = reinterpret_cast<const uint4*>(dense + c * 32);
    const uint4 v0 = src[0], v1 = src[1];
    const uint32_t w[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};  // group g = w[g]
    uint32_t word = 0, out[4] = {0u, 0u, 0u, 0u};
    bool bad = false;
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      uint32_t nz = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) nz |= (((w[g] >> (8 * i)) & nz_mask) != 0u ? 1u : 0u) << i;
      int i0, i1;
      pick_24(nz, i0, i1, bad);
      word |= (uint32_t)(i0 | (i1 << 2)) << (4 * g);
      const uint32_t kept = ((w[g] >> (8 * i0)) & 0xFFu) | (((w[g] >> (8 * i1)) & 0xFFu) << 8);
      out[g >> 1] |= kept << (16 * (g & 1));
    }
    if (bad) atomicOr(err, ERRW_BAD_SPARSITY);
    reinterpret_cast<uint4*>(comp)[c] = make_uint4(out[0], out[1], out[2], out[3]);
    meta[c] = word;
  }
}

// Packed sub-byte codes (the fp4 / fp6 element types of kind::f8f6f4: element i of a
// row at bits [b i, b i + b) of a little-endian bit stream), read and written through
// 32-bit words held in registers.  `w` has one spare zero word past the data.
__device__ __forceinline__ uint32_t get_code(const uint32_t* w, int bit, int b) {
  const uint64_t v = (uint64_t)w[bit >> 5] | ((uint64_t)w[(bit >> 5) + 1] << 32);
  return (uint32_t)(v >> (bit & 31)) & ((1u << b) - 1u);
}
__device__ __forceinline__ void put_code(uint32_t* w, int bit, int b, uint32_t code) {
  uint64_t v = (uint64_t)w[bit >> 5] | ((uint64_t)w[(bit >> 5) + 1] << 32);
  const uint64_t m = (uint64_t)((1u << b) - 1u) << (bit & 31);
  v = (v & ~m) | (((uint64_t)code << (bit & 31)) & m);
  w[bit >> 5] = (uint32_t)v;
  w[(bit >> 5) + 1] = (uint32_t)(v >> 32);
}

// 2:4 pruning of packed fp4 (b = 4) / fp6 (b = 6) codes: group g of four elements
// keeps the same two positions as the byte-wide pruning (hash of the group's index
// over the whole matrix) and zeroes the others; one thread per 16 elements (b * 2
// bytes: two or three whole 32-bit words).
__global__ void prune_24_sub_kernel(uint8_t* m, int64_t chunks, int b, uint64_t group0,
                                    uint64_t seed) {
  const uint8_t pairs[6][2] = {{0, 1}, {0, 2}, {0, 3}, {1, 2}, {1, 3}, {2, 3}};
  const int nw = b / 2;  // 32-bit words per 16 elements: 2 (fp4) or 3 (fp6)
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < chunks;
       c += (int64_t)gridDim.x * blockDim.x) {
    uint32_t* src = reinterpret_cast<uint32_t*>(m + c * (2 * b));
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    for (int i = 0; i < nw; ++i) w[i] = src[i];
#pragma unroll
    for (int gi = 0; gi < 4; ++gi) {
      const uint64_t h = hash64(seed ^ 0x3C6EF372FE94F82Bull, group0 + (uint64_t)(c * 4 + gi));
      const int p = (int)((h >> 32) % 6u);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (i != pairs[p][0] && i != pairs[p][1]) put_code(w, (4 * gi + i) * b, b, 0u);
    }
    for (int i = 0; i < nw; ++i) src[i] = w[i];
  }
}

// 2:4 compressor of packed fp4 / fp6 codes: one thread per 32 dense elements (b * 4
// bytes) writes the 16 kept elements (b * 2 bytes, packed the same way) and one
// canonical metadata word (group g's nibble idx0 | idx1 << 2 at bits 4g).  A code is
// zero when its bits under nz_mask are (the sign bit is left out: -0 counts as zero).
__global__ void compress_24_sub_kernel(const uint8_t* dense, int64_t chunks, int b,
                                       uint32_t nz_mask, uint8_t* comp, uint32_t* meta,
                                       uint32_t* err) {
  const int nw_in = b, nw_out = b / 2;  // 32-bit words in and out
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < chunks;
       c += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(dense + c * (4 * b));
    uint32_t w[7] = {0u, 0u, 0u, 0u, 0u, 0u, 0u}, out[4] = {0u, 0u, 0u, 0u};
    for (int i = 0; i < nw_in; ++i) w[i] = src[i];
    uint32_t word = 0;
    bool bad = false;
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      uint32_t nz = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        nz |= ((get_code(w, (4 * g + i) * b, b) & nz_mask) != 0u ? 1u : 0u) << i;
      int i0, i1;
      pick_24(nz, i0, i1, bad);
      word |= (uint32_t)(i0 | (i1 << 2)) << (4 * g);
      put_code(out, (2 * g) * b, b, get_code(w, (4 * g + i0) * b, b));
      put_code(out, (2 * g + 1) * b, b, get_code(w, (4 * g + i1) * b, b));
    }
    if (bad) atomicOr(err, ERRW_BAD_SPARSITY);
    uint32_t* dst = reinterpret_cast<uint32_t*>(comp + c * (2 * b));
    for (int i = 0; i < nw_out; ++i) dst[i] = out[i];
    meta[c] = word;
  }
}

__global__ void compress_24_kernel(const uint16_t* dense, int64_t chunks, uint16_t* comp,
                                   uint32_t* meta, uint32_t* err) {
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < chunks;
       c += (int64_t)gridDim.x * blockDim.x) {
    uint16_t e[32];
    const uint4* src = reinterpret_cast<const uint4*>(dense + c * 32);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 v = src[i];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        e[8 * i + 2 * j] = (uint16_t)(w[j] & 0xFFFF);
        e[8 * i + 2 * j + 1] = (uint16_t)(w[j] >> 16);
      }
    }
    uint32_t word = 0, out[8];
    bool bad = false;
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      uint32_t nz = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) nz |= ((e[4 * g + i] & 0x7FFF) != 0 ? 1u : 0u) << i;
      int i0, i1;
      pick_24(nz, i0, i1, bad);  // fewer than two non-zeros: the lowest unused indices
      word |= (uint32_t)(i0 | (i1 << 2)) << (4 * g);
      out[g] = (uint32_t)e[4 * g + i0] | ((uint32_t)e[4 * g + i1] << 16);
    }
    if (bad) atomicOr(err, ERRW_BAD_SPARSITY);
    uint4* dst = reinterpret_cast<uint4*>(comp + c * 16);
    dst[0] = make_uint4(out[0], out[1], out[2], out[3]);
    dst[1] = make_uint4(out[4], out[5], out[6], out[7]);
    meta[c] = word;
  }
}

// Canonical 2:4 metadata -> TMEM-ready blocks.  One thread per output word.
// Block (rb, kb) covers rows [128 rb, 128 rb + 128) and dense K [128 kb, 128 kb + 128);
// word (L, c) of the block is TMEM lane L, column c (the metadata of the c-th
// dense-K-32 MMA).  For kind::f16 with M = 128 a lane holds two rows' 16-bit
// halves of one K half: lane L = 16*m2 + 8*k1 + m0 carries rows 16*m2 + m0 (low
// half) and 16*m2 + 8 + m0 (high half), K half k1 (dense K [16 k1, 16 k1 + 16)
// of the MMA), i.e. canonical nibbles 4*k1 .. 4*k1 + 3 of each row's word.
__global__ void meta_ready_kernel(const uint32_t* canon, int64_t M, int64_t kw,
                                  int64_t k_blocks, int64_t total, uint32_t* ready) {
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(idx & 3);
    const int L = (int)((idx >> 2) & 127);
    const int64_t blk = idx >> 9;
    const int64_t kb = blk % k_blocks, rb = blk / k_blocks;
    const int m2 = L >> 4, k1 = (L >> 3) & 1, m0 = L & 7;
    const int64_t r_lo = rb * 128 + m2 * 16 + m0, r_hi = r_lo + 8;
    const int64_t chunk = kb * 4 + c;
    const uint32_t w_lo = (r_lo < M && chunk < kw) ? canon[r_lo * kw + chunk] : 0x44444444u;
    const uint32_t w_hi = (r_hi < M && chunk < kw) ? canon[r_hi * kw + chunk] : 0x44444444u;
    ready[idx] = ((w_lo >> (16 * k1)) & 0xFFFFu) | (((w_hi >> (16 * k1)) & 0xFFFFu) << 16);
  }
}

// Canonical 2:4 metadata -> TMEM-ready blocks for the 8-bit kinds (f8f6f4, i8).
// A sparse MMA of dense K = 64 reads 64 metadata bits per row, one bit per dense
// element: lane L holds row L, and the K order runs along the lane's bits (CuTe's
// tmem_e_frg for 8-bit A), so column j of an MMA is the row's canonical word of
// dense K [32 j, 32 j + 32).  Block (rb, kb) covers rows [128 rb, 128 rb + 128)
// and dense K [256 kb, 256 kb + 256) (one ring slot, 4 MMAs, 8 columns), stored
// as two halves of 128 lanes x 4 words; half h, word (L, c) is the canonical word
// 8 kb + 4 h + c of row 128 rb + L.
__global__ void meta_ready_u8_kernel(const uint32_t* canon, int64_t M, int64_t kw,
                                     int64_t k_blocks, int64_t total, uint32_t* ready) {
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(idx & 3);
    const int L = (int)((idx >> 2) & 127);
    const int h = (int)((idx >> 9) & 1);
    const int64_t blk = idx >> 10;
    const int64_t kb = blk % k_blocks, rb = blk / k_blocks;
    const int64_t r = rb * 128 + L;
    const int64_t chunk = kb * 8 + h * 4 + c;
    ready[idx] = (r < M && chunk < kw) ? canon[r * kw + chunk] : 0x44444444u;
  }
}

// Canonical NVFP4 scale factors -> the engine's scale-factor blocks.  One thread
// per output word (the 4 scales of one row for one MMA of K = 64).  Block b of
// `block_rows` rows and K slot s (256 elements = 16 scales per row) hold 4 MMA
// sub-blocks of padded_rows words; word w of a sub-block is row
// (w % 128) / 4 + 32 * ((w % 128) % 4 + 4 * (w / 128)) of the block, i.e. byte
// layout [32 rows][row group][4 scales] per 512 bytes: the source layout of
// tcgen05.cp.32x128b.warpx4 for the 4x1 scale-factor data path.
// Scale factors [rows][sf_cols] -> the engine's TMEM-ready blocks.  A group is 4
// consecutive scale bytes of a row (NVFP4: one MMA's 4 scales; MXFP8: one scale
// of each of 4 MMAs; MXFP4: 2 scales of each of 2 MMAs); a ring slot holds
// `groups` groups.  Per [row block][slot][group] the block is padded_rows / 4
// lines of 16 bytes: word (4 l + c) of each 128-row half q holds the group of
// row 32 c + l + 128 q, the layout tcgen05.cp.32x128b.warpx4 spreads over the
// four TMEM lane quarters.
__global__ void sf_ready_kernel(const uint8_t* sf, int64_t rows, int64_t sf_cols, int block_rows,
                                int padded_rows, int64_t slots, int groups, int64_t total,
                                uint32_t* ready) {
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int w = (int)(idx % padded_rows);
    const int64_t t = idx / padded_rows;
    const int kk = (int)(t % groups);
    const int64_t bs = t / groups;
    const int64_t slot = bs % slots, blk = bs / slots;
    const int wl = w & 127, q = w >> 7;
    const int local = (wl >> 2) + 32 * ((wl & 3) + 4 * q);
    const int64_t r = blk * block_rows + local;
    uint32_t v = 0;
    if (local < block_rows && r < rows) {
      const int64_t c0 = (slot * groups + kk) * 4;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (c0 + j < sf_cols) v |= (uint32_t)sf[r * sf_cols + c0 + j] << (8 * j);
    }
    ready[idx] = v;
  }
}

static int grid_for(int64_t n, int sm_count) {
  int64_t g = (n + 255) / 256;
  const int64_t cap = (int64_t)sm_count * 16;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (int)g;
}

cudaError_t launch_fill_f32(float* out, int64_t rows, int64_t cols, int64_t row0, uint64_t seed,
                            int dist, int sm_count, cudaStream_t s) {
  const int64_t n = rows * cols;
  fill_f32_kernel<<<grid_for(n, sm_count), 256, 0, s>>>(out, n, (uint64_t)(row0 * cols), seed,
                                                         dist);
  return cudaGetLastError();
}

cudaError_t launch_quant_bf16(const float* in, int64_t n, uint16_t* out, int sm_count,
                              cudaStream_t s) {
  quant_bf16_kernel<<<grid_for(n, sm_count), 256, 0, s>>>(in, n, out);
  return cudaGetLastError();
}

cudaError_t launch_quant_e4m3(const float* in, int64_t n, uint8_t* out, int sm_count,
                              cudaStream_t s) {
  quant_e4m3_kernel<<<grid_for(n / 2 + 1, sm_count), 256, 0, s>>>(in, n, out);
  return cudaGetLastError();
}

cudaError_t launch_quant_elem(int qe, const float* in, int64_t n, void* out, int sm_count,
                              cudaStream_t s) {
  const int grid = grid_for(n, sm_count);
  if (qe == QE_S8) quant_elem_kernel<QE_S8><<<grid, 256, 0, s>>>(in, n, out);
  else if (qe == QE_TF32) quant_elem_kernel<QE_TF32><<<grid, 256, 0, s>>>(in, n, out);
  else if (qe == QE_U8) quant_elem_kernel<QE_U8><<<grid, 256, 0, s>>>(in, n, out);
  else if (qe == QE_F16) quant_elem_kernel<QE_F16><<<grid, 256, 0, s>>>(in, n, out);
  else quant_elem_kernel<QE_E5M2><<<grid, 256, 0, s>>>(in, n, out);
  return cudaGetLastError();
}

cudaError_t launch_quant_sub(int qs, const float* in, int64_t n, uint8_t* out, int sm_count,
                             cudaStream_t s) {
  const int64_t groups = n / 16;
  const int grid = grid_for(groups, sm_count);
  if (qs == QS_E2M1) quant_sub_kernel<QS_E2M1><<<grid, 256, 0, s>>>(in, groups, out);
  else if (qs == QS_E2M3) quant_sub_kernel<QS_E2M3><<<grid, 256, 0, s>>>(in, groups, out);
  else quant_sub_kernel<QS_E3M2><<<grid, 256, 0, s>>>(in, groups, out);
  return cudaGetLastError();
}

cudaError_t launch_quant_nvfp4(const float* in, int64_t rows, int64_t cols, uint8_t* out,
                               uint8_t* sf, int sm_count, cudaStream_t s, int block) {
  const int64_t blocks = rows * cols / block;
  if (block == 32)
    quant_nvfp4_kernel<2><<<grid_for(blocks, sm_count), 256, 0, s>>>(in, blocks, out, sf);
  else
    quant_nvfp4_kernel<1><<<grid_for(blocks, sm_count), 256, 0, s>>>(in, blocks, out, sf);
  return cudaGetLastError();
}

cudaError_t launch_prune_24(uint16_t* m, int64_t rows, int64_t cols, int64_t row0, uint64_t seed,
                            int sm_count, cudaStream_t s) {
  const int64_t groups = rows * (cols / 4);
  prune_24_kernel<<<grid_for(groups, sm_count), 256, 0, s>>>(m, groups,
                                                             (uint64_t)(row0 * (cols / 4)), seed);
  return cudaGetLastError();
}

size_t sf_ready_bytes(int64_t rows, int64_t sf_cols, int groups, int block_rows,
                      int padded_rows) {
  const int64_t slots = (sf_cols + 4 * groups - 1) / (4 * groups);
  return (size_t)((rows + block_rows - 1) / block_rows) * (size_t)slots * (size_t)groups *
         (size_t)padded_rows * 4;
}

cudaError_t launch_sf_ready(const uint8_t* sf, int64_t rows, int64_t sf_cols, int groups,
                            int block_rows, int padded_rows, uint8_t* ready, int sm_count,
                            cudaStream_t s) {
  const int64_t slots = (sf_cols + 4 * groups - 1) / (4 * groups);
  const int64_t blocks = (rows + block_rows - 1) / block_rows;
  const int64_t total = blocks * slots * groups * padded_rows;  // words: sf_ready_bytes(...) / 4
  sf_ready_kernel<<<grid_for(total, sm_count), 256, 0, s>>>(sf, rows, sf_cols, block_rows,
                                                            padded_rows, slots, groups, total,
                                                            reinterpret_cast<uint32_t*>(ready));
  return cudaGetLastError();
}

template <int HALVES>
static void launch_quant_mx_h(const float* in, int64_t blocks, int elem, uint8_t* out, uint8_t* sf,
                              int grid, cudaStream_t s) {
  switch (elem) {
    case 0: quant_mx_kernel<0, HALVES><<<grid, 256, 0, s>>>(in, blocks, out, sf); break;
    case 1: quant_mx_kernel<1, HALVES><<<grid, 256, 0, s>>>(in, blocks, out, sf); break;
    case 2: quant_mx_kernel<2, HALVES><<<grid, 256, 0, s>>>(in, blocks, out, sf); break;
    case 3: quant_mx_kernel<3, HALVES><<<grid, 256, 0, s>>>(in, blocks, out, sf); break;
    default: quant_mx_kernel<4, HALVES><<<grid, 256, 0, s>>>(in, blocks, out, sf); break;
  }
}

cudaError_t launch_quant_mx(const float* in, int64_t rows, int64_t cols, int elem, uint8_t* out,
                            uint8_t* sf, int sm_count, cudaStream_t s, int block) {
  const int64_t blocks = rows * (cols / block);
  const int grid = grid_for(blocks, sm_count);
  if (block == 64) launch_quant_mx_h<2>(in, blocks, elem, out, sf, grid, s);
  else launch_quant_mx_h<1>(in, blocks, elem, out, sf, grid, s);
  return cudaGetLastError();
}

size_t meta_ready_bytes(int64_t M, int64_t K, int elem_bits) {
  // tf32: a pair of elements is a group of four 16-bit halves, so its metadata is the
  // 16-bit layout of twice the K
  if (elem_bits == 32) return meta_ready_bytes(M, 2 * K, 16);
  // one block per 128 rows and ring slot: 128 dense K and 2 KB (16-bit), 256 and 4 KB (8-bit)
  const int64_t k_slot = elem_bits == 8 ? 256 : 128;
  return (size_t)((M + 127) / 128) * (size_t)((K + k_slot - 1) / k_slot) * (size_t)(k_slot * 16);
}

cudaError_t launch_meta_ready(const uint32_t* canon, int64_t M, int64_t K, uint32_t* ready,
                              int sm_count, cudaStream_t s, int elem_bits) {
  if (elem_bits == 32) return launch_meta_ready(canon, M, 2 * K, ready, sm_count, s, 16);
  const int64_t k_blocks = (K + (elem_bits == 8 ? 255 : 127)) / (elem_bits == 8 ? 256 : 128);
  const int64_t total = (int64_t)(meta_ready_bytes(M, K, elem_bits) / 4);
  if (elem_bits == 8)
    meta_ready_u8_kernel<<<grid_for(total, sm_count), 256, 0, s>>>(canon, M, K / 32, k_blocks,
                                                                   total, ready);
  else
    meta_ready_kernel<<<grid_for(total, sm_count), 256, 0, s>>>(canon, M, K / 32, k_blocks, total,
                                                                ready);
  return cudaGetLastError();
}

cudaError_t launch_prune_12_f32(uint32_t* m, int64_t rows, int64_t cols, int64_t row0,
                                uint64_t seed, int sm_count, cudaStream_t s) {
  const int64_t pairs = rows * (cols / 2);
  prune_12_f32_kernel<<<grid_for(pairs, sm_count), 256, 0, s>>>(
      reinterpret_cast<uint2*>(m), pairs, (uint64_t)(row0 * (cols / 2)), seed);
  return cudaGetLastError();
}

cudaError_t launch_compress_12_f32(const uint32_t* dense, int64_t rows, int64_t K, uint32_t* comp,
                                   uint32_t* meta, uint32_t* err, int sm_count, cudaStream_t s) {
  const int64_t chunks = rows * (K / 16);
  compress_12_f32_kernel<<<grid_for(chunks, sm_count), 256, 0, s>>>(dense, chunks, comp, meta, err);
  return cudaGetLastError();
}

cudaError_t launch_prune_24_u8(uint8_t* m, int64_t rows, int64_t cols, int64_t row0, uint64_t seed,
                               int sm_count, cudaStream_t s) {
  const int64_t groups = rows * (cols / 4);
  prune_24_u8_kernel<<<grid_for(groups, sm_count), 256, 0, s>>>(
      reinterpret_cast<uint32_t*>(m), groups, (uint64_t)(row0 * (cols / 4)), seed);
  return cudaGetLastError();
}

cudaError_t launch_compress_24_u8(const uint8_t* dense, int64_t rows, int64_t K, uint32_t nz_mask,
                                  uint8_t* comp, uint32_t* meta, uint32_t* err, int sm_count,
                                  cudaStream_t s) {
  const int64_t chunks = rows * (K / 32);
  compress_24_u8_kernel<<<grid_for(chunks, sm_count), 256, 0, s>>>(dense, chunks, nz_mask, comp,
                                                                   meta, err);
  return cudaGetLastError();
}

cudaError_t launch_prune_24_sub(uint8_t* m, int64_t rows, int64_t cols, int64_t row0, int bits,
                               uint64_t seed, int sm_count, cudaStream_t s) {
  const int64_t chunks = rows * (cols / 16);
  prune_24_sub_kernel<<<grid_for(chunks, sm_count), 256, 0, s>>>(m, chunks, bits,
                                                                 (uint64_t)(row0 * (cols / 4)), seed);
  return cudaGetLastError();
}

cudaError_t launch_compress_24_sub(const uint8_t* dense, int64_t rows, int64_t K, int bits,
                                   uint32_t nz_mask, uint8_t* comp, uint32_t* meta, uint32_t* err,
                                   int sm_count, cudaStream_t s) {
  const int64_t chunks = rows * (K / 32);
  compress_24_sub_kernel<<<grid_for(chunks, sm_count), 256, 0, s>>>(dense, chunks, bits, nz_mask,
                                                                    comp, meta, err);
  return cudaGetLastError();
}

cudaError_t launch_compress_24(const uint16_t* dense, int64_t rows, int64_t K, uint16_t* comp,
                               uint32_t* meta, uint32_t* err, int sm_count, cudaStream_t s) {
  const int64_t chunks = rows * (K / 32);
  compress_24_kernel<<<grid_for(chunks, sm_count), 256, 0, s>>>(dense, chunks, comp, meta, err);
  return cudaGetLastError();
}

}  // namespace b2g
