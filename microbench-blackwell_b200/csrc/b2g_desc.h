// b2g_desc.h -- tcgen05 instruction and shared-memory descriptor encoders,
// usable from host and device code.
//
// Bit layouts follow the PTX ISA "Instruction descriptor" and "Shared memory
// descriptor" tables for tcgen05.mma (sm_100a).  The reference builds the same
// words at umma_throughput/umma_tput.cu:147-156 (SMEM descriptor, no swizzle)
// and :190-255 / tcgen05_sparse_mma/tcgen05_sparse_mma.cu:191-228 (instruction
// descriptor); tests/test_descriptors.py pins these encoders against the
// reference's own encoders compiled from its sources.
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define B2G_HD __host__ __device__ __forceinline__
#else
#define B2G_HD inline
#endif

namespace b2g {

// Kind codes follow the reference's KIND_ID (tcgen05_sparse_mma.cu:16-22).
enum Kind : int {
  KIND_TF32 = 0,
  KIND_F16 = 1,
  KIND_F8F6F4 = 2,
  KIND_I8 = 3,
  KIND_MXF8F6F4 = 4,
  KIND_MXF4 = 5,
  KIND_MXF4NVF4 = 6,
};

B2G_HD bool kind_block_scaled(int kind) {
  return kind == KIND_MXF8F6F4 || kind == KIND_MXF4 || kind == KIND_MXF4NVF4;
}

// Instruction descriptor (32 bits).
//   dense kinds:  [0,2) sparse selector, [2] sparse flag, [3] saturate,
//                 [4,6) D format (1 = f32, 2 = s32), [7,10) A type, [10,13) B type,
//                 [13] negate A, [14] negate B, [15] A MN-major, [16] B MN-major,
//                 [17,23) N >> 3, [24,29) M >> 4, [30,32) max shift (.ws)
//   block-scaled: [0,2) sparse selector, [2] sparse flag, [4,6) B scale-factor id,
//                 [7,10) A type, [10,13) B type, [17,23) N >> 3, [23] scale type
//                 (1 = ue8m0, 0 = ue4m3), [24,29) M >> 4, [29,31) A scale-factor id
// For M in {128, 256}, (M >> 4) << 24 equals the reference's (M >> 7) << 27.
B2G_HD uint32_t encode_idesc(int kind, int a_type, int b_type, int m, int n, int sparse,
                             int scale_type) {
  uint32_t d = 0;
  d |= (sparse ? 1u : 0u) << 2;
  if (kind_block_scaled(kind)) {
    uint32_t bt = (kind == KIND_MXF4 || kind == KIND_MXF4NVF4) ? ((uint32_t)b_type & 3u)
                                                              : (uint32_t)b_type;
    d |= ((uint32_t)a_type & 7u) << 7;
    d |= (bt & 7u) << 10;
    d |= ((uint32_t)(n >> 3) & 0x3Fu) << 17;
    d |= ((uint32_t)scale_type & 1u) << 23;
    d |= ((uint32_t)(m >> 4) & 0x1Fu) << 24;
  } else {
    uint32_t dfmt = (kind == KIND_I8) ? 2u : 1u;
    d |= dfmt << 4;
    d |= ((uint32_t)a_type & 7u) << 7;
    d |= ((uint32_t)b_type & 7u) << 10;
    d |= ((uint32_t)(n >> 3) & 0x3Fu) << 17;
    d |= ((uint32_t)(m >> 4) & 0x1Fu) << 24;
  }
  return d;
}

// Shared-memory matrix descriptor (64 bits):
//   [0,14) start address >> 4, [16,30) leading byte offset >> 4,
//   [32,46) stride byte offset >> 4, [46,48) version = 1 (sm_100),
//   [49,52) base offset, [52] LBO mode, [61,64) layout
//   (0 none, 1 128B/base32B, 2 128B, 4 64B, 6 32B).
enum Swizzle : int { SWZ_NONE = 0, SWZ_128B = 2, SWZ_64B = 4, SWZ_32B = 6 };

B2G_HD uint64_t encode_smem_desc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                 int swizzle) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= (uint64_t)((uint32_t)swizzle & 7u) << 61;
  return d;
}

}  // namespace b2g
