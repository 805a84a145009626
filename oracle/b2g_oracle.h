/*
 * b2g_oracle.h -- CPU restatement of the GEMM path, used ONLY as a test checker
 * and as the timed CPU baseline.  Nothing in the product (libb2g) links or calls
 * this code.
 *
 * The reference (lookup1980/microbench-blackwell) computes no observable GEMM
 * result and has no host reference GEMM, no seeded generator and no 2:4
 * compressor; everything here is restated from the mathematics, the OCP 8-bit
 * floating point / MX v1.0 format definitions and the PTX ISA sparse-metadata
 * convention.  GEMM values are therefore "parity unpinned" against the
 * reference; the reference pins only the metadata word 0x44444444 for kept
 * indices {0,1} (tcgen05_sparse_mma/tcgen05_sparse_mma.cu:331), the format
 * table (umma_throughput/umma_tput.cu:68-121,
 * tcgen05_sparse_mma/benchmark.py:20-33) and the A/B operand layouts
 * (cutlass_gemm_mainloop/cutlass_gemm_bench.cu:78-80).
 */
#ifndef B2G_ORACLE_H
#define B2G_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- seeded generator: splitmix64 finaliser over (seed, counter) ---- */
uint64_t orc_hash(uint64_t seed, uint64_t counter);
/* uniform[-1,1) with 24-bit resolution */
float orc_uniform(uint64_t seed, uint64_t counter);
/* normal(0,1) by the Irwin-Hall sum of 12 24-bit uniforms */
float orc_normal(uint64_t seed, uint64_t counter);
/* fill rows [r0, r0+nrows) of an R x cols row-major matrix (counter r*cols+c) */
void orc_fill(float* out, int64_t r0, int64_t nrows, int64_t cols, uint64_t seed, int dist);

/* ---- scalar codecs (round to nearest even, saturating to the max finite) ---- */
uint16_t orc_f32_to_bf16(float x);
float orc_bf16_to_f32(uint16_t b);
uint8_t orc_f32_to_e4m3(float x);
float orc_e4m3_to_f32(uint8_t b);
uint8_t orc_f32_to_e2m1(float x); /* 4-bit code in the low nibble */
float orc_e2m1_to_f32(uint8_t code);
uint8_t orc_f32_to_e5m2(float x);
float orc_e5m2_to_f32(uint8_t b);
int8_t orc_f32_to_s8(float x);
uint8_t orc_f32_to_u8(float x);
uint16_t orc_f32_to_f16(float x);
float orc_f16_to_f32(uint16_t h);
float orc_f32_to_tf32(float x);
uint8_t orc_f32_to_e2m3(float x); /* 6-bit code */
float orc_e2m3_to_f32(uint8_t c);
uint8_t orc_f32_to_e3m2(float x);
float orc_e3m2_to_f32(uint8_t c);
/* elem 0 e2m1, 1 e2m3, 2 e3m2, packed 16 per 8 / 12 bytes; n % 16 == 0 */
void orc_quant_sub(const float* in, int64_t n, int elem, uint8_t* out, float* out_deq);
/* elem 0 int8, 1 tf32 (fp32 storage), 2 e5m2, 3 uint8, 4 fp16 */
void orc_quant_elem(const float* in, int64_t n, int elem, void* out, float* out_deq);

/* ---- row quantisers; out_deq (nullable) receives the dequantised fp32 ---- */
void orc_quant_bf16(const float* in, int64_t n, uint16_t* out, float* out_deq);
void orc_quant_e4m3(const float* in, int64_t n, uint8_t* out, float* out_deq);
/* NVFP4: rows x cols (cols % 16 == 0); packed e2m1 rows x cols/2 bytes, low
 * nibble = even column; sf rows x cols/16 ue4m3 = e4m3(amax/6). */
/* OCP MX: rows x cols (cols % 32 == 0), elem 0 = e4m3 (out rows x cols bytes),
 * 1 = e2m1 (out packed rows x cols/2, low nibble = even column); sf rows x cols/32
 * E8M0 bytes (scale 2^(sf - 127)). */
void orc_quant_mx(const float* in, int64_t rows, int64_t cols, int elem, uint8_t* out,
                  uint8_t* out_sf, float* out_deq);
void orc_quant_mx_block(const float* in, int64_t rows, int64_t cols, int elem, int block,
                        uint8_t* out, uint8_t* out_sf, float* out_deq);
void orc_quant_nvfp4(const float* in, int64_t rows, int64_t cols, uint8_t* out_packed,
                     uint8_t* out_sf, float* out_deq);
void orc_quant_nvfp4_block(const float* in, int64_t rows, int64_t cols, int block,
                           uint8_t* out_packed, uint8_t* out_sf, float* out_deq);

/* ---- 2:4 structured sparsity ---- */
/* zero 2 of every 4 along each row; group counter r*(cols/4)+g (absolute row r) */
void orc_prune_24(uint16_t* bf16, int64_t r0, int64_t nrows, int64_t cols, uint64_t seed);
/* returns 0 on success, -1 if some group holds more than 2 non-zeros */
int orc_compress_24(const uint16_t* dense, int64_t rows, int64_t K, uint16_t* comp,
                    uint32_t* meta);
void orc_decompress_24(const uint16_t* comp, const uint32_t* meta, int64_t rows, int64_t K,
                       uint16_t* dense);
/* The same three on 8-bit elements (e4m3, e5m2, s8, u8): same group counter, same
 * metadata words ([rows][K/32], group g at bits 4g..4g+3 as idx0 | idx1 << 2).  An
 * element is non-zero when (byte & nz_mask) != 0: 0x7F for the fp8 formats, whose
 * 0x80 is -0, 0xFF for the integers. */
void orc_prune_24_u8(uint8_t* m, int64_t r0, int64_t nrows, int64_t cols, uint64_t seed);
/* packed fp4 / fp6 (bits 4 or 6) codes of kind::f8f6f4: 2:4 pruning and compression */
void orc_prune_24_sub(uint8_t* m, int64_t r0, int64_t nrows, int64_t cols, uint64_t seed,
                      int bits);
int orc_compress_24_sub(const uint8_t* dense, int64_t rows, int64_t K, int bits, uint8_t nz_mask,
                        uint8_t* comp, uint32_t* meta);
int orc_compress_24_u8(const uint8_t* dense, int64_t rows, int64_t K, uint8_t nz_mask,
                       uint8_t* comp, uint32_t* meta);
void orc_decompress_24_u8(const uint8_t* comp, const uint32_t* meta, int64_t rows, int64_t K,
                          uint8_t* dense);
/* tf32 (32-bit words): structured sparsity 1:2, one kept element of every pair.
 * The pruner keeps element (hash(seed, r*(cols/2)+g) >> 32) & 1 of pair g of absolute
 * row r.  The metadata describes each pair as a group of 4 16-bit halves: nibble g
 * of word w (pair w*8+g) is 0x4 (halves 0, 1: element 0 kept) or 0xE (halves 2, 3:
 * element 1 kept); words [rows][K/16].  An element is non-zero when its 31 low bits
 * are (the sign of -0 does not count); a pair with two non-zeros fails (-1); a pair
 * of zeros keeps element 0. */
void orc_prune_12_f32(uint32_t* m, int64_t r0, int64_t nrows, int64_t cols, uint64_t seed);
int orc_compress_12_f32(const uint32_t* dense, int64_t rows, int64_t K, uint32_t* comp,
                        uint32_t* meta);
void orc_decompress_12_f32(const uint32_t* comp, const uint32_t* meta, int64_t rows, int64_t K,
                           uint32_t* dense);

/* ---- FP32 GEMM: C[m][n] = alpha * sum_k A[m][k] * B[n][k] (B stored [N][K]) ---- */
void orc_gemm_f32(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
                  int64_t lda, int64_t ldb, int64_t ldc, float alpha, int nthreads);

#ifdef __cplusplus
}
#endif
#endif
