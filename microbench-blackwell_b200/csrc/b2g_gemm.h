// b2g_gemm.h -- internal interface between the C ABI layer (b2g_api.cu) and the
// kernel translation units.  Not part of the public ABI.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace b2g {

// Arguments of the dense / sparse GEMM kernels (passed by value).
struct GemmArgs {
  int M, N;
  int num_m_tiles, num_n_tiles;  // tiles of (128 * CG) x tile_n
  int k_blocks;                  // ring slots per tile (one 128-byte K slice each)
  int tile_n;                    // N extent of the MMA
  int stages;                    // ring depth
  int group_m;                   // grouped raster height (in M tiles)
  int elem_bits;                 // bits per stored A/B element (16, 8, 4)
  int tx_a_bits, tx_b_bits;      // A / B bits per element the TMA's completion counts: 0 =
                                 // the shared-memory bytes; 4 / 6 for the unpacking maps of
                                 // fp4 / fp6, which count the packed bytes they read
  uint32_t idesc;                // tcgen05 instruction descriptor
  float alpha;
  __nv_bfloat16* C;
  int64_t ldc;
  int c_vec_ok;                  // C base 16B aligned and ldc % 8 == 0
  uint32_t* err;                 // device error word
  uint32_t* trace;               // optional progress trace, kTraceWords per CTA (host-mapped)
  // Split tail: tiles [tail_start, num tiles) are each computed as tail_split
  // K ranges on different clusters.  Split s > 0 writes its fp32 partial tile to
  // `part` and stamps its flags with `epoch`; split 0 waits for the stamps and
  // adds the partials in its epilogue.  tail_split <= 1: no split.
  int tail_start;
  int tail_split;
  float* part;                   // [tail tile][split - 1][tile rows][tile_n] fp32
  uint32_t* flags;               // [tail tile][split - 1][CTA rank][epilogue warp]
  uint32_t epoch;                // this launch's stamp, never 0
  uint64_t wait_ns;              // limit of every bounded wait (0: kWaitLimitNs)
};

// Progress trace layout, per CTA (blockIdx.x * kTraceWords + slot).
enum TraceSlot : int {
  TR_STAGE = 0,        // 1 started, 2 TMEM allocated, 3 set-up synced, 5 roles done,
                       // 6 teardown synced, 7 TMEM freed
  TR_TMA_ISSUED = 1,   // ring slots loaded by the producer
  TR_FULL_SEEN = 2,    // ring slots the MMA issuer saw full
  TR_MMA_ISSUED = 3,   // ring slots whose MMAs were issued and committed
  TR_TILES_MMA = 4,    // accumulators committed
  TR_TILES_EPI = 5,    // tiles stored by the epilogue (warp 2)
  TR_TFULL_SEEN = 6,   // accumulators the epilogue saw full (warp 2)
  TR_TIMEOUTS = 7,     // bit 0 producer, 1 MMA full, 2 MMA tempty, 3 epilogue, 4 drain
  TR_TMEM_BASE = 8,
  kTraceWords = 16
};

// Kernel variants: dense, structured-sparse A (kind::f16, tf32, f8f6f4, i8).
// Block-scaled variants: NVFP4 (e2m1, ue4m3 per 16, kind::mxf4nvf4), MXFP8 (e4m3,
// E8M0 per 32, kind::mxf8f6f4), MXFP4 (e2m1, E8M0 per 32, kind::mxf4), and MXF8_SP:
// 2:4-sparse A on kind::mxf8f6f4 (8-bit element types, E8M0 per 64 dense K), and
// MXF4_SP: 4:8-sparse A in pairs on kind::mxf4 (packed e2m1, E8M0 per 64 dense K);
// NVFP4_SP: the same on kind::mxf4nvf4 block16 (ue4m3 per 32 dense K).
enum GemmVariant : int { GEMM_DENSE = 0, GEMM_SPARSE = 1, GEMM_NVFP4 = 2, GEMM_MXF8 = 3,
                         GEMM_MXF4 = 4, GEMM_MXF8_SP = 5, GEMM_MXF4_SP = 6, GEMM_NVFP4_SP = 7 };
__host__ __device__ constexpr bool gemm_block_scaled(int var) { return var >= GEMM_NVFP4; }
// variants whose A is structured-sparse (2:4 metadata in the ring slot)
__host__ __device__ constexpr bool gemm_sparse(int var) {
  return var == GEMM_SPARSE || var == GEMM_MXF8_SP || var == GEMM_MXF4_SP ||
         var == GEMM_NVFP4_SP;
}
// 4-byte scale-factor groups per ring slot (4 MMAs): NVFP4 4 scales per MMA, MXFP8
// 1, MXFP4 2; the sparse forms read as many scales per MMA as the dense one of their
// kind (measured for kind::mxf8f6f4: the scale byte the MMA names applies to its 64
// dense K), each over twice the dense K: sparse MXFP8 1, sparse MXFP4 2, sparse NVFP4 4
__host__ __device__ constexpr int gemm_sf_groups(int var) {
  return (var == GEMM_NVFP4 || var == GEMM_NVFP4_SP)
             ? 4
             : ((var == GEMM_MXF4 || var == GEMM_MXF4_SP) ? 2 : 1);
}

// The side operands (2:4 metadata, scale factors) of one ring slot are contiguous
// blocks of the engine-layout buffers in HBM.  Their tensor maps view those
// buffers as rows of kSideLine bytes, so that the TMA box of a block moves whole
// 256-byte lines (boxes of 16-byte rows, the TMEM lane width, would split the same
// bytes into 16x the row requests); a block lands in shared memory byte for byte,
// as tcgen05.cp reads it.  Every block is a multiple of kSideLine bytes.
constexpr int kSideLine = 256;

// Tensor maps of one launch: A, B, and the side operands (sparse: e = metadata;
// block-scaled: e = SFA blocks, f = SFB blocks; sparse block-scaled: e = metadata,
// f = SFA, g = SFB).  Unused maps are zero.
struct GemmMaps {
  CUtensorMap a, b, e, f, g;
};

// kind: the tcgen05 kind (sets the 2:4 metadata bytes and columns of a sparse slot)
size_t gemm_smem_bytes(int stages, int b_rows, int var, int m_sub, int k_atoms, int kind);
int gemm_kernel_threads(int m_sub);  // threads per CTA of the GEMM kernel
int gemm_tmem_columns(int tile_n, int var, bool ts, int m_sub, int kind);
// ts: A operand from TMEM (dense variant only).  m_sub: 128-row A sub-tiles per
// CTA; a tile then spans 128 * m_sub * cg rows.  k_atoms: 128-byte K atoms per
// ring slot (2 only for dense SS with one sub-tile).  ws: the weight-stationary
// MMA form (tcgen05.mma.ws{.sp}; cta_group 1, SS, one sub-tile, one K atom).
cudaError_t gemm_launch(int kind, int cg, int var, bool ts, int m_sub, int k_atoms, bool ws,
                        const GemmMaps& maps, const GemmArgs& a, int grid, size_t smem,
                        cudaStream_t stream);
cudaError_t gemm_max_active_clusters(int kind, int cg, int var, bool ts, int m_sub, int k_atoms,
                                     bool ws, int smem, int* out);
// Default A sub-tiles per CTA: 2 for sparse and block-scaled problems with a long K
// (the un-overlapped epilogue is then a small share) and enough 2-sub-tile tiles to
// give every cluster one; 2 for dense 256-column pair tiles with a long K whose
// 512-row waves take no longer than the 256-row ones; else 1.
int gemm_default_m_sub(int var, int64_t M, int64_t N, int64_t K, int cg, int tile_n,
                       int clusters);

// Data generation / quantisation / 2:4 (datagen.cu)
cudaError_t launch_fill_f32(float* out, int64_t rows, int64_t cols, int64_t row0, uint64_t seed,
                            int dist, int sm_count, cudaStream_t s);
cudaError_t launch_quant_bf16(const float* in, int64_t n, uint16_t* out, int sm_count,
                              cudaStream_t s);
// qs: 0 e2m1 (8 bytes per 16 elements), 1 e2m3, 2 e3m2 (12 bytes per 16); n % 16 == 0
cudaError_t launch_quant_sub(int qs, const float* in, int64_t n, uint8_t* out, int sm_count,
                             cudaStream_t s);
// qe: 0 int8, 1 tf32 (fp32 storage), 2 e5m2, 3 uint8, 4 fp16 -- element-wise, no scale factors
cudaError_t launch_quant_elem(int qe, const float* in, int64_t n, void* out, int sm_count,
                              cudaStream_t s);
cudaError_t launch_quant_e4m3(const float* in, int64_t n, uint8_t* out, int sm_count,
                              cudaStream_t s);
// NVFP4: packed e2m1 and one ue4m3 scale = e4m3(amax / 6) per `block` elements (16;
// 32 for the 4:8-sparse GEMM, whose MMA reads its four scales over 128 dense K)
cudaError_t launch_quant_nvfp4(const float* in, int64_t rows, int64_t cols, uint8_t* out,
                               uint8_t* sf, int sm_count, cudaStream_t s, int block = 16);
cudaError_t launch_prune_24(uint16_t* m, int64_t rows, int64_t cols, int64_t row0, uint64_t seed,
                            int sm_count, cudaStream_t s);
// 2:4 prune / compress of 8-bit codes (same group counter and metadata as the
// 16-bit forms); nz_mask: the bits of a non-zero element (0x7F fp8, 0xFF integers).
cudaError_t launch_prune_24_u8(uint8_t* m, int64_t rows, int64_t cols, int64_t row0, uint64_t seed,
                               int sm_count, cudaStream_t s);
cudaError_t launch_compress_24_u8(const uint8_t* dense, int64_t rows, int64_t K, uint32_t nz_mask,
                                  uint8_t* comp, uint32_t* meta, uint32_t* err, int sm_count,
                                  cudaStream_t s);
// tf32 structured 1:2 prune / compress (metadata [rows][K/16] words; nibble 0x4 or 0xE
// per pair, the pair read as four 16-bit halves)
cudaError_t launch_prune_12_f32(uint32_t* m, int64_t rows, int64_t cols, int64_t row0,
                                uint64_t seed, int sm_count, cudaStream_t s);
cudaError_t launch_compress_12_f32(const uint32_t* dense, int64_t rows, int64_t K, uint32_t* comp,
                                   uint32_t* meta, uint32_t* err, int sm_count, cudaStream_t s);
// Canonical 2:4 metadata ([M][K/32] words) -> the engine's TMEM-ready layout, in
// the order [row block][K slot].  16-bit A (kind::f16): blocks of 128 rows x 128
// dense K, each 128 lanes x 4 words; 8-bit A (kind::f8f6f4, kind::i8): blocks of
// 128 rows x 256 dense K, two halves of 128 lanes x 4 words; tf32 (elem_bits 32): the
// 16-bit layout of 2 K (its [M][K/16] words).  Rows >= M and K >= K are padded with
// 0x4444 nibbles.
cudaError_t launch_meta_ready(const uint32_t* canon, int64_t M, int64_t K, uint32_t* ready,
                              int sm_count, cudaStream_t s, int elem_bits = 16);
size_t meta_ready_bytes(int64_t M, int64_t K, int elem_bits = 16);
// Canonical NVFP4 scale factors ([rows][K/16] ue4m3) -> the engine's blocks:
// for A, per 128-row block and 256-K slot, 4 MMA sub-blocks of 512 bytes laid out
// [32 rows][4 row groups][4 scales]; for B the same per tile_n-row block with 256
// rows (8 row groups, zero-padded past tile_n and past the matrix).
// Scale factors [rows][sf_cols] -> TMEM-ready blocks of `groups` 4-byte groups per
// ring slot, per block_rows rows padded to padded_rows (NVFP4: groups 4; MXFP8: 1;
// MXFP4: 2).
size_t sf_ready_bytes(int64_t rows, int64_t sf_cols, int groups, int block_rows, int padded_rows);
cudaError_t launch_sf_ready(const uint8_t* sf, int64_t rows, int64_t sf_cols, int groups,
                            int block_rows, int padded_rows, uint8_t* ready, int sm_count,
                            cudaStream_t s);
// OCP MX quantisation: elem 0 = e4m3 (rows x cols bytes), 1 = e2m1 (packed rows x
// cols/2), 2 = e5m2, 3 = e2m3, 4 = e3m2 (packed fp6); sf rows x cols/block E8M0, one
// scale per `block` (32, the OCP MX block, or 64: the block of the 2:4-sparse
// kind::mxf8f6f4 MMA, whose 64 dense K share one scale per row) elements.
cudaError_t launch_quant_mx(const float* in, int64_t rows, int64_t cols, int elem, uint8_t* out,
                            uint8_t* sf, int sm_count, cudaStream_t s, int block = 32);
cudaError_t launch_compress_24(const uint16_t* dense, int64_t rows, int64_t K, uint16_t* comp,
                               uint32_t* meta, uint32_t* err, int sm_count, cudaStream_t s);
// 2:4 prune / compress of packed fp4 (bits 4) and fp6 (bits 6) codes of kind::f8f6f4:
// prune needs cols % 16, compress K % 32; metadata as for the 8-bit codes.
cudaError_t launch_prune_24_sub(uint8_t* m, int64_t rows, int64_t cols, int64_t row0, int bits,
                               uint64_t seed, int sm_count, cudaStream_t s);
cudaError_t launch_compress_24_sub(const uint8_t* dense, int64_t rows, int64_t K, int bits,
                                   uint32_t nz_mask, uint8_t* comp, uint32_t* meta, uint32_t* err,
                                   int sm_count, cudaStream_t s);

// tcgen05.mma instruction probe (probe.cu)
struct ProbeArgs {
  uint32_t idesc;
  int a_rows;          // A rows per CTA
  int b_rows;          // B rows per CTA
  int depth, iters, mode;
  uint32_t tmem_cols;
  uint32_t d_col, a_col, sf_col, meta_col;  // TMEM column offsets
  uint32_t sf_word;    // scale-factor fill (1.0 in the scale format)
  unsigned long long* result;  // [cycles, total mmas, median latency]
  uint32_t* err;
};
cudaError_t probe_launch(int kid, int sp, int ws, int cg, int ts, const ProbeArgs& p, size_t smem,
                         cudaStream_t s);

// Bounded-wait self-test (selftest.cu): one warp waits with limit_ns on an mbarrier
// (mode 0) or on the word at `flag` (mode 1) that nothing completes; writes the
// time until the wait expired to elapsed_ns[0] (0 if it did not expire).
cudaError_t wait_selftest_launch(int mode, uint64_t limit_ns, const uint32_t* flag, uint32_t* err,
                                 unsigned long long* elapsed_ns, cudaStream_t s);

// TMA 2D streaming probe (tma2d.cu).  *_prepare sets the kernel's shared-memory
// attribute and loads its module; call it before timing a launch.
cudaError_t tma2d_stream_prepare(int smem_bytes);
cudaError_t bulk1d_stream_prepare(int smem_bytes);
cudaError_t bulk1d_stream_launch(const void* data, uint64_t chunks, uint32_t load_bytes, int stages,
                                 int grid, int smem_bytes, uint32_t* err, cudaStream_t s);
// dynamic shared memory of the latency probe: the opt-in maximum less its static part
cudaError_t tma2d_latency_smem(int device, int* smem_bytes);
cudaError_t tma2d_latency_launch(const CUtensorMap& tm, int64_t row0, int box_w, int box_h,
                                 int grid, int smem_bytes, uint32_t* cycles, uint32_t* err,
                                 cudaStream_t s);
cudaError_t tma2d_stream_launch(const CUtensorMap& tm, uint64_t height, int box_w, int box_h,
                                int stages, int grid, int smem_bytes, uint32_t* err,
                                cudaStream_t s);

}  // namespace b2g
