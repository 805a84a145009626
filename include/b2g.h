/*
 * b2g.h -- C ABI of libb2g, the B200 (sm_100a) tensor-core GEMM engine.
 *
 * The reference (lookup1980/microbench-blackwell) has no library and no FFI: its
 * only interface is "make VAR=... -> ./x.out -> stdout RESULT line -> CSV".  Each
 * entry point below names the reference code it replaces.  The thin drop-in mains
 * under microbench-blackwell_b200/drivers/ (one per reference benchmark directory)
 * call this ABI; so do the ctypes wrapper and the multi-GPU driver.
 *
 * Conventions
 *   - Plain C types only.  Every pointer argument named d_* is a CUDA device
 *     pointer owned by the caller; h_* pointers are host memory.
 *   - Every call returns b2g_status.  No exception ever crosses the ABI.
 *   - Calls that take a `stream` are asynchronous on that stream (cudaStream_t
 *     passed as void*; NULL = legacy default stream).
 *   - A handle binds one CUDA device.  Use one handle per host thread.
 *   - Kernel-side waits are bounded: a wait that exceeds its time limit makes the
 *     kernel record an error word and return; b2g_check() reports it as
 *     B2G_ERR_TIMEOUT.  No kernel traps.
 */
#ifndef B2G_H
#define B2G_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B2G_ABI_VERSION 2

#if defined(__GNUC__)
#define B2G_API __attribute__((visibility("default")))
#else
#define B2G_API
#endif

typedef enum b2g_status {
  B2G_OK = 0,
  B2G_ERR_INVALID = 1,      /* bad argument: size, alignment, null pointer, combination */
  B2G_ERR_CUDA = 2,         /* a CUDA runtime / driver call failed */
  B2G_ERR_TIMEOUT = 3,      /* a kernel-side bounded wait expired */
  B2G_ERR_UNSUPPORTED = 4,  /* valid request this build does not implement */
  B2G_ERR_NO_DEVICE = 5,    /* no CUDA device, or it is not sm_100 */
  B2G_ERR_MISMATCH = 6      /* a device-side self check failed */
} b2g_status;

/* Operand formats.  Values 0-5 are the reference's MMA_FORMAT codes
 * (umma_throughput/umma_tput.cu:68-75); 6 is the NVFP4 path
 * (tcgen05_sparse_mma/tcgen05_sparse_mma.cu:106-108, kind::mxf4nvf4 with ue4m3 scales);
 * 7-12 are the remaining element types of the sparse benchmark's type table
 * (tcgen05_sparse_mma/Makefile:62-103 and benchmark.py:20-33: tf32, e5m2, e2m3,
 * e3m2, f16, u8).
 * b2g_gemm is built for every format (and 2:4-sparse A in BF16, F16, E4M3, E5M2, S8
 * and U8); every format also runs
 * in the probe (b2g_probe_mma).  E2M1, E2M3 and E3M2 run on kind::f8f6f4: they
 * stay packed in memory (16 elements per 8 or 12 bytes) and the TMA unpacks them
 * into the MMA's 16-byte chunks; for them K, lda and ldb are multiples of 128 and
 * A, B are 32-byte aligned. */
typedef enum b2g_format {
  B2G_FMT_BF16 = 0,   /* bf16 x bf16 -> f32, instruction K = 16 */
  B2G_FMT_E4M3 = 1,   /* fp8 e4m3 x e4m3 -> f32, K = 32 */
  B2G_FMT_S8 = 2,     /* int8 x int8 -> s32 (kind::i8), K = 32; C = bf16(alpha * fp32(acc)) */
  B2G_FMT_E2M1 = 3,   /* fp4 e2m1 x e2m1 (kind::f8f6f4, no scales) -> f32, K = 32 */
  B2G_FMT_MXF8 = 4,   /* MX e4m3, ue8m0 scale per 32 (GEMM: kind::mxf8f6f4) */
  B2G_FMT_MXF4 = 5,   /* MX e2m1 packed, ue8m0 scale per 32 (GEMM: kind::mxf4) */
  B2G_FMT_NVFP4 = 6,  /* e2m1 with one ue4m3 scale per 16 K elements */
  B2G_FMT_TF32 = 7,   /* tf32 x tf32 -> f32 (kind::tf32), K = 8; operands stored as fp32 */
  B2G_FMT_E5M2 = 8,   /* fp8 e5m2 x e5m2 -> f32 (kind::f8f6f4), K = 32 */
  B2G_FMT_E2M3 = 9,   /* fp6 e2m3 x e2m3 (kind::f8f6f4) -> f32, K = 32 */
  B2G_FMT_E3M2 = 10,  /* fp6 e3m2 x e3m2 (kind::f8f6f4) -> f32, K = 32 */
  B2G_FMT_F16 = 11,   /* fp16 x fp16 (kind::f16, type code 0) -> f32, K = 16 */
  B2G_FMT_U8 = 12     /* uint8 x uint8 (kind::i8, type code 0) -> s32, K = 32 */
} b2g_format;

typedef struct b2g_handle b2g_handle;

/* One GEMM C = alpha * A . B, fp32 accumulate, bf16 C.
 *   A row-major  [M][lda]  (K contiguous)          -- cutlass_gemm_bench.cu:78
 *   B col-major  [N][ldb]  (K contiguous per column) -- cutlass_gemm_bench.cu:79
 *   C row-major  [M][ldc]  bf16
 * Leading dimensions are in ELEMENTS of the stored type (for packed e2m1, in
 * elements too: two per byte).  For sparse = 1 (bf16, fp16, e4m3, e5m2, e2m1, e2m3,
 * e3m2, s8, u8, the MX e4m3 / e5m2 of mx_scale and B2G_FMT_MXF8; tf32 1:2; MXFP4 and
 * NVFP4 4:8 in pairs, with sfa / sfb one E8M0 per 64 K or one ue4m3 per 32 K: the
 * sparse MMA's scale blocks), A
 * is the 2:4-compressed operand [M][K/2] (lda counts compressed elements) and meta
 * is the metadata produced by b2g_compress_24 / b2g_compress_24_format.  For NVFP4, sfa/sfb hold one ue4m3 byte per 16 K elements,
 * row-major [M][K/16] and [N][K/16]. */
typedef struct b2g_gemm_desc {
  int32_t format;           /* b2g_format */
  int32_t sparse;           /* 0 dense, 1 = A is 2:4 structured-sparse */
  int64_t M, N, K;          /* logical (dense-equivalent) sizes */
  int64_t lda, ldb, ldc;
  const void* A;
  const void* B;
  void* C;
  const void* sfa;
  const void* sfb;
  const void* meta;
  float alpha;              /* per-tensor scale_a * scale_b, applied in the epilogue */
  int32_t cta_group;        /* 0 = auto, 1, 2 */
  int32_t ab_mode;          /* 0 = SS (A from SMEM), 1 = TS (A from TMEM) */
  int32_t tile_n;           /* 0 = auto; else N extent of one CTA-group tile */
  int32_t stages;           /* 0 = auto; SMEM ring depth */
  int32_t max_ctas;         /* 0 = one persistent CTA per SM; else cap */
  int32_t meta_layout;      /* sparse: 0 = canonical (b2g_compress_24 output; converted
                               per call in the handle's scratch), 1 = engine layout
                               (b2g_sparse_meta_prepare output, used as is) */
  int32_t raster_m;         /* 0 = auto; tile rows per raster group (L2 reuse) */
  int32_t m_sub;            /* 0 = auto, 1, 2 = 128-row A sub-tiles per CTA that share one
                               B tile (2 halves B's bytes per MMA; one accumulator).  Auto
                               picks 2 for sparse and block-scaled shapes with a full grid
                               of tiles, and for dense SS f16 / f8f6f4 pair tiles of 256
                               columns with K >= 8192 and at least 4 waves of 512-row
                               tiles; dense takes 2 on request up to tile_n 256 */
  int32_t split_tail;       /* 0 = auto, 1 = off, 2..4 = at most that many K splits of
                               each tile of the last, partial wave (one accumulator
                               buffer, m_sub = 2, never splits).  Splits use the
                               handle's workspace: calls of one handle on different
                               streams must not overlap */
  int32_t b_format;         /* 0 = B has A's format; else B's own format, where A and B
                               are both kind::f8f6f4 element types (E4M3, E5M2, E2M1,
                               E2M3, E3M2): the kind takes any pair of them.  No other
                               kind mixes A and B types */
  int32_t mx_scale;         /* 1 = OCP MX block scaling of those kind::f8f6f4 element
                               formats (A's and B's): one E8M0 scale per 32 K in sfa /
                               sfb ([M][K/32], [N][K/32]), through kind::mxf8f6f4 (what
                               B2G_FMT_MXF8 is for e4m3); operands from b2g_quantize_mx.
                               With sparse = 1 (e4m3, e5m2, or B2G_FMT_MXF8): 2:4-sparse
                               A on kind::mxf8f6f4 (tcgen05.mma.sp ... block_scale), A
                               the compressed codes, meta as for the 8-bit kinds; a
                               sparse MMA applies ONE scale per row to its 64 dense K
                               (32 kept elements of A), so sfa / sfb then hold one E8M0
                               per 64 K ([M][K/64], [N][K/64]; b2g_quantize_mx_block
                               with block 64), K % 64 == 0; m_sub 1 by default (2
                               needs tile_n <= 192) */
  int32_t instruction;      /* 0 = tcgen05.mma; 1 = the weight-stationary tcgen05.mma.ws
                               (.ws.sp for sparse = 1), the reference's INSTRUCTION=ws
                               (tcgen05_sparse_mma/tcgen05_sparse_mma.cu:80-81,343-483;
                               umma_throughput has no .ws): cta_group 1 (0 picks it),
                               SS, m_sub 1, tile_n 64 / 128 / 256 (auto: 256 dense,
                               128 sparse for N >= 256), the kinds without block
                               scaling (bf16, fp16, tf32, the f8f6f4 types, s8, u8) */
} b2g_gemm_desc;

/* Lifecycle.  b2g_create replaces the per-process setup of every reference
 * main (umma_tput.cu:547-563, tma2d_tput.cu:147-165). */
B2G_API b2g_status b2g_create(int device, b2g_handle** out);
B2G_API b2g_status b2g_destroy(b2g_handle* h);
B2G_API const char* b2g_status_string(b2g_status s);
B2G_API const char* b2g_last_error(const b2g_handle* h);
B2G_API int b2g_abi_version(void);

/* Device facts read at b2g_create: SM count, clock (kHz), compute capability. */
B2G_API b2g_status b2g_device_info(const b2g_handle* h, int* sm_count, int* clock_khz,
                           int* cc_major, int* cc_minor);

/* GEMM.  Replaces the MMA issue loop of umma_throughput/umma_tput.cu:413-522 and
 * tcgen05_sparse_mma/tcgen05_sparse_mma.cu:343-516 with a full tiled GEMM. */
B2G_API b2g_status b2g_gemm(b2g_handle* h, const b2g_gemm_desc* d, void* stream);

/* The launch configuration b2g_gemm would use for `d` on a device with sm_count
 * SMs, decided on the host without a device: for introspection and tests.
 * max_clusters caps the co-resident clusters (0: sm_count / cta_group; b2g_gemm
 * passes its occupancy query's answer for cta_group 2).  Only shapes and options
 * are checked, not pointers; msg (may be NULL, msg_len bytes) receives the reason
 * of a non-OK status, the same text b2g_last_error reports for b2g_gemm. */
typedef struct b2g_gemm_plan {
  int32_t variant;       /* 0 dense, 1 2:4 sparse, 2 NVFP4, 3 MXFP8, 4 MXFP4, 5 2:4-sparse MX
                            (kind::mxf8f6f4 .sp), 6 4:8-sparse MXFP4 (kind::mxf4 .sp), 7
                            4:8-sparse NVFP4 (kind::mxf4nvf4 block16 .sp) */
  int32_t kind;          /* tcgen05 kind, b2g_encode_idesc numbering */
  int32_t cta_group;
  int32_t tile_m;        /* A rows of one (pair) tile: 128 x m_sub x cta_group */
  int32_t tile_n;
  int32_t m_sub;
  int32_t stages;        /* shared-memory ring depth */
  int32_t smem_bytes;    /* dynamic shared memory per CTA */
  int32_t tmem_columns;  /* TMEM columns allocated per CTA */
  int32_t num_m_tiles, num_n_tiles, k_blocks;
  int32_t raster_m;      /* tile rows per raster group */
  int32_t tail_start;    /* first tile of the split tail (= tiles when none) */
  int32_t tail_split;    /* K splits of each tail tile (1 = none) */
  int32_t units;         /* work units of the persistent schedule */
  int32_t clusters;      /* persistent clusters launched: grid = clusters x cta_group */
  int32_t threads;       /* threads per CTA */
  int32_t k_atoms;       /* 128-byte K atoms per ring slot (k_blocks counts slots): 2 for
                            dense SS tiles up to 128 columns whose ring keeps 4 stages */
  int32_t instruction;   /* 0 tcgen05.mma, 1 tcgen05.mma.ws */
  int32_t reserved[2];
} b2g_gemm_plan;
B2G_API b2g_status b2g_plan_gemm(const b2g_gemm_desc* d, int sm_count, int max_clusters,
                         b2g_gemm_plan* out, char* msg, int msg_len);

/* End-to-end GEMM on HOST buffers: the descriptor's A, B, C (and sfa, sfb, meta)
 * are host pointers (page-locked for full copy speed).  Copies the operands into
 * the handle's device workspace (grown on demand and kept), runs b2g_gemm and
 * copies C back, all on `stream`, then synchronizes `stream` and reports device
 * errors like b2g_check.  This is the host-buffer path of the reference's mains,
 * which fill host memory and cudaMemcpy it to the device (tma2d_tput.cu:169-176). */
B2G_API b2g_status b2g_gemm_host(b2g_handle* h, const b2g_gemm_desc* d, void* stream);

/* Reads the handle's device error word (after synchronizing `stream`) and
 * clears it; B2G_ERR_TIMEOUT if any kernel recorded a wait timeout. */
B2G_API b2g_status b2g_check(b2g_handle* h, void* stream);

/* Limit, in nanoseconds, of every kernel-side bounded wait of the handle's later
 * b2g_gemm and b2g_selftest_wait launches: 1000 .. 2e9, or 0 for the default of
 * 2 s.  It only has to exceed the longest legitimate wait, which is one output
 * tile's main loop (tens of microseconds).  The reference's waits are unbounded
 * spins (umma_throughput/umma_tput.cu:510-520). */
B2G_API b2g_status b2g_set_wait_limit(b2g_handle* h, uint64_t ns);

/* Failure-detection self-test (no counterpart in the reference, whose waits
 * cannot expire: umma_throughput/umma_tput.cu:510-520).  One warp waits, through
 * the GEMM's bounded-wait code and with the handle's wait limit, on something
 * that nothing completes: mode 0, a phase of an mbarrier no thread arrives at
 * (the GEMM's ring and accumulator barriers); mode 1, a global word no thread
 * sets (the GEMM's split-tail flags).  Nothing else is in flight.  The wait
 * expires, the kernel records the timeout in the handle's error word and
 * returns.  The call synchronises `stream` and returns b2g_check's status:
 * B2G_ERR_TIMEOUT when the bound worked; the error word is cleared, so the handle
 * is ready for the next GEMM.  *elapsed_ns (nullable) receives the device time
 * from the start of the wait to its expiry. */
B2G_API b2g_status b2g_selftest_wait(b2g_handle* h, int mode, uint64_t* elapsed_ns, void* stream);

/* 2:4 compressor.  Not in the reference, which writes the constant metadata
 * word 0x44444444 (tcgen05_sparse_mma.cu:327-332).  d_dense is bf16 row-major
 * [M][K] with at most 2 non-zeros in every aligned group of 4 along K.
 * Outputs: d_comp bf16 [M][K/2] (kept values in ascending index order) and
 * d_meta, one uint32 per 32 dense K elements per row ([M][K/32] words, row
 * major); group g (0..7) of the word occupies bits [4g, 4g+4) as
 * idx0 | idx1 << 2 with idx0 < idx1.  K must be a multiple of 32.
 * Groups with fewer than 2 non-zeros keep the lowest free indices.
 * The engine's own TMEM metadata layout is derived from this canonical form
 * inside b2g_gemm. */
B2G_API b2g_status b2g_compress_24(b2g_handle* h, const void* d_dense, int64_t M, int64_t K,
                           void* d_comp, void* d_meta, void* stream);

/* 2:4 prune / compress / metadata preparation for every A format the sparse GEMM
 * takes: 16-bit (B2G_FMT_BF16, B2G_FMT_F16: the same as b2g_prune_24,
 * b2g_compress_24 and b2g_sparse_meta_prepare) and 8-bit (B2G_FMT_E4M3, E5M2 on
 * kind::f8f6f4; B2G_FMT_S8, U8 on kind::i8).  The reference issues
 * tcgen05.mma.sp for these kinds with the constant metadata word 0x44444444
 * (tcgen05_sparse_mma/tcgen05_sparse_mma.cu:327-332,343-483); it prunes and
 * compresses nothing.  The 8-bit forms use the same group counter, the same
 * canonical metadata ([M][K/32] words, group g at bits 4g..4g+3) and a compressed
 * A of [M][K/2] bytes; an fp8 element counts as zero when its 7 low bits are
 * (0x80 is -0), an integer when all 8 are.  b2g_prune_24_format needs cols % 4 and
 * a 4-byte aligned matrix; b2g_compress_24_format K % 32 and 16-byte alignment.
 * B2G_FMT_TF32 (kind::tf32 .sp) is structured 1:2: one of every two K elements
 * kept; its canonical metadata is [M][K/16] words (each pair described as a group
 * of four 16-bit halves), prune needs cols % 2, compress and meta_prepare K % 16.
 * B2G_FMT_E2M1, E2M3, E3M2 (packed fp4 / fp6 of kind::f8f6f4) are 2:4 element by
 * element (-0 counts as zero), compressed [M][K/2] elements packed the same way,
 * metadata as for the 8-bit codes; prune needs cols % 16, compress K % 32.
 * B2G_FMT_MXF4 and B2G_FMT_NVFP4 (kind::mxf4 / mxf4nvf4 .sp) are 4:8 in pairs: a byte
 * of packed e2m1 (two elements) is the unit, 2 of every 4 bytes kept (a byte is zero when both of its
 * elements are), compressed [M][K/4] bytes, canonical metadata [M][K/64] words
 * (the 8-bit words over the bytes); prune needs cols % 8, compress K % 64.  Every
 * K here counts elements. */
B2G_API b2g_status b2g_prune_24_format(b2g_handle* h, int format, void* d, int64_t rows,
                                       int64_t cols, int64_t row0, uint64_t seed, void* stream);
B2G_API b2g_status b2g_compress_24_format(b2g_handle* h, int format, const void* d_dense,
                                          int64_t M, int64_t K, void* d_comp, void* d_meta,
                                          void* stream);
B2G_API size_t b2g_sparse_meta_bytes_format(int format, int64_t M, int64_t K);
B2G_API b2g_status b2g_sparse_meta_prepare_format(b2g_handle* h, int format, const void* d_meta,
                                                  int64_t M, int64_t K, void* d_ready,
                                                  void* stream);

/* 2:4 sparse bf16 GEMM for callers that cannot allocate device memory (no
 * counterpart in the reference).  b2g_gemm needs a handle, and handles own
 * device memory; a plugin inside a framework whose caching allocator owns the
 * GPU's memory, or a latency-critical loop where cudaMalloc/cudaFree may
 * synchronise the device, cannot make those allocations.  This entry point takes
 * no handle and allocates nothing: it runs on the current device, and its
 * scratch (an error word and the metadata in the engine's layout) lives in a
 * static device array of the library, 16 MiB of metadata at most.  The metadata
 * takes ceil(M/128) * ceil(K/128) * 2048 bytes, so it accepts
 * ceil(M/128) * ceil(K/128) <= 8192 (e.g. M = 8192, K = 16384) and rejects larger
 * problems with B2G_ERR_INVALID.  The descriptor is that of b2g_gemm with format = bf16,
 * sparse = 1, meta_layout = 0 (canonical metadata from b2g_compress_24); the
 * caller passes A (compressed), B, C and the metadata as device pointers.
 * The call synchronises `stream` and returns B2G_ERR_TIMEOUT if a kernel wait
 * expired.  All calls share one scratch array: calls that overlap on the GPU
 * race and must be serialised.  The first call on a device looks up the array's
 * device address (again after the device's context changes, e.g. after
 * cudaDeviceReset) and should come before any stream capture.  *err_msg
 * (nullable) receives a message for any non-OK status. */
B2G_API b2g_status b2g_gemm_sparse_noalloc(const b2g_gemm_desc* d, void* stream,
                                           const char** err_msg);

/* Converts canonical metadata ([M][K/32] words) into the engine's TMEM-ready
 * layout, for callers that reuse one sparse operand across many GEMMs
 * (b2g_gemm_desc.meta_layout = 1).  d_ready holds b2g_sparse_meta_bytes(M, K)
 * bytes.  The reference has no counterpart: it writes 0x44444444 straight into
 * TMEM (tcgen05_sparse_mma.cu:327-332). */
B2G_API size_t b2g_sparse_meta_bytes(int64_t M, int64_t K);
B2G_API b2g_status b2g_sparse_meta_prepare(b2g_handle* h, const void* d_meta, int64_t M, int64_t K,
                                   void* d_ready, void* stream);

/* Seeded synthetic operands.  Same values as the CPU oracle's
 * generator (splitmix64 counter hash).  dist: 0 = uniform[-1,1), 1 = normal(0,1)
 * (Irwin-Hall sum of 12 uniforms, so CPU and GPU agree bit for bit).
 * d_out receives rows [row0, row0+rows) of a matrix `cols` wide; element (r, c)
 * uses counter r*cols + c, so an M-row shard is the matching slice of the whole
 * matrix.  (The reference fills its tiles with byte patterns instead:
 * umma_tput.cu:257-266, tma2d_tput.cu:169-173.) */
B2G_API b2g_status b2g_fill_f32(b2g_handle* h, float* d_out, int64_t rows, int64_t cols,
                        int64_t row0, uint64_t seed, int dist, void* stream);
/* fp32 -> operand format (round to nearest even, saturating):
 *   B2G_FMT_BF16: 2 bytes per element; B2G_FMT_E4M3: 1 byte (clip to +-448);
 *   B2G_FMT_NVFP4: packed e2m1, two per byte (even K index in the low nibble),
 *   plus d_sf: one ue4m3 scale per 16 elements = e4m3(amax/6), rows x cols/16;
 *   B2G_FMT_S8: 1 byte, round to nearest even, saturate to [-128, 127];
 *   B2G_FMT_U8: 1 byte, round to nearest even, saturate to [0, 255];
 *   B2G_FMT_F16: 2 bytes, IEEE binary16, round to nearest even (overflow to inf);
 *   B2G_FMT_TF32: 4 bytes, fp32 rounded to 10 mantissa bits (nearest even);
 *   B2G_FMT_E5M2: 1 byte (clip to +-57344);
 *   B2G_FMT_E2M1 / E2M3 / E3M2: packed along the row, each 16 elements in 8 bytes
 *   (4 bits each) or 12 bytes (6 bits each), element i of a group at bits
 *   [4i, 4i+4) / [6i, 6i+6) little-endian; clip to +-6 / +-7.5 / +-28; cols % 16;
 *   B2G_FMT_MXF8 / B2G_FMT_MXF4: OCP MX v1.0, e4m3 bytes / packed e2m1, plus d_sf:
 *   one E8M0 byte per 32 elements, 2^s with s = clamp(floor(log2(amax)) - emax,
 *   -127, 127), emax 8 (e4m3) or 2 (e2m1); rows x cols/32.
 * d_in is rows x cols fp32 row-major. */
B2G_API b2g_status b2g_quantize(b2g_handle* h, int format, const float* d_in, int64_t rows,
                        int64_t cols, void* d_out, void* d_sf, void* stream);
/* OCP MX v1.0 block-32 quantisation to any kind::f8f6f4 element format
 * (B2G_FMT_E4M3, E5M2, E2M1, E2M3, E3M2): one E8M0 scale per 32 elements,
 * 2^s with s = clamp(floor(log2(amax)) - emax, -127, 127), emax 8 / 15 / 2 / 2 / 4;
 * elements x * 2^-s converted as b2g_quantize converts them (saturating, nearest
 * even) and stored in that format's layout (e2m1 / fp6 packed).  d_sf receives
 * rows x cols/32 bytes; cols % 32 == 0, d_in 16-byte aligned. */
B2G_API b2g_status b2g_quantize_mx(b2g_handle* h, int elem_format, const float* d_in, int64_t rows,
                           int64_t cols, void* d_out, void* d_sf, void* stream);
/* The same with one scale per `block` elements, 32 (b2g_quantize_mx) or 64: the scale
 * block of the 2:4-sparse kind::mxf8f6f4 GEMM (sparse = 1 with mx_scale), whose MMAs
 * apply one scale per row to 64 dense K.  d_sf receives rows x cols/block bytes;
 * cols % block == 0.  The reference's sparse probe writes one constant scale per row
 * (tcgen05_sparse_mma/tcgen05_sparse_mma.cu:320-325). */
B2G_API b2g_status b2g_quantize_mx_block(b2g_handle* h, int elem_format, const float* d_in,
                                         int64_t rows, int64_t cols, int block, void* d_out,
                                         void* d_sf, void* stream);
/* NVFP4 quantisation (as b2g_quantize with B2G_FMT_NVFP4: packed e2m1, one ue4m3 scale
 * e4m3(amax/6) per block) with a block of 16 or 32 elements: 32 is the scale block of
 * the 4:8-sparse NVFP4 GEMM (kind::mxf4nvf4 block16 .sp), whose MMA reads four scales
 * per row over its 128 dense K.  d_sf receives rows x cols/block bytes; cols % block
 * == 0.  The reference's sparse probe writes constant scale words
 * (tcgen05_sparse_mma/tcgen05_sparse_mma.cu:320-325). */
B2G_API b2g_status b2g_quantize_nvfp4_block(b2g_handle* h, const float* d_in, int64_t rows,
                                            int64_t cols, int block, void* d_out, void* d_sf,
                                            void* stream);
/* Zeroes 2 of every 4 consecutive elements along each row of a rows x cols bf16
 * matrix holding rows [row0, row0+rows), at positions drawn from `seed` (group
 * counter r*(cols/4)+g for absolute row r). */
B2G_API b2g_status b2g_prune_24(b2g_handle* h, void* d_bf16, int64_t rows, int64_t cols,
                        int64_t row0, uint64_t seed, void* stream);

/* TMA 2D load latency probe.  Replaces tma2d_latency/tma2d_lat.cu:43-100: SMs x
 * ctas_per_sm CTAs each issue ONE box_w x box_h fp32 box load of d_data (width x
 * height, row-major) at rows row0 + cta * box_h, and write to d_cycles[cta] the
 * clock64 cycles from before the issue to the mbarrier's completion (0xFFFFFFFF
 * if the bounded wait expired).  Each CTA takes all the shared memory a block may
 * opt into, whatever the box (which must fit in it).  The caller flushes L2 between launches and picks row0 so that
 * a launch reads rows that no earlier launch read.  Synchronous (returns after the
 * launch, with b2g_check's status). */
B2G_API b2g_status b2g_tma2d_latency(b2g_handle* h, const float* d_data, uint64_t width,
                             uint64_t height, int box_w, int box_h, int ctas_per_sm,
                             int64_t row0, uint32_t* d_cycles, void* stream);

/* 1D bulk-copy streaming probe.  Replaces tma_throughput/tma_tput.cu:41-76: one
 * thread per CTA streams `bytes` of d_data (16-byte aligned) in load_bytes chunks
 * (a multiple of 16) with cp.async.bulk through a num_stages-slot mbarrier ring
 * (num_stages x load_bytes <= 227 KB); grid = SMs x ctas_per_sm; bytes must be a
 * multiple of load_bytes.  *elapsed_ms (may be NULL) is the CUDA-event time of
 * the launch alone: the kernel's set-up (shared-memory attribute, module load)
 * runs before the start event.  Time a second call for a warm figure. */
B2G_API b2g_status b2g_stream_bulk1d(b2g_handle* h, const void* d_data, uint64_t bytes,
                             int ctas_per_sm, int num_stages, uint32_t load_bytes,
                             float* elapsed_ms, void* stream);

/* TMA 2D streaming probe.  Replaces tma2d_throughput/tma2d_tput.cu:50-134: one
 * warp per CTA streams d_data (fp32, width x height) through a num_stages-slot
 * mbarrier ring of box_w x box_h tiles; grid = SMs x ctas_per_sm.
 * *elapsed_ms (may be NULL) is the CUDA-event time of the launch alone, as for
 * b2g_stream_bulk1d. */
B2G_API b2g_status b2g_stream_tma2d(b2g_handle* h, const float* d_data, uint64_t width,
                            uint64_t height, int ctas_per_sm, int num_stages,
                            int box_w, int box_h, float* elapsed_ms, void* stream);

/* Instruction-rate probe for the RESULT line of umma_tput.cu:539-542 and
 * tcgen05_sparse_mma.cu:531-537 / :592-595.  Runs the engine's MMA issue path on
 * one resident tile: iters batches of depth MMAs, each batch committed to an
 * mbarrier and waited.  mode 0 = throughput, 1 = latency (median of 100).
 * Outputs clock64 cycles of the issuing CTA and the MMA count. */
typedef struct b2g_probe_desc {
  int32_t kind;        /* reference KIND_ID: 0 tf32, 1 f16, 2 f8f6f4, 3 i8, 4 mxf8f6f4, 5 mxf4, 6 mxf4nvf4 */
  int32_t a_type;      /* reference A_TYPE_CODE */
  int32_t b_type;      /* reference B_TYPE_CODE */
  int32_t a_bits, b_bits;
  int32_t sparse;
  int32_t ab_mode;     /* 0 SS, 1 TS */
  int32_t cta_group;
  int32_t m, n, k;     /* instruction shape */
  int32_t depth;
  int32_t scale_type;  /* 1 ue8m0, 0 ue4m3 */
  int32_t mode;        /* 0 throughput, 1 latency */
  int32_t iters;       /* 0 = 1000 */
  int32_t instruction; /* 0 mma, 1 ws */
} b2g_probe_desc;
B2G_API b2g_status b2g_probe_mma(b2g_handle* h, const b2g_probe_desc* p, uint64_t* cycles,
                         uint64_t* total_mmas, uint64_t* median_cycles);

/* Progress trace (diagnostics; no counterpart in the reference, whose kernels
 * are observed only through clock64 and ncu).  b2g_trace_enable allocates a
 * host-mapped buffer of max_ctas x 16 words into which later b2g_gemm launches
 * write per-CTA progress counters (slot meanings: csrc/b2g_gemm.h TraceSlot);
 * max_ctas = 0 disables tracing.  b2g_trace_read copies the words out with plain
 * host loads, so it works while a kernel is still running. */
B2G_API b2g_status b2g_trace_enable(b2g_handle* h, int max_ctas);
B2G_API b2g_status b2g_trace_read(const b2g_handle* h, uint32_t* out, int nwords);

/* Descriptor encoders (host-side, no GPU needed), the engine's own encodings of
 * the bit layouts the reference builds at umma_tput.cu:147-156 and :190-255 and
 * tcgen05_sparse_mma.cu:191-228.  Exposed so tests can pin them. */
B2G_API uint32_t b2g_encode_idesc(int kind, int a_type, int b_type, int m, int n,
                          int sparse, int scale_type);
B2G_API uint64_t b2g_encode_smem_desc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                              int swizzle /* 0 none, 2 = 128B */);

#ifdef __cplusplus
}
#endif
#endif /* B2G_H */
