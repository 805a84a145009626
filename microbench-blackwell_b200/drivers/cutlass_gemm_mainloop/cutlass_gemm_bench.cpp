// Drop-in main for cutlass_gemm_mainloop/ (reference:
// cutlass_gemm_mainloop/cutlass_gemm_bench.cu:131-233).
//
// The reference times one CTA of a CUTLASS sm100 1-SM GEMM (cluster 1x1x1) on
// M = TILE_M, N = TILE_N, K = 131072 (zeroed bf16 or e4m3 operands, bf16 D), one
// warm-up and 20 timed launches back to back, and prints
//   M,N,K,TILE_M,TILE_N,TILE_K,STAGES,dtype,time_ms,TFLOPS
// This main does the same with the engine's cta_group::1 GEMM on one CTA
// (b2g_gemm, max_ctas = 1).  The engine's shapes: a 128-row CTA tile (TILE_M = 64
// runs it with the upper 64 rows zero-filled, i.e. at the cost of a 128-row
// tile, which is also what the M = 64 MMA costs per row), TILE_N a multiple of
// 32 up to 256, and a K slot of 128 bytes (TILE_K = 64 for bf16, 128 for e4m3).
// Other shapes print "Cannot implement" and exit 1, as the reference does when
// CUTLASS rejects a configuration; STAGES = 0 picks the deepest ring that fits.
#include <cuda_runtime.h>

#include <cstdio>

#include "b2g.h"

#ifndef TILE_M
#define TILE_M 128
#endif
#ifndef TILE_N
#define TILE_N 128
#endif
#ifndef TILE_K
#define TILE_K 64
#endif
#ifndef STAGES
#define STAGES 0
#endif
#ifndef DTYPE_ID
#define DTYPE_ID 0
#endif

#if DTYPE_ID == 0
static const char* dtype_str = "BF16";
static const int kFormat = B2G_FMT_BF16;
static const int kElemBytes = 2;
#elif DTYPE_ID == 1
static const char* dtype_str = "FP8_E4M3";
static const int kFormat = B2G_FMT_E4M3;
static const int kElemBytes = 1;
#else
#error "Unknown DTYPE_ID (0=BF16, 1=FP8_E4M3)"
#endif

static constexpr int K_DIM = 131072;
static constexpr int WARMUP_ITERS = 1;
static constexpr int BENCH_ITERS = 20;

static int cannot(const char* why) {
  fprintf(stderr, "Cannot implement: TILE_M=%d TILE_N=%d TILE_K=%d STAGES=%d dtype=%s error=%s\n",
          TILE_M, TILE_N, TILE_K, STAGES, dtype_str, why);
  return 1;
}

int main() {
  const int M = TILE_M, N = TILE_N, K = K_DIM;
  if (TILE_M != 64 && TILE_M != 128) return cannot("the engine's 1-SM tile has 128 rows");
  if (TILE_N < 32 || TILE_N > 256 || TILE_N % 32) return cannot("TILE_N must be 32..256, step 32");
  if (TILE_K * kElemBytes != 128) return cannot("the engine's K slot is 128 bytes");

  b2g_handle* h = nullptr;
  if (b2g_create(0, &h) != B2G_OK) {
    fprintf(stderr, "Init failed: no sm_100 device\n");
    return 1;
  }
  void *A = nullptr, *B = nullptr, *D = nullptr;
  if (cudaMalloc(&A, (size_t)M * K * kElemBytes) != cudaSuccess ||
      cudaMalloc(&B, (size_t)N * K * kElemBytes) != cudaSuccess ||
      cudaMalloc(&D, (size_t)M * N * 2) != cudaSuccess) {
    fprintf(stderr, "Init failed: %s\n", cudaGetErrorString(cudaGetLastError()));
    return 1;
  }
  cudaMemset(A, 0, (size_t)M * K * kElemBytes);
  cudaMemset(B, 0, (size_t)N * K * kElemBytes);

  b2g_gemm_desc d = {};
  d.format = kFormat;
  d.M = M;
  d.N = N;
  d.K = K;
  d.lda = K;
  d.ldb = K;
  d.ldc = N;
  d.A = A;
  d.B = B;
  d.C = D;
  d.alpha = 1.0f;
  d.cta_group = 1;
  d.tile_n = TILE_N;
  d.stages = STAGES;
  d.max_ctas = 1;
  if (b2g_gemm(h, &d, nullptr) != B2G_OK) return cannot(b2g_last_error(h));
  for (int i = 1; i < WARMUP_ITERS; ++i) b2g_gemm(h, &d, nullptr);
  if (b2g_check(h, nullptr) != B2G_OK) {
    fprintf(stderr, "Init failed: %s\n", b2g_last_error(h));
    return 1;
  }

  cudaEvent_t start, stop;
  cudaEventCreate(&start);
  cudaEventCreate(&stop);
  cudaEventRecord(start);
  for (int i = 0; i < BENCH_ITERS; ++i) b2g_gemm(h, &d, nullptr);
  cudaEventRecord(stop);
  cudaEventSynchronize(stop);
  if (b2g_check(h, nullptr) != B2G_OK) {
    fprintf(stderr, "Kernel failed: %s\n", b2g_last_error(h));
    return 1;
  }
  float total_ms = 0.0f;
  cudaEventElapsedTime(&total_ms, start, stop);
  const double avg_ms = total_ms / BENCH_ITERS;
  const double tflops = 2.0 * M * N * (double)K / (avg_ms * 1e-3) / 1e12;
  printf("%d,%d,%d,%d,%d,%d,%d,%s,%g,%g\n", M, N, K, TILE_M, TILE_N, TILE_K, STAGES, dtype_str,
         avg_ms, tflops);
  cudaEventDestroy(start);
  cudaEventDestroy(stop);
  cudaFree(A);
  cudaFree(B);
  cudaFree(D);
  b2g_destroy(h);
  return 0;
}
