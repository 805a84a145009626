// Drop-in main for tma2d_latency/ (reference: tma2d_latency/tma2d_lat.cu:103-244).
//
// Same macros and output: NUM_ITERS launches of SMs x CTAS_PER_SM CTAs, each CTA
// timing ONE SMEM_WIDTH x SMEM_HEIGHT fp32 TMA 2D load with clock64, every launch
// after an L2 flush and on rows no earlier launch read; per launch the min /
// median / max over the CTAs go to stderr, then one more launch (rows 0..) gives
// the overall min and max, and stdout gets SUMMARY,<median of the launch
// medians>,<min>,<max>.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <vector>

#include "b2g.h"

#ifndef CTAS_PER_SM
#error "CTAS_PER_SM must be defined"
#endif
#ifndef SMEM_WIDTH
#error "SMEM_WIDTH must be defined"
#endif
#ifndef SMEM_HEIGHT
#error "SMEM_HEIGHT must be defined"
#endif
static_assert(SMEM_WIDTH <= 256 && SMEM_HEIGHT <= 256, "TMA box dimensions are at most 256");
static_assert(SMEM_WIDTH % 4 == 0, "box rows must be multiples of 16 bytes");

constexpr int NUM_ITERS = 10;

#define CHECK(expr)                                                                     \
  do {                                                                                  \
    cudaError_t e__ = (expr);                                                           \
    if (e__ != cudaSuccess) {                                                           \
      fprintf(stderr, "CUDA error %s:%d: %s\n", __FILE__, __LINE__, cudaGetErrorString(e__)); \
      return 1;                                                                         \
    }                                                                                   \
  } while (0)

#define B2G(h, expr)                                                                    \
  do {                                                                                  \
    b2g_status s__ = (expr);                                                            \
    if (s__ != B2G_OK) {                                                                \
      fprintf(stderr, "Kernel failed: %s: %s\n", b2g_status_string(s__), b2g_last_error(h)); \
      return 1;                                                                         \
    }                                                                                   \
  } while (0)

int main() {
  b2g_handle* h = nullptr;
  if (b2g_create(0, &h) != B2G_OK) {
    fprintf(stderr, "Init failed: no sm_100 device\n");
    return 1;
  }
  int sms = 0, l2 = 0, max_smem = 0;
  b2g_device_info(h, &sms, nullptr, nullptr, nullptr);
  CHECK(cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, 0));
  CHECK(cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, 0));
  const int blocks = sms * CTAS_PER_SM;
  const size_t tile_bytes = (size_t)SMEM_WIDTH * SMEM_HEIGHT * sizeof(float);
  const uint64_t height = (uint64_t)NUM_ITERS * blocks * SMEM_HEIGHT;
  fprintf(stderr,
          "Config: CTAS_PER_SM=%d SMEM_WIDTH=%d SMEM_HEIGHT=%d TILE_BYTES=%zu\n"
          "  num_sms=%d l2_size=%.2f MiB max_smem=%.1f KiB\n",
          CTAS_PER_SM, SMEM_WIDTH, SMEM_HEIGHT, tile_bytes, sms, l2 / (1024.0 * 1024.0),
          max_smem / 1024.0);

  float* d_data = nullptr;
  CHECK(cudaMalloc(&d_data, (size_t)SMEM_WIDTH * height * sizeof(float)));
  // seeded values written on the device (the reference copies host rand() values)
  B2G(h, b2g_fill_f32(h, d_data, (int64_t)height, SMEM_WIDTH, 0, SMEM_WIDTH + SMEM_HEIGHT, 0,
                      nullptr));
  void* flush = nullptr;
  CHECK(cudaMalloc(&flush, (size_t)l2));
  uint32_t* d_cycles = nullptr;
  CHECK(cudaMalloc(&d_cycles, (size_t)blocks * sizeof(uint32_t)));
  std::vector<uint32_t> cyc(blocks);

  auto launch = [&](int64_t row0) -> int {
    CHECK(cudaMemset(flush, 0xA5, (size_t)l2));  // evict the data from L2
    CHECK(cudaDeviceSynchronize());
    B2G(h, b2g_tma2d_latency(h, d_data, SMEM_WIDTH, height, SMEM_WIDTH, SMEM_HEIGHT, CTAS_PER_SM,
                             row0, d_cycles, nullptr));
    CHECK(cudaMemcpy(cyc.data(), d_cycles, (size_t)blocks * sizeof(uint32_t),
                     cudaMemcpyDeviceToHost));
    std::sort(cyc.begin(), cyc.end());
    if (cyc.back() == 0xFFFFFFFFu) {
      fprintf(stderr, "Kernel failed: a load did not complete\n");
      return 1;
    }
    return 0;
  };

  std::vector<uint32_t> medians(NUM_ITERS);
  for (int i = 0; i < NUM_ITERS; ++i) {
    if (launch((int64_t)i * blocks * SMEM_HEIGHT)) return 1;
    medians[i] = cyc[blocks / 2];
    fprintf(stderr, "  iter %d: min=%u med=%u max=%u cycles\n", i, cyc.front(), medians[i],
            cyc.back());
  }
  std::sort(medians.begin(), medians.end());
  const uint32_t overall_med = medians[NUM_ITERS / 2];
  if (launch(0)) return 1;
  printf("SUMMARY,%u,%u,%u\n", overall_med, cyc.front(), cyc.back());

  cudaFree(d_cycles);
  cudaFree(flush);
  cudaFree(d_data);
  b2g_destroy(h);
  return 0;
}
