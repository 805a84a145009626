// Drop-in main for tma_throughput/ (reference: tma_throughput/tma_tput.cu:90-119).
//
// Same macros and behaviour: about 2 GB (rounded to whole rounds of
// SMs x CTAS_PER_SM x NUM_STAGES loads of LOAD_SIZE bytes) of host-initialised
// fp32 copied to the device, L2 flushed, then one untimed warm-up launch, the L2 flush and the timed streaming launch: one thread
// per CTA, SMs x CTAS_PER_SM CTAs, NUM_STAGES cp.async.bulk loads of LOAD_SIZE
// bytes in flight per CTA.  The streaming kernel is the last launch, so that
// `ncu --metrics ...` on this process reports its counters.  Also prints the
// event-timed bandwidth.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <vector>

#include "b2g.h"

#ifndef CTAS_PER_SM
#error "CTAS_PER_SM must be defined"
#endif
#ifndef NUM_STAGES
#error "NUM_STAGES must be defined"
#endif
#ifndef LOAD_SIZE
#error "LOAD_SIZE must be defined"
#endif
static_assert(LOAD_SIZE % 16 == 0, "LOAD_SIZE must be a multiple of 16 bytes");

#define CHECK(expr)                                                                     \
  do {                                                                                  \
    cudaError_t e__ = (expr);                                                           \
    if (e__ != cudaSuccess) {                                                           \
      fprintf(stderr, "CUDA error %s:%d: %s\n", __FILE__, __LINE__, cudaGetErrorString(e__)); \
      return 1;                                                                         \
    }                                                                                   \
  } while (0)

int main() {
  const size_t kMaxVolume = 2ull << 30;
  b2g_handle* h = nullptr;
  b2g_status st = b2g_create(0, &h);
  if (st != B2G_OK) {
    fprintf(stderr, "Kernel failed: %s\n", b2g_status_string(st));
    return 1;
  }
  int sms = 0, l2 = 0;
  b2g_device_info(h, &sms, nullptr, nullptr, nullptr);
  CHECK(cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, 0));
  const size_t round = (size_t)sms * CTAS_PER_SM * (size_t)LOAD_SIZE * NUM_STAGES;
  const size_t bytes = kMaxVolume / round * round;
  std::vector<float> host(bytes / sizeof(float));
  srand((unsigned)NUM_STAGES * LOAD_SIZE);
  for (auto& x : host) x = (float)rand();
  void* d = nullptr;
  CHECK(cudaMalloc(&d, bytes));
  CHECK(cudaMemcpy(d, host.data(), bytes, cudaMemcpyHostToDevice));
  // one untimed warm-up launch (first-launch costs stay out of the timed one)
  st = b2g_stream_bulk1d(h, d, bytes, CTAS_PER_SM, NUM_STAGES, LOAD_SIZE, nullptr, nullptr);
  if (st != B2G_OK) {
    fprintf(stderr, "Kernel failed: %s\n", b2g_last_error(h));
    return 1;
  }
  void* flush = nullptr;
  CHECK(cudaMalloc(&flush, (size_t)l2));
  CHECK(cudaMemset(flush, 0xA5, (size_t)l2));
  CHECK(cudaDeviceSynchronize());
  CHECK(cudaFree(flush));
  float ms = 0.0f;
  st = b2g_stream_bulk1d(h, d, bytes, CTAS_PER_SM, NUM_STAGES, LOAD_SIZE, &ms, nullptr);
  if (st != B2G_OK) {
    fprintf(stderr, "Kernel failed: %s\n", b2g_last_error(h));
    return 1;
  }
  printf("streamed %.3f GB in %.3f ms: %.1f GB/s (event time)\n", bytes / 1e9, ms,
         bytes / 1e6 / ms);
  CHECK(cudaFree(d));
  b2g_destroy(h);
  return 0;
}
