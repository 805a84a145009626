// Drop-in main for umma_latency/ (reference: umma_latency/umma_lat.cu:483-563).
//
// Compile-time configuration through the same macros, the same stdout contract:
//   RESULT,<M>,<N>,<K>,<median cycles>
//   Done!
// and exit 0; on error "CUDA Error: <message>" and exit 1.  The measurement is the
// engine's tcgen05 probe (b2g_probe_mma) in latency mode: 100 round trips of one
// MMA issued, committed and waited on, timed with clock64; the median is printed.
#include <cstdio>

#include "b2g.h"

#ifndef MMA_FORMAT
#error "MMA_FORMAT must be defined (0=BF16, 1=E4M3, 2=S8, 3=F4, 4=MXF8, 5=MXF4)"
#endif
#ifndef MMA_M
#error "MMA_M must be defined (e.g., -DMMA_M=128)"
#endif
#ifndef MMA_N
#error "MMA_N must be defined (e.g., -DMMA_N=64)"
#endif
#ifndef MMA_K
#error "MMA_K must be defined (e.g., -DMMA_K=16)"
#endif
#ifndef CTA_GROUP
#error "CTA_GROUP must be defined (1=1SM, 2=2SM)"
#endif
#ifndef AB_LAYOUT
#error "AB_LAYOUT must be defined (0=SS_MODE, 1=TS_MODE)"
#endif
#if MMA_FORMAT < 0 || MMA_FORMAT > 5
#error "MMA_FORMAT must be 0..5"
#endif
#if MMA_FORMAT > 3 && MMA_M < 128
#error "MX_SCALED requires MMA_M >= 128 (M/128 descriptor encoding)"
#endif

int main() {
  // MMA_FORMAT -> tcgen05 kind, operand type codes, scale type (as in the
  // umma_throughput drop-in: E4M3 is type code 0, MXF4 runs mxf8f6f4 with e2m1)
  static const int kKind[6] = {1, 2, 3, 2, 4, 4};
  static const int kType[6] = {1, 0, 1, 5, 0, 5};
  static const int kScale[6] = {0, 0, 0, 0, 1, 1};
  b2g_handle* h = nullptr;
  b2g_status st = b2g_create(0, &h);
  if (st != B2G_OK) {
    printf("CUDA Error: %s\n", b2g_status_string(st));
    return 1;
  }
  b2g_probe_desc p = {};
  p.kind = kKind[MMA_FORMAT];
  p.a_type = p.b_type = kType[MMA_FORMAT];
  p.a_bits = p.b_bits = MMA_FORMAT == 0 ? 16 : (MMA_FORMAT == 3 || MMA_FORMAT == 5 ? 4 : 8);
  p.sparse = 0;
  p.ab_mode = AB_LAYOUT;
  p.cta_group = CTA_GROUP;
  p.m = MMA_M;
  p.n = MMA_N;
  p.k = MMA_K;
  p.depth = 1;
  p.scale_type = kScale[MMA_FORMAT];
  p.mode = 1;
  uint64_t cycles = 0, total = 0, median = 0;
  st = b2g_probe_mma(h, &p, &cycles, &total, &median);
  if (st != B2G_OK) {
    printf("CUDA Error: %s\n", b2g_last_error(h));
    b2g_destroy(h);
    return 1;
  }
  printf("RESULT,%d,%d,%d,%llu\n", MMA_M, MMA_N, MMA_K, (unsigned long long)median);
  b2g_destroy(h);
  printf("Done!\n");
  return 0;
}
