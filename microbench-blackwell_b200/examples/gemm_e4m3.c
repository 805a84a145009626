/* gemm_e4m3.c -- the C binding of one GEMM through libb2g: BASELINE cfg2 (e4m3
 * 8192^3, per-tensor scales 1/64, cta_group::2 256 x 256 tiles) on device buffers
 * the caller owns.
 *
 *   cc -I include -c microbench-blackwell_b200/examples/gemm_e4m3.c
 *   link: -L microbench-blackwell_b200/lib -lb2g
 */
#include <stddef.h>

#include "b2g.h"

/* dA: [8192][8192] e4m3 (row-major A), dB: [8192][8192] e4m3 (B stored [N][K]),
 * dC: [8192][8192] bf16; stream: a cudaStream_t or NULL.  Returns a b2g_status. */
int b2g_example_gemm_e4m3(const void* dA, const void* dB, void* dC, void* stream) {
  b2g_handle* h;
  if (b2g_create(/*device*/ 0, &h) != B2G_OK) return B2G_ERR_NO_DEVICE; /* no sm_100 GPU */
  b2g_gemm_desc d = {0};
  d.format = B2G_FMT_E4M3;
  d.M = d.N = d.K = 8192;
  d.lda = d.ldb = 8192; /* elements */
  d.ldc = 8192;
  d.A = dA; /* device pointers; B is [N][K] */
  d.B = dB;
  d.C = dC;
  d.alpha = 1.0f / 4096; /* scale_a * scale_b */
  d.cta_group = 2;       /* 0 = auto */
  d.tile_n = 256;
  b2g_status s = b2g_gemm(h, &d, stream); /* async on `stream` */
  if (s == B2G_OK) s = b2g_check(h, stream); /* sync + device error word */
  b2g_destroy(h);
  return (int)s;
}
