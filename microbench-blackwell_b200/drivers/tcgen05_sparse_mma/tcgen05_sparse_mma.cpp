// Drop-in main for tcgen05_sparse_mma/ (reference:
// tcgen05_sparse_mma/tcgen05_sparse_mma.cu:600-619 and its RESULT lines
// :531-537, :592-595).
//
// Same macros, same stdout lines:
//   RESULT,throughput,inst,kind,acode,bcode,sparsity,layout,cg,M,N,K,depth,
//          cycles,total_mmas,cycles_per_mma(%.6f),A_bytes,B_bytes
//   RESULT,latency,inst,kind,acode,bcode,sparsity,layout,cg,M,N,K,median,A_bytes,B_bytes
// A_bytes / B_bytes are the operand sizes of one MMA as the reference defines
// them (tcgen05_sparse_mma.cu:131-137): A holds M/cta_group rows of K/2 (sparse)
// or K stored elements.  Exit 0 on success; "CUDA Error: <message>" and 1 on error.
#include <cstdio>

#include "b2g.h"

#if !defined(BENCH_MODE) || !defined(INSTRUCTION_ID) || !defined(KIND_ID) ||          \
    !defined(A_TYPE_CODE) || !defined(B_TYPE_CODE) || !defined(A_BITS) || !defined(B_BITS) || \
    !defined(SPARSITY) || !defined(AB_LAYOUT_ID) || !defined(CTA_GROUP) || !defined(MMA_M) || \
    !defined(MMA_N) || !defined(MMA_K) || !defined(MMA_DEPTH) || !defined(SCALE_TYPE_ID)
#error "all configuration macros must be defined (see the Makefile)"
#endif
#if INSTRUCTION_ID == 1 && CTA_GROUP != 1
#error "tcgen05.mma.ws(.sp) supports CTA_GROUP=1 only"
#endif
#if INSTRUCTION_ID == 1 && KIND_ID >= 4
#error "tcgen05.mma.ws(.sp) is restricted to non-block-scaled kinds"
#endif
#if CTA_GROUP != 1 && CTA_GROUP != 2
#error "CTA_GROUP must be 1 or 2"
#endif

static constexpr int cdiv(int a, int b) { return (a + b - 1) / b; }
static constexpr int kStoredK = SPARSITY ? MMA_K / 2 : MMA_K;
static constexpr int kABytes = cdiv(MMA_M / CTA_GROUP * kStoredK * A_BITS, 8);
static constexpr int kBBytes = cdiv(MMA_K * MMA_N * B_BITS, 8);

int main() {
  b2g_handle* h = nullptr;
  b2g_status st = b2g_create(0, &h);
  if (st != B2G_OK) {
    printf("CUDA Error: %s\n", b2g_status_string(st));
    return 1;
  }
  b2g_probe_desc p = {};
  p.kind = KIND_ID;
  p.a_type = A_TYPE_CODE;
  p.b_type = B_TYPE_CODE;
  p.a_bits = A_BITS;
  p.b_bits = B_BITS;
  p.sparse = SPARSITY;
  p.ab_mode = AB_LAYOUT_ID;
  p.cta_group = CTA_GROUP;
  p.m = MMA_M;
  p.n = MMA_N;
  p.k = MMA_K;
  p.depth = MMA_DEPTH;
  p.scale_type = SCALE_TYPE_ID;
  p.mode = BENCH_MODE;
  p.iters = 1000;
  p.instruction = INSTRUCTION_ID;
  uint64_t cycles = 0, total = 0, median = 0;
  st = b2g_probe_mma(h, &p, &cycles, &total, &median);
  if (st != B2G_OK) {
    printf("CUDA Error: %s\n", b2g_last_error(h));
    b2g_destroy(h);
    return 1;
  }
  if (BENCH_MODE == 0)
    printf("RESULT,throughput,%d,%d,%d,%d,%d,%d,%d,%d,%d,%d,%d,%llu,%llu,%.6f,%d,%d\n",
           INSTRUCTION_ID, KIND_ID, A_TYPE_CODE, B_TYPE_CODE, SPARSITY, AB_LAYOUT_ID, CTA_GROUP,
           MMA_M, MMA_N, MMA_K, MMA_DEPTH, (unsigned long long)cycles, (unsigned long long)total,
           total ? (double)cycles / (double)total : 0.0, kABytes, kBBytes);
  else
    printf("RESULT,latency,%d,%d,%d,%d,%d,%d,%d,%d,%d,%d,%llu,%d,%d\n", INSTRUCTION_ID, KIND_ID,
           A_TYPE_CODE, B_TYPE_CODE, SPARSITY, AB_LAYOUT_ID, CTA_GROUP, MMA_M, MMA_N, MMA_K,
           (unsigned long long)median, kABytes, kBBytes);
  b2g_destroy(h);
  return 0;
}
