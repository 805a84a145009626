// probe.cu -- tcgen05.mma instruction-rate / latency probe (b2g_probe_mma).
//
// The measurement the reference's umma_throughput/umma_tput.cu:491-522 and
// tcgen05_sparse_mma/tcgen05_sparse_mma.cu:485-597 make, from this engine's own
// PTX wrappers: one CTA (or one cta_group::2 pair) keeps A and B resident in
// SMEM (K-major), re-issues `depth`
// MMAs of the requested form per batch, commits the batch to an mbarrier and
// waits.  Throughput mode returns clock64 cycles over `iters` batches; latency
// mode returns the median of 100 single-MMA round trips.  Operands use the
// reference's no-swizzle core-matrix layout, so the rates compare one to one
// with its published tables; the GEMM itself stages 128-byte swizzled tiles.
//
// Forms: kinds tf32, f16, f8f6f4, i8, mxf8f6f4, mxf4 (block32), mxf4nvf4
// (block32 for ue8m0 scales, block16 for ue4m3), dense or 2:4 sparse (.sp),
// .ws (cta_group::1), SS or TS operands, cta_group 1 or 2.  Operand contents are
// fixed byte patterns (values do not change the issue rate).  The host rejects
// shapes outside the tcgen05 shape tables before any launch; every wait is
// bounded.
#include <cuda_runtime.h>
#include <stdint.h>

#include "b2g_desc.h"
#include "b2g_gemm.h"
#include "b2g_ptx.cuh"

namespace b2g {

// Form kind ids: the reference's KIND_ID 0..6, plus 7 = mxf4nvf4 with block16.
enum ProbeKind : int {
  PK_TF32 = 0, PK_F16 = 1, PK_F8F6F4 = 2, PK_I8 = 3, PK_MXF8F6F4 = 4, PK_MXF4 = 5,
  PK_MXF4NVF4_B32 = 6, PK_MXF4NVF4_B16 = 7
};

constexpr int kProbeThreads = 128;

// The instruction: literal strings per form.  Operands: %0 D, %1 A (desc or
// TMEM), %2 B desc, %3 idesc, %4 accumulate, %5 metadata, %6 SFA, %7 SFB, %8 issue
// predicate (the whole issuing warp executes the asm; one elected lane issues).
#define B2G_PROBE_BODY(HEAD, KIND, AOP, META, SF)                                              \
  "{\n\t.reg .pred p, e;\n\tsetp.ne.b32 p, %4, 0;\n\tsetp.ne.b32 e, %8, 0;\n\t@e " HEAD ".kind::" \
  KIND " [%0], " AOP ", %2, " META "%3" SF ", p;\n\t}"

#define B2G_PROBE_KINDS(HEAD, AOP, META)                                                  \
  if constexpr (KID == PK_TF32) asm volatile(B2G_PROBE_BODY(HEAD, "tf32", AOP, META, "") B2G_PROBE_OPS); \
  else if constexpr (KID == PK_F16) asm volatile(B2G_PROBE_BODY(HEAD, "f16", AOP, META, "") B2G_PROBE_OPS); \
  else if constexpr (KID == PK_F8F6F4) asm volatile(B2G_PROBE_BODY(HEAD, "f8f6f4", AOP, META, "") B2G_PROBE_OPS); \
  else if constexpr (KID == PK_I8) asm volatile(B2G_PROBE_BODY(HEAD, "i8", AOP, META, "") B2G_PROBE_OPS); \
  else if constexpr (KID == PK_MXF8F6F4) asm volatile(B2G_PROBE_BODY(HEAD, "mxf8f6f4.block_scale", AOP, META, ", [%6], [%7]") B2G_PROBE_OPS); \
  else if constexpr (KID == PK_MXF4) asm volatile(B2G_PROBE_BODY(HEAD, "mxf4.block_scale.block32", AOP, META, ", [%6], [%7]") B2G_PROBE_OPS); \
  else if constexpr (KID == PK_MXF4NVF4_B32) asm volatile(B2G_PROBE_BODY(HEAD, "mxf4nvf4.block_scale.block32", AOP, META, ", [%6], [%7]") B2G_PROBE_OPS); \
  else asm volatile(B2G_PROBE_BODY(HEAD, "mxf4nvf4.block_scale.block16", AOP, META, ", [%6], [%7]") B2G_PROBE_OPS)

template <int KID, int SP, int WS, int CG>
__device__ __forceinline__ void probe_mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                             uint32_t acc, uint32_t meta, uint32_t sfa,
                                             uint32_t sfb, uint32_t on) {
#define B2G_PROBE_OPS \
  ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(meta), "r"(sfa), "r"(sfb), "r"(on) : "memory"
  if constexpr (WS && SP) { B2G_PROBE_KINDS("tcgen05.mma.ws.sp.cta_group::1", "%1", "[%5], "); }
  else if constexpr (WS) { B2G_PROBE_KINDS("tcgen05.mma.ws.cta_group::1", "%1", ""); }
  else if constexpr (SP && CG == 2) { B2G_PROBE_KINDS("tcgen05.mma.sp.cta_group::2", "%1", "[%5], "); }
  else if constexpr (SP) { B2G_PROBE_KINDS("tcgen05.mma.sp.cta_group::1", "%1", "[%5], "); }
  else if constexpr (CG == 2) { B2G_PROBE_KINDS("tcgen05.mma.cta_group::2", "%1", ""); }
  else { B2G_PROBE_KINDS("tcgen05.mma.cta_group::1", "%1", ""); }
#undef B2G_PROBE_OPS
}

template <int KID, int SP, int WS, int CG>
__device__ __forceinline__ void probe_mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc,
                                             uint32_t acc, uint32_t meta, uint32_t sfa,
                                             uint32_t sfb, uint32_t on) {
#define B2G_PROBE_OPS \
  ::"r"(d), "r"(a), "l"(b), "r"(idesc), "r"(acc), "r"(meta), "r"(sfa), "r"(sfb), "r"(on) : "memory"
  if constexpr (WS && SP) { B2G_PROBE_KINDS("tcgen05.mma.ws.sp.cta_group::1", "[%1]", "[%5], "); }
  else if constexpr (WS) { B2G_PROBE_KINDS("tcgen05.mma.ws.cta_group::1", "[%1]", ""); }
  else if constexpr (SP && CG == 2) { B2G_PROBE_KINDS("tcgen05.mma.sp.cta_group::2", "[%1]", "[%5], "); }
  else if constexpr (SP) { B2G_PROBE_KINDS("tcgen05.mma.sp.cta_group::1", "[%1]", "[%5], "); }
  else if constexpr (CG == 2) { B2G_PROBE_KINDS("tcgen05.mma.cta_group::2", "[%1]", ""); }
  else { B2G_PROBE_KINDS("tcgen05.mma.cta_group::1", "[%1]", ""); }
#undef B2G_PROBE_OPS
}

#undef B2G_PROBE_KINDS
#undef B2G_PROBE_BODY

__device__ __forceinline__ void tmem_st_32x32b_x1(uint32_t taddr, uint32_t v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(v) : "memory");
}

template <int KID, int SP, int WS, int CG, int TS>
__global__ void __launch_bounds__(kProbeThreads, 1) probe_kernel(const ProbeArgs p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5;
  const uint32_t rank = (CG == 2) ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;

  // resident operands: deterministic non-zero byte patterns, 128-byte rows
  const int a_bytes = p.a_rows * 128, b_bytes = p.b_rows * 128;
  for (int i = threadIdx.x; i < a_bytes + b_bytes; i += kProbeThreads)
    smem[i] = (uint8_t)((i * 13 + 17 * (int)rank + 1) & 0x3F) | 0x01;
  const uint32_t sA = smem_u32(smem), sB = sA + (uint32_t)a_bytes;
  const uint32_t bar_a = smem_u32(&bar);
  if (threadIdx.x == 0) {
    mbar_init(bar_a, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc<CG>(smem_u32(&tmem_slot), p.tmem_cols);
    tmem_relinquish<CG>();
  }
  tc_fence_before();
  __syncthreads();
  if (CG == 2) cluster_sync();
  tc_fence_after();
  const uint32_t tbase = tmem_slot;
  // TMEM side operands, one column at a time for all 128 lanes (each warp its
  // lane quarter): TS A, scale factors, sparse metadata
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  if (TS)
    for (uint32_t c = 0; c < 16; ++c) tmem_st_32x32b_x1(tbase + lane_off + p.a_col + c, 0x3C003C00u);
  for (uint32_t c = 0; c < 16; ++c) tmem_st_32x32b_x1(tbase + lane_off + p.sf_col + c, p.sf_word);
  for (uint32_t c = 0; c < 4; ++c) tmem_st_32x32b_x1(tbase + lane_off + p.meta_col + c, 0x44444444u);
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  if (CG == 2) cluster_sync();
  tc_fence_after();

  // no-swizzle K-major operands as the reference probes them
  // (umma_tput.cu:147-156): 8-row x 16-byte core matrices, SBO = 128 bytes
  // between row groups, LBO = rows x 16 bytes between K groups
  const uint64_t adesc = encode_smem_desc(sA, (uint32_t)p.a_rows * 16u, 128, SWZ_NONE);
  const uint64_t bdesc = encode_smem_desc(sB, (uint32_t)p.b_rows * 16u, 128, SWZ_NONE);
  const uint32_t d = tbase + p.d_col, a_t = tbase + p.a_col;
  const uint32_t meta = tbase + p.meta_col, sfa = tbase + p.sf_col, sfb = sfa + 4;
  // Warp 0 of the leader CTA issues as a whole, converged warp: every lane executes
  // each tcgen05 asm, predicated on one lane elected once, as the GEMM's MMA warp
  // does.  (One diverged lane issuing alone takes tens of cycles per tcgen05.mma,
  // more than a cta_group::2 M = 128, N = 128 MMA takes to execute.)
  const bool elected = elect_one();  // every warp, converged
  const bool issue_warp = leader && warp == 0;
  const uint32_t on = (issue_warp && elected) ? 1u : 0u;
  auto mma = [&](uint32_t acc) {
    if constexpr (TS) probe_mma_ts<KID, SP, WS, CG>(d, a_t, bdesc, p.idesc, acc, meta, sfa, sfb, on);
    else probe_mma_ss<KID, SP, WS, CG>(d, adesc, bdesc, p.idesc, acc, meta, sfa, sfb, on);
  };
  auto commit = [&]() {
    if (CG == 2) tc_commit_mc<CG>(bar_a, 0x3, on);
    else tc_commit<CG>(bar_a, on);
  };
  volatile int* ab = &abort_flag;
  uint32_t phase = 0;
  unsigned long long t0 = 0, t1 = 0, med = 0;
  if (p.mode == 0) {
    t0 = clock64_now();
    for (int it = 0; it < p.iters; ++it) {
      if (issue_warp) {
        mma(0u);
#pragma unroll 8
        for (int m = 1; m < p.depth; ++m) mma(1u);
        commit();
      }
      if (!mbar_wait(bar_a, phase, ab, p.err, ERRW_TIMEOUT_OTHER)) break;
      phase ^= 1u;
    }
    t1 = clock64_now();
  } else {
    constexpr int kSamples = 100;
    unsigned long long s[kSamples];
    int n = 0;
    for (; n < kSamples; ++n) {
      const unsigned long long a = clock64_now();
      if (issue_warp) {
        mma(1u);
        commit();
      }
      if (!mbar_wait(bar_a, phase, ab, p.err, ERRW_TIMEOUT_OTHER)) break;
      phase ^= 1u;
      s[n] = clock64_now() - a;
    }
    if (threadIdx.x == 0 && n > 0) {
      for (int i = 1; i < n; ++i) {  // insertion sort of the samples
        const unsigned long long v = s[i];
        int j = i - 1;
        while (j >= 0 && s[j] > v) {
          s[j + 1] = s[j];
          --j;
        }
        s[j + 1] = v;
      }
      med = (n % 2) ? s[n / 2] : (s[n / 2 - 1] + s[n / 2]) / 2;
    }
  }
  if (leader && threadIdx.x == 0) {  // (the thread that took the median)
    p.result[0] = t1 - t0;
    p.result[1] = (unsigned long long)p.depth * (unsigned long long)p.iters;
    p.result[2] = med;
  }
  tc_fence_before();
  __syncthreads();
  if (CG == 2) cluster_sync();
  tc_fence_after();
  if (warp == 0) tmem_dealloc<CG>(tbase, p.tmem_cols);
}

// ------------------------------------------------------------------ dispatch
template <int KID, int SP, int WS, int CG, int TS>
static cudaError_t probe_launch_one(const ProbeArgs& p, size_t smem, cudaStream_t s) {
  auto* fn = probe_kernel<KID, SP, WS, CG, TS>;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(CG, 1, 1);
  cfg.blockDim = dim3(kProbeThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CG;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fn, p);
}

template <int KID, int SP, int WS, int CG>
static cudaError_t probe_ts(int ts, const ProbeArgs& p, size_t smem, cudaStream_t s) {
  return ts ? probe_launch_one<KID, SP, WS, CG, 1>(p, smem, s)
            : probe_launch_one<KID, SP, WS, CG, 0>(p, smem, s);
}

template <int KID, int SP>
static cudaError_t probe_shape(int ws, int cg, int ts, const ProbeArgs& p, size_t smem,
                               cudaStream_t s) {
  if constexpr (KID < PK_MXF8F6F4) {  // .ws exists for the dense kinds only
    if (ws) return probe_ts<KID, SP, 1, 1>(ts, p, smem, s);
  } else if (ws) {
    return cudaErrorInvalidValue;
  }
  return cg == 2 ? probe_ts<KID, SP, 0, 2>(ts, p, smem, s) : probe_ts<KID, SP, 0, 1>(ts, p, smem, s);
}

template <int KID>
static cudaError_t probe_sp(int sp, int ws, int cg, int ts, const ProbeArgs& p, size_t smem,
                            cudaStream_t s) {
  return sp ? probe_shape<KID, 1>(ws, cg, ts, p, smem, s) : probe_shape<KID, 0>(ws, cg, ts, p, smem, s);
}

cudaError_t probe_launch(int kid, int sp, int ws, int cg, int ts, const ProbeArgs& p, size_t smem,
                         cudaStream_t s) {
  switch (kid) {
    case PK_TF32: return probe_sp<PK_TF32>(sp, ws, cg, ts, p, smem, s);
    case PK_F16: return probe_sp<PK_F16>(sp, ws, cg, ts, p, smem, s);
    case PK_F8F6F4: return probe_sp<PK_F8F6F4>(sp, ws, cg, ts, p, smem, s);
    case PK_I8: return probe_sp<PK_I8>(sp, ws, cg, ts, p, smem, s);
    case PK_MXF8F6F4: return probe_sp<PK_MXF8F6F4>(sp, 0, cg, ts, p, smem, s);
    case PK_MXF4: return probe_sp<PK_MXF4>(sp, 0, cg, ts, p, smem, s);
    case PK_MXF4NVF4_B32: return probe_sp<PK_MXF4NVF4_B32>(sp, 0, cg, ts, p, smem, s);
    case PK_MXF4NVF4_B16: return probe_sp<PK_MXF4NVF4_B16>(sp, 0, cg, ts, p, smem, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace b2g
