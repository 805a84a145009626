// b2g_ptx.cuh -- inline-PTX wrappers for the sm_100a features the engine uses:
// mbarriers (bounded waits), TMA tiled loads, cluster addressing, and the
// tcgen05 family (TMEM alloc, MMA issue, commit, TMEM loads).
//
// Every wait in this engine is bounded by wall time (%globaltimer): on expiry the
// waiter records an error word in global memory, raises a CTA-local abort flag
// and returns false, so that no kernel can hang the GPU.  No wrapper traps.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace b2g {

// Error word bits written by kernels (read back by b2g_check).
enum : uint32_t {
  ERRW_TIMEOUT_PRODUCER = 1u << 0,
  ERRW_TIMEOUT_MMA = 1u << 1,
  ERRW_TIMEOUT_EPILOGUE = 1u << 2,
  ERRW_TIMEOUT_OTHER = 1u << 3,
  ERRW_BAD_SPARSITY = 1u << 8,
};

// Upper bound of any single wait.  The longest legitimate wait in this engine is
// one output tile's main loop (tens of microseconds); 2 s is generous.  Kernels
// take a shorter limit at run time (b2g_set_wait_limit); 0 selects this one.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// One lane of a converged warp (elect.sync over the full mask).  The issuing roles
// call it once and keep the answer, so that the same thread issues every MMA and
// the commits that track them.
__device__ __forceinline__ bool elect_one() {
  uint32_t p;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.b32 %0, 1, 0, P;\n\t}"
      : "=r"(p));
  return p != 0u;
}

// Shared::cluster address of the same variable in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(addr), "r"(rank));
  return out;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Arrive on an mbarrier of any CTA in the cluster (addr from mapa_shared).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase of parity `parity` to complete.  Returns false (and
// raises *abort) if the time limit expires, or if *abort was raised by another
// role of this CTA.
__device__ __forceinline__ uint64_t clock64_now() {
  uint64_t c;
  asm volatile("mov.u64 %0, %%clock64;" : "=l"(c));
  return c;
}

// Three independent bounds, whichever trips first: wall time (%globaltimer),
// SM cycles (%clock64, kWaitLimitNs at up to 2.5 GHz) and a poll count.
constexpr uint32_t kWaitMaxPolls = 1u << 26;

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort,
                                          uint32_t* err_word, uint32_t err_bit,
                                          uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  if (limit_ns == 0 || limit_ns > kWaitLimitNs) limit_ns = kWaitLimitNs;
  const uint64_t t0 = globaltimer_ns();
  const uint64_t c0 = clock64_now();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0u) {
      if (*abort) return false;
      if (globaltimer_ns() - t0 > limit_ns || clock64_now() - c0 > limit_ns * 5 / 2 ||
          i >= kWaitMaxPolls) {
        *abort = 1;
        if (err_word) atomicOr(err_word, err_bit);
        return false;
      }
    }
  }
}

// Bounded wait (one thread) for a global word to read `want` (ld.acquire.gpu),
// e.g. the split-tail epilogue's wait for another cluster's partial tile.  Same
// contract as mbar_wait.
__device__ __forceinline__ bool flag_wait(const uint32_t* f, uint32_t want, volatile int* abort,
                                          uint32_t* err_word, uint32_t err_bit,
                                          uint64_t limit_ns = kWaitLimitNs) {
  if (limit_ns == 0 || limit_ns > kWaitLimitNs) limit_ns = kWaitLimitNs;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0;; ++i) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
    if (v == want) return true;
    if ((i & 63u) == 0u) {
      if (*abort) return false;
      if (globaltimer_ns() - t0 > limit_ns || i >= kWaitMaxPolls) {
        *abort = 1;
        if (err_word) atomicOr(err_word, err_bit);
        return false;
      }
    }
    __nanosleep(64);
  }
}

// Progress trace (optional diagnostic): relaxed system-scope stores into a
// host-mapped buffer, readable by the host while a kernel is still running.
// `base` is this CTA's trace row or nullptr (tracing off); the null test is on
// the base pointer, before any offset is applied.
__device__ __forceinline__ void trace_store(uint32_t* base, int slot, uint32_t v) {
  if (base != nullptr)
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(base + slot), "r"(v) : "memory");
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// 1D bulk copy global -> this CTA's shared memory (no tensor map, no multicast):
// both addresses 16-byte aligned, bytes a multiple of 16; completion on `bar`.
__device__ __forceinline__ void bulk_load_1d(uint32_t dst, const void* src, uint32_t bytes,
                                             uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
      : "memory");
}

// 2D tiled load into this CTA's shared memory, completion on a barrier of this CTA.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, int32_t x, int32_t y,
                                            uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(bar), "l"(policy)
      : "memory");
}

// 2D tiled load into this CTA's shared memory whose completion is signalled on
// an mbarrier of either CTA of the pair (cluster address).  Plain, non-
// multicast form: each CTA of the pair fetches its own half of the operands.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const void* tmap, int32_t x,
                                                 int32_t y, uint32_t cluster_bar,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(cluster_bar), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t l2_policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---------------------------------------------------------------- tcgen05
template <int CG>
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::%2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols), "n"(CG)
               : "memory");
}

template <int CG>
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::%0.sync.aligned;" ::"n"(CG) : "memory");
}

template <int CG>
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::%2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols),
               "n"(CG)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Commit all prior tcgen05 async ops of this thread to an mbarrier (one arrive).
// `bar` may be a shared::cta address or a shared::cluster address of the peer CTA.
// The issuing helpers below take `on`: every lane of a converged warp executes
// the instruction's asm and only the lane with `on` != 0 issues it, so the warp
// never diverges around a tcgen05 issue (its operands stay warp-uniform).

template <int CG>
__device__ __forceinline__ void tc_commit(uint32_t bar, uint32_t on = 1u) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "setp.ne.b32 e, %2, 0;\n\t"
      "@e tcgen05.commit.cta_group::%1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(
          bar),
      "n"(CG), "r"(on)
      : "memory");
}

// Commit to the mbarrier at the same shared-memory offset in every CTA of
// `cta_mask` (cta_group::2 pairs: mask 0b11).  This is the tcgen05.commit
// multicast arrive, not a TMA load.
template <int CG>
__device__ __forceinline__ void tc_commit_mc(uint32_t bar, uint16_t cta_mask, uint32_t on = 1u) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "setp.ne.b32 e, %3, 0;\n\t"
      "@e tcgen05.commit.cta_group::%2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;\n\t}" ::"r"(bar),
      "h"(cta_mask), "n"(CG), "r"(on)
      : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]  -- dense kinds (SS operands): 0 tf32, 1 f16,
// 2 f8f6f4, 3 i8 (s32 accumulator).
template <int CG, int KIND>
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate, uint32_t on = 1u) {
  static_assert(KIND >= 0 && KIND <= 3, "mma_ss: dense kinds tf32 / f16 / f8f6f4 / i8 only");
  if constexpr (KIND == 0) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "setp.ne.b32 e, %6, 0;\n\t"
        "@e tcgen05.mma.cta_group::%5.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "n"(CG), "r"(on)
        : "memory");
  } else if constexpr (KIND == 3) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "setp.ne.b32 e, %6, 0;\n\t"
        "@e tcgen05.mma.cta_group::%5.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "n"(CG), "r"(on)
        : "memory");
  } else if constexpr (KIND == 1) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "setp.ne.b32 e, %6, 0;\n\t"
        "@e tcgen05.mma.cta_group::%5.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "n"(CG), "r"(on)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "setp.ne.b32 e, %6, 0;\n\t"
        "@e tcgen05.mma.cta_group::%5.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "n"(CG), "r"(on)
        : "memory");
  }
}

// D[tmem] (+)= A[tmem] * B[smem] -- dense kinds, TS operands.
template <int CG, int KIND>
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate, uint32_t on = 1u) {
  static_assert(KIND == 1 || KIND == 2, "mma_ts: dense kinds f16 / f8f6f4 only");
  if constexpr (KIND == 1) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "setp.ne.b32 e, %6, 0;\n\t"
        "@e tcgen05.mma.cta_group::%5.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "n"(CG), "r"(on)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "setp.ne.b32 e, %6, 0;\n\t"
        "@e tcgen05.mma.cta_group::%5.kind::f8f6f4 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "n"(CG), "r"(on)
        : "memory");
  }
}

// SMEM -> TMEM copy of a 128-row x 32-byte matrix (8 TMEM columns) described by an
// SMEM matrix descriptor (any swizzle mode the descriptor names).
template <int CG>
__device__ __forceinline__ void tc_cp_128x256b(uint32_t taddr, uint64_t sdesc, uint32_t on = 1u) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "setp.ne.b32 e, %3, 0;\n\t"
      "@e tcgen05.cp.cta_group::%2.128x256b [%0], %1;\n\t}" ::"r"(taddr),
      "l"(sdesc), "n"(CG), "r"(on)
      : "memory");
}

// D[tmem] (+)= A[smem] * B[smem] with A structured-sparse (compressed in SMEM,
// metadata in TMEM at `meta_tmem`): kind::tf32 (1:2, dense K 16 per MMA), kind::f16
// (2:4, dense K 32), kind::f8f6f4 and kind::i8 (2:4, dense K 64).
template <int CG, int KIND>
__device__ __forceinline__ void mma_sp(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t meta_tmem, uint32_t idesc, uint32_t accumulate,
                                       uint32_t on = 1u) {
  static_assert(KIND >= 0 && KIND <= 3, "mma_sp: kinds tf32 / f16 / f8f6f4 / i8");
  if constexpr (KIND == 0) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "setp.ne.b32 e, %7, 0;\n\t"
        "@e tcgen05.mma.sp.cta_group::%6.kind::tf32 [%0], %1, %2, [%3], %4, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(meta_tmem), "r"(idesc), "r"(accumulate), "n"(CG), "r"(on)
        : "memory");
  } else if constexpr (KIND == 1) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "setp.ne.b32 e, %7, 0;\n\t"
        "@e tcgen05.mma.sp.cta_group::%6.kind::f16 [%0], %1, %2, [%3], %4, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(meta_tmem), "r"(idesc), "r"(accumulate), "n"(CG), "r"(on)
        : "memory");
  } else if constexpr (KIND == 2) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "setp.ne.b32 e, %7, 0;\n\t"
        "@e tcgen05.mma.sp.cta_group::%6.kind::f8f6f4 [%0], %1, %2, [%3], %4, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(meta_tmem), "r"(idesc), "r"(accumulate), "n"(CG), "r"(on)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "setp.ne.b32 e, %7, 0;\n\t"
        "@e tcgen05.mma.sp.cta_group::%6.kind::i8 [%0], %1, %2, [%3], %4, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(meta_tmem), "r"(idesc), "r"(accumulate), "n"(CG), "r"(on)
        : "memory");
  }
}

// SMEM -> TMEM copy of a 128-lane x 16-byte block (4 TMEM columns), described by
// a no-swizzle SMEM matrix descriptor.  Asynchronous; ordered with the issuing
// thread's later tcgen05.mma.  With cta_group::2 each CTA of the pair copies
// from its own SMEM into its own TMEM.
template <int CG>
__device__ __forceinline__ void tc_cp_128x128b(uint32_t taddr, uint64_t sdesc, uint32_t on = 1u) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "setp.ne.b32 e, %3, 0;\n\t"
      "@e tcgen05.cp.cta_group::%2.128x128b [%0], %1;\n\t}" ::"r"(taddr),
      "l"(sdesc), "n"(CG), "r"(on)
      : "memory");
}

// Weight-stationary MMA (tcgen05.mma.ws, cta_group::1 only; M 32 / 64 / 128, N 64 /
// 128 / 256), dense or structured-sparse A, kinds tf32 / f16 / f8f6f4 / i8 (the
// form takes no block scaling).  The same operands as mma_ss / mma_sp; no B
// collector buffer is named, so B is read from shared memory by every MMA.
#define B2G_WS_ASM(OP, KINDNAME, META)                                                      \
  "{\n\t.reg .pred p, e;\n\tsetp.ne.b32 p, %4, 0;\n\tsetp.ne.b32 e, %5, 0;\n\t@e " OP        \
  ".cta_group::1.kind::" KINDNAME " [%0], %1, %2, " META "%3, p;\n\t}"
#define B2G_WS_KINDS(OP, META, ...)                                                        \
  if constexpr (KIND == 0) asm volatile(B2G_WS_ASM(OP, "tf32", META) __VA_ARGS__);            \
  else if constexpr (KIND == 1) asm volatile(B2G_WS_ASM(OP, "f16", META) __VA_ARGS__);        \
  else if constexpr (KIND == 2) asm volatile(B2G_WS_ASM(OP, "f8f6f4", META) __VA_ARGS__);     \
  else asm volatile(B2G_WS_ASM(OP, "i8", META) __VA_ARGS__)
template <int KIND>
__device__ __forceinline__ void mma_ws_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate, uint32_t on = 1u) {
  static_assert(KIND >= 0 && KIND <= 3, "mma_ws_ss: kinds tf32 / f16 / f8f6f4 / i8");
  B2G_WS_KINDS("tcgen05.mma.ws", "",
               ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(on)
               : "memory");
}
template <int KIND>
__device__ __forceinline__ void mma_ws_sp(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t meta_tmem, uint32_t idesc, uint32_t accumulate,
                                          uint32_t on = 1u) {
  static_assert(KIND >= 0 && KIND <= 3, "mma_ws_sp: kinds tf32 / f16 / f8f6f4 / i8");
  B2G_WS_KINDS("tcgen05.mma.ws.sp", "[%6], ",
               ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(on),
               "r"(meta_tmem)
               : "memory");
}
#undef B2G_WS_KINDS
#undef B2G_WS_ASM

// Block-scaled MMA by kind: NVFP4 (kind 6: mxf4nvf4, block16, ue4m3), MXFP8
// (kind 4: mxf8f6f4, one E8M0 per 32), MXFP4 (kind 5: mxf4, block32, E8M0).  Scale
// factors in TMEM at sfa_tmem / sfb_tmem (4x1 data-path layout, replicated over
// the lane quarters); the addresses may carry the byte select in bits 30-31
// (matching the descriptor's SF ids).
template <int CG, int KIND>
__device__ __forceinline__ void mma_bs(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t sfa_tmem, uint32_t sfb_tmem,
                                       uint32_t accumulate, uint32_t on = 1u) {
  static_assert(KIND == 4 || KIND == 5 || KIND == 6,
                "mma_bs: block-scaled kinds 4 (mxf8f6f4), 5 (mxf4), 6 (mxf4nvf4)");
  if constexpr (KIND == 6) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "setp.ne.b32 e, %8, 0;\n\t"
        "@e tcgen05.mma.cta_group::%7.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], "
        "[%6], p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem), "n"(CG),
        "r"(on)
        : "memory");
  } else if constexpr (KIND == 4) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "setp.ne.b32 e, %8, 0;\n\t"
        "@e tcgen05.mma.cta_group::%7.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;"
        "\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem), "n"(CG),
        "r"(on)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "setp.ne.b32 e, %8, 0;\n\t"
        "@e tcgen05.mma.cta_group::%7.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;"
        "\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem), "n"(CG),
        "r"(on)
        : "memory");
  }
}

// Structured-sparse A on a block-scaled kind (tcgen05.mma.sp ... block_scale):
// kind::mxf8f6f4 (2:4 on 8-bit elements), kind::mxf4 block32 or kind::mxf4nvf4
// block16 (4:8 in pairs of packed e2m1); metadata columns at meta_tmem as for mma_sp with an 8-bit kind, scale
// factors as for mma_bs (E8M0, the addresses' bits 30-31 carrying the byte select).
#define B2G_SP_BS_ASM(KINDNAME)                                                             \
  "{\n\t.reg .pred p, e;\n\tsetp.ne.b32 p, %5, 0;\n\tsetp.ne.b32 e, %9, 0;\n\t"             \
  "@e tcgen05.mma.sp.cta_group::%8.kind::" KINDNAME " [%0], %1, %2, [%3], %4, [%6], [%7], p;\n\t}"
template <int CG, int KIND>
__device__ __forceinline__ void mma_sp_bs(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t meta_tmem, uint32_t idesc, uint32_t sfa_tmem,
                                          uint32_t sfb_tmem, uint32_t accumulate, uint32_t on = 1u) {
  static_assert(KIND >= 4 && KIND <= 6, "mma_sp_bs: kinds 4 (mxf8f6f4), 5 (mxf4), 6 (mxf4nvf4)");
  if constexpr (KIND == 6)
    asm volatile(B2G_SP_BS_ASM("mxf4nvf4.block_scale.block16")::"r"(d_tmem), "l"(a_desc),
                 "l"(b_desc), "r"(meta_tmem), "r"(idesc), "r"(accumulate), "r"(sfa_tmem),
                 "r"(sfb_tmem), "n"(CG), "r"(on)
                 : "memory");
  else if constexpr (KIND == 4)
    asm volatile(B2G_SP_BS_ASM("mxf8f6f4.block_scale")::"r"(d_tmem), "l"(a_desc), "l"(b_desc),
                 "r"(meta_tmem), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem),
                 "n"(CG), "r"(on)
                 : "memory");
  else
    asm volatile(B2G_SP_BS_ASM("mxf4.block_scale.block32")::"r"(d_tmem), "l"(a_desc),
                 "l"(b_desc), "r"(meta_tmem), "r"(idesc), "r"(accumulate), "r"(sfa_tmem),
                 "r"(sfb_tmem), "n"(CG), "r"(on)
                 : "memory");
}
#undef B2G_SP_BS_ASM

// SMEM -> TMEM copy of a 32-row x 16-byte block, replicated into all four TMEM
// lane quarters (4 columns): the scale-factor layout of block-scaled MMAs.
template <int CG>
__device__ __forceinline__ void tc_cp_32x128b_warpx4(uint32_t taddr, uint64_t sdesc,
                                                     uint32_t on = 1u) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "setp.ne.b32 e, %3, 0;\n\t"
      "@e tcgen05.cp.cta_group::%2.32x128b.warpx4 [%0], %1;\n\t}" ::"r"(taddr),
      "l"(sdesc), "n"(CG), "r"(on)
      : "memory");
}

// 32 lanes x 32 consecutive fp32 columns: thread i of the warp gets lane
// (warp's lane quarter * 32 + i), columns [col, col+32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

}  // namespace b2g
