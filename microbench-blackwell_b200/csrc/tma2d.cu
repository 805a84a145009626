// tma2d.cu -- TMA HBM -> SMEM streaming: 2D tiles (b2g_stream_tma2d) and 1D bulk
// copies (b2g_stream_bulk1d).
//
// The standalone form of the GEMM's operand stager, for the measurement of
// tma2d_throughput/tma2d_tput.cu:50-134: each CTA is one warp whose elected lane
// walks the rows of an fp32 matrix (width x height) in box_w x box_h boxes, one
// box every gridDim.x boxes, keeping `stages` loads in flight in an mbarrier
// ring (wait for a slot's previous load, re-arm it with expect_tx, re-issue).
// The data are only landed in SMEM, as in the reference; DRAM read bandwidth
// is read from ncu counters or from the event time the host returns.
// Every wait is bounded.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "b2g_gemm.h"
#include "b2g_ptx.cuh"

namespace b2g {

// Waits for the loads still in flight in a ring whose next slot is `slot`: all
// `stages` slots when the ring has wrapped, else slots [0, slot).  Oldest first.
__device__ __forceinline__ void drain_ring(const uint64_t* bars, int slot, bool wrapped,
                                           int stages, uint32_t phase_bits, volatile int* abort,
                                           uint32_t* err) {
  const int inflight = wrapped ? stages : slot;
  int s = wrapped ? slot : 0;
  for (int i = 0; i < inflight; ++i) {
    if (!mbar_wait(smem_u32(&bars[s]), (phase_bits >> s) & 1u, abort, err, ERRW_TIMEOUT_OTHER))
      return;
    phase_bits ^= 1u << s;
    if (++s == stages) s = 0;
  }
}

__global__ void __launch_bounds__(32, 1)
    tma2d_stream_kernel(const __grid_constant__ CUtensorMap tm, uint64_t height, int box_h,
                        uint32_t box_bytes, int stages, uint32_t* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  __shared__ uint64_t bars[16];
  __shared__ int abort_flag;
  if (threadIdx.x != 0) return;  // one issuing thread; the rest of the warp has no role
  const uint32_t base = smem_u32(smem);
  for (int s = 0; s < stages; ++s) mbar_init(smem_u32(&bars[s]), 1);
  abort_flag = 0;
  fence_mbar_init();
  const uint64_t policy = l2_policy_evict_normal();
  const int64_t stride = (int64_t)gridDim.x * box_h;
  uint32_t phase_bits = 0;  // bit s: parity of slot s's next completion
  int64_t row = (int64_t)blockIdx.x * box_h;
  // the ring position is a wrapping counter: no 64-bit division in the issue loop
  int slot = 0;
  bool wrapped = false;  // every slot has a load in flight
  for (; row < (int64_t)height; row += stride) {
    const uint32_t bar = smem_u32(&bars[slot]);
    if (wrapped) {  // the slot's previous load must have landed
      if (!mbar_wait(bar, (phase_bits >> slot) & 1u, &abort_flag, err, ERRW_TIMEOUT_OTHER)) return;
      phase_bits ^= 1u << slot;
    }
    mbar_arrive_expect_tx(bar, box_bytes);
    tma_load_2d(base + (uint32_t)slot * box_bytes, &tm, 0, (int32_t)row, bar, policy);
    if (++slot == stages) {
      slot = 0;
      wrapped = true;
    }
  }
  drain_ring(bars, slot, wrapped, stages, phase_bits, &abort_flag, err);
}

// Kernel set-up kept out of any timed interval: the shared-memory attribute, and
// the attribute query that makes a lazily loaded module load now rather than at
// the first launch.
static cudaError_t stream_prepare(const void* fn, int smem_bytes) {
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
  if (e != cudaSuccess) return e;
  cudaFuncAttributes fa;
  return cudaFuncGetAttributes(&fa, fn);
}

cudaError_t tma2d_stream_prepare(int smem_bytes) {
  return stream_prepare(reinterpret_cast<const void*>(tma2d_stream_kernel), smem_bytes);
}

// (tma2d_stream_prepare must have run for this smem_bytes)
cudaError_t tma2d_stream_launch(const CUtensorMap& tm, uint64_t height, int box_w, int box_h,
                                int stages, int grid, int smem_bytes, uint32_t* err,
                                cudaStream_t s) {
  const uint32_t box_bytes = (uint32_t)box_w * (uint32_t)box_h * 4u;
  tma2d_stream_kernel<<<grid, 32, smem_bytes, s>>>(tm, height, box_h, box_bytes, stages, err);
  return cudaGetLastError();
}

// TMA 2D load latency (b2g_tma2d_latency), the measurement of
// tma2d_latency/tma2d_lat.cu:43-100: each CTA's elected thread issues one box load
// of rows [row0 + blockIdx.x * box_h, + box_h) and records the clock64 cycles from
// before its expect_tx to the barrier's completion: one sample per CTA and launch,
// nothing else in flight.  The wait is bounded; an expired wait records 0xFFFFFFFF.
__global__ void __launch_bounds__(32, 1)
    tma2d_latency_kernel(const __grid_constant__ CUtensorMap tm, int64_t row0, int box_h,
                         uint32_t box_bytes, uint32_t* cycles, uint32_t* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x != 0) return;  // one issuing and timing thread
  const uint32_t b = smem_u32(&bar);
  mbar_init(b, 1);
  abort_flag = 0;
  fence_mbar_init();
  const uint64_t policy = l2_policy_evict_normal();
  const int32_t row = (int32_t)(row0 + (int64_t)blockIdx.x * box_h);
  const uint64_t t0 = clock64_now();
  mbar_arrive_expect_tx(b, box_bytes);
  tma_load_2d(smem_u32(smem), &tm, 0, row, b, policy);
  const bool ok = mbar_wait(b, 0, &abort_flag, err, ERRW_TIMEOUT_OTHER);
  const uint64_t t1 = clock64_now();
  cycles[blockIdx.x] = ok ? (uint32_t)(t1 - t0) : 0xFFFFFFFFu;
}

cudaError_t tma2d_latency_smem(int device, int* smem_bytes) {
  // everything a block may opt into, less the kernel's static shared memory
  int optin = 0;
  cudaError_t e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
  if (e != cudaSuccess) return e;
  cudaFuncAttributes fa;
  e = cudaFuncGetAttributes(&fa, tma2d_latency_kernel);
  if (e != cudaSuccess) return e;
  *smem_bytes = optin - (int)fa.sharedSizeBytes;
  return cudaSuccess;
}

cudaError_t tma2d_latency_launch(const CUtensorMap& tm, int64_t row0, int box_w, int box_h,
                                 int grid, int smem_bytes, uint32_t* cycles, uint32_t* err,
                                 cudaStream_t s) {
  cudaError_t e = cudaFuncSetAttribute(tma2d_latency_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
  if (e != cudaSuccess) return e;
  const uint32_t box_bytes = (uint32_t)box_w * (uint32_t)box_h * 4u;
  tma2d_latency_kernel<<<grid, 32, smem_bytes, s>>>(tm, row0, box_h, box_bytes, cycles, err);
  return cudaGetLastError();
}

// 1D bulk streaming (b2g_stream_bulk1d), the measurement of
// tma_throughput/tma_tput.cu:41-76: each CTA's elected thread copies chunks
// blockIdx.x, blockIdx.x + gridDim.x, ... of `load_bytes` each with
// cp.async.bulk into a `stages`-slot mbarrier ring, waiting for a slot's previous
// copy before reusing it.  Every wait is bounded.
__global__ void __launch_bounds__(32, 1)
    bulk1d_stream_kernel(const uint8_t* data, uint64_t chunks, uint32_t load_bytes, int stages,
                         uint32_t* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint64_t bars[16];
  __shared__ int abort_flag;
  if (threadIdx.x != 0) return;
  const uint32_t base = smem_u32(smem_raw);
  for (int s = 0; s < stages; ++s) mbar_init(smem_u32(&bars[s]), 1);
  abort_flag = 0;
  fence_mbar_init();
  uint32_t phase_bits = 0;
  int slot = 0;
  bool wrapped = false;
  for (uint64_t c = blockIdx.x; c < chunks; c += gridDim.x) {
    const uint32_t bar = smem_u32(&bars[slot]);
    if (wrapped) {
      if (!mbar_wait(bar, (phase_bits >> slot) & 1u, &abort_flag, err, ERRW_TIMEOUT_OTHER)) return;
      phase_bits ^= 1u << slot;
    }
    mbar_arrive_expect_tx(bar, load_bytes);
    bulk_load_1d(base + (uint32_t)slot * load_bytes, data + c * load_bytes, load_bytes, bar);
    if (++slot == stages) {
      slot = 0;
      wrapped = true;
    }
  }
  drain_ring(bars, slot, wrapped, stages, phase_bits, &abort_flag, err);
}

cudaError_t bulk1d_stream_prepare(int smem_bytes) {
  return stream_prepare(reinterpret_cast<const void*>(bulk1d_stream_kernel), smem_bytes);
}

// (bulk1d_stream_prepare must have run for this smem_bytes)
cudaError_t bulk1d_stream_launch(const void* data, uint64_t chunks, uint32_t load_bytes, int stages,
                                 int grid, int smem_bytes, uint32_t* err, cudaStream_t s) {
  bulk1d_stream_kernel<<<grid, 32, smem_bytes, s>>>(static_cast<const uint8_t*>(data), chunks,
                                                    load_bytes, stages, err);
  return cudaGetLastError();
}

}  // namespace b2g
