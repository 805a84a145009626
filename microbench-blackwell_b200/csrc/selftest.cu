// selftest.cu -- b2g_selftest_wait: the engine's failure detection, exercised
// without a fault.
//
// The reference's waits are unbounded spins (umma_throughput/umma_tput.cu:510-520):
// a lost arrival there hangs the GPU.  Every wait of this engine is bounded
// instead.  This kernel makes one such wait run out on purpose, with nothing else
// in flight (no TMA, no MMA, no TMEM held): one warp waits, through the same
// bounded-wait code the GEMM uses and with the handle's wait limit, on
//   mode 0: phase 0 of an mbarrier whose one pending arrival never comes (the
//           ring and accumulator barriers of the GEMM), or
//   mode 1: a global word that no thread sets (the split-tail epilogue's flag).
// On expiry the waiter records ERRW_TIMEOUT_OTHER in the error word and the
// kernel returns; the host reads B2G_ERR_TIMEOUT through b2g_check and the
// context stays usable.
#include <cuda_runtime.h>
#include <stdint.h>

#include "b2g_gemm.h"
#include "b2g_ptx.cuh"

namespace b2g {

__global__ void __launch_bounds__(32, 1)
    wait_selftest_kernel(int mode, uint64_t limit_ns, const uint32_t* flag, uint32_t* err,
                         unsigned long long* elapsed_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncwarp();
  const uint64_t t0 = globaltimer_ns();
  bool ok;
  if (mode == 0) {
    // every lane waits, as the GEMM's roles do; the first to expire raises the
    // abort flag and the others return on it
    ok = mbar_wait(smem_u32(&bar), 0, &abort_flag, err, ERRW_TIMEOUT_OTHER, limit_ns);
  } else {
    // one lane polls, as the split-tail epilogue does; the result is shared
    bool got = true;
    if (threadIdx.x == 0) got = flag_wait(flag, 1u, &abort_flag, err, ERRW_TIMEOUT_OTHER, limit_ns);
    ok = __shfl_sync(0xffffffffu, got ? 1 : 0, 0) != 0;
  }
  ok = __all_sync(0xffffffffu, ok);
  if (threadIdx.x == 0) elapsed_ns[0] = ok ? 0ull : (unsigned long long)(globaltimer_ns() - t0);
}

cudaError_t wait_selftest_launch(int mode, uint64_t limit_ns, const uint32_t* flag, uint32_t* err,
                                 unsigned long long* elapsed_ns, cudaStream_t s) {
  wait_selftest_kernel<<<1, 32, 0, s>>>(mode, limit_ns, flag, err, elapsed_ns);
  return cudaGetLastError();
}

}  // namespace b2g
