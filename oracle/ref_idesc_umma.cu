// Host program built against the reference's own umma_throughput/umma_tput.cu,
// included from where it lies (REF_SRC), to print the instruction descriptors
// its encoders produce (umma_tput.cu:190-255) for one (MMA_M, MMA_N).  The
// encoders are __device__ constexpr; --expt-relaxed-constexpr lets host code
// evaluate them.  Output: "umma <format> <M> <N> <idesc hex>" per format.
// Test infrastructure only (golden vectors for tests/test_descriptors.py).
#define main ref_umma_main
#include REF_SRC
#undef main
#include <cstdio>

int main() {
  printf("umma 0 %d %d 0x%08x\n", MMA_M, MMA_N, make_i_desc<MMAFormat::BF16>());
  printf("umma 1 %d %d 0x%08x\n", MMA_M, MMA_N, make_i_desc<MMAFormat::E4M3>());
  printf("umma 2 %d %d 0x%08x\n", MMA_M, MMA_N, make_i_desc<MMAFormat::S8>());
  printf("umma 3 %d %d 0x%08x\n", MMA_M, MMA_N, make_i_desc<MMAFormat::F4>());
  if (MMA_M >= 128) {
    printf("umma 4 %d %d 0x%08x\n", MMA_M, MMA_N, make_i_desc<MMAFormat::MXF8>());
    printf("umma 5 %d %d 0x%08x\n", MMA_M, MMA_N, make_i_desc<MMAFormat::MXF4>());
  }
  return 0;
}
