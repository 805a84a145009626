// Host program built against the reference's own
// tcgen05_sparse_mma/tcgen05_sparse_mma.cu, included from where it lies
// (REF_SRC), to print the instruction descriptor its encoder produces
// (tcgen05_sparse_mma.cu:191-228) for the -D configuration it was built with.
// Output: "sparse <kind> <a> <b> <sparsity> <M> <N> <scale> <idesc hex>".
// Test infrastructure only (golden vectors for tests/test_descriptors.py).
#define main ref_sparse_main
#include REF_SRC
#undef main
#include <cstdio>

int main() {
  printf("sparse %d %d %d %d %d %d %d 0x%08x\n", KIND_ID, A_TYPE_CODE, B_TYPE_CODE, SPARSITY,
         MMA_M, MMA_N, SCALE_TYPE_ID, make_i_desc());
  return 0;
}
