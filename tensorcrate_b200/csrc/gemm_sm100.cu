// placeholder until the tcgen05 kernel lands
#include "gemm.cuh"
namespace tc {
int gemm_tc_run(int, int, size_t, size_t, size_t, const void *, const void *, void *, bool, cudaStream_t) {
  return TC_ENOTSUP;
}
}  // namespace tc
