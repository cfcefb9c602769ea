// tcgen05 weight-streaming projection (bf16) — placeholder until the kernel lands.
#include "linear.cuh"

namespace ssd {
bool linear_tc_supported(int, int, int) { return false; }
size_t linear_tc_workspace(int, int, int) { return 0; }
int linear_tc(cudaStream_t, const void*, const void*, void*, int, int, int, int, void*, size_t) {
  return SSD_ERR_UNSUPPORTED;
}
}  // namespace ssd
