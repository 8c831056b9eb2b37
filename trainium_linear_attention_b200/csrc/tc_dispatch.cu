// Tensor-core kernels not yet specialised in this build report themselves off.
#include "tc_kernels.cuh"

namespace la {
bool tc_chunked_enabled() { return true; }
bool tc_parallel_enabled() { return false; }
bool tc_sliding_enabled() { return true; }
int launch_parallel_tc(const void *, const void *, const void *, void *, int64_t, int64_t, float,
                       const DeviceInfo &, cudaStream_t) { return LA_ERR_UNSUPPORTED; }
}  // namespace la
