// Placeholder until the tcgen05 kernels land: the tensor-core path is off.
#include "tc_kernels.cuh"

namespace la {
bool tc_kernels_enabled() { return false; }
int launch_parallel_tc(const void *, const void *, const void *, void *, int64_t, int64_t, float,
                       const DeviceInfo &, cudaStream_t) { return LA_ERR_UNSUPPORTED; }
int launch_chunked_state_tc(const void *, const void *, float *, int64_t, int64_t, int, int,
                            int64_t, const DeviceInfo &, cudaStream_t) { return LA_ERR_UNSUPPORTED; }
int launch_chunked_output_tc(const void *, const void *, const void *, void *, const float *,
                             float *, const float *, int64_t, int64_t, float, bool, int, int64_t,
                             const DeviceInfo &, cudaStream_t) { return LA_ERR_UNSUPPORTED; }
int launch_sliding_tc(const void *, const void *, const void *, void *, int64_t, int64_t, int64_t,
                      const DeviceInfo &, cudaStream_t) { return LA_ERR_UNSUPPORTED; }
}  // namespace la
