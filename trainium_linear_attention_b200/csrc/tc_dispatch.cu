// Which tensor-core paths this build enables (each has its own kernel file:
// tc_chunked.cu, tc_parallel.cu, tc_sliding.cu).
#include "tc_kernels.cuh"

namespace la {
bool tc_chunked_enabled() { return true; }
bool tc_sliding_enabled() { return true; }
}  // namespace la
