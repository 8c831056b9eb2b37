// Host side of TMA: tensor-map encoding through the driver entry point (the
// library has no link-time dependency on libcuda).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

namespace la {

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)ptr;
    cudaGetLastError();
  });
  return fn;
}

// 3-D map over a contiguous (bh, n, d) bf16 tensor with a (1, box_rows, d)
// box; rows outside [0, n) read as zero.  False if it cannot be encoded (no
// driver entry point, base not 16-byte aligned, d * 2 not a multiple of 16).
inline bool make_tmap_3d(CUtensorMap *map, const void *base, int64_t bh, int64_t n, int d,
                         int box_rows, CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || ((uintptr_t)base & 15) || (d * 2) % 16) return false;
  cuuint64_t gdim[3] = {(cuuint64_t)d, (cuuint64_t)n, (cuuint64_t)bh};
  cuuint64_t gstride[2] = {(cuuint64_t)d * 2, (cuuint64_t)n * d * 2};
  cuuint32_t box[3] = {(cuuint32_t)d, (cuuint32_t)box_rows, 1};
  cuuint32_t estride[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), gdim, gstride,
            box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace la
