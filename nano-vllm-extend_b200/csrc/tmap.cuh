// Tensor-map (TMA descriptor) encoding through the driver entry point fetched
// at run time, so the library needs no link-time libcuda dependency.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace gdn {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled, or nullptr when the driver does not provide it.
EncodeTiledFn encode_tiled();

}  // namespace gdn
