// ah_tma.cuh — host-side TMA tensor-map encoding shared by the kernels that
// load tiles with cp.async.bulk.tensor (prefill GEMM, decode attention).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include "ah_common.cuh"

namespace ah {

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda);
// null when the driver does not provide it.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

// A row-major [rows][inner] matrix of `elem`-byte elements read in boxes of
// box_inner x box_rows; out-of-range box elements read as zero.
int encode_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint32_t elem, uint64_t inner,
              uint64_t rows, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swizzle);

}  // namespace ah
