// Host-side TMA tensor-map construction (see tma_host.cpp).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/ptxstd.h"

namespace ptxstd {

// 2-D tiled map over a row-major [outer, inner] tensor with the given row stride (bytes), box
// box_inner x box_outer elements. Returns a ptxstd_status.
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint64_t inner,
                 uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                 uint32_t box_outer, CUtensorMapSwizzle swizzle);

}  // namespace ptxstd
