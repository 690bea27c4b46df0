// Host helper: encode a 2-D tiled TMA descriptor (no multicast anywhere).
#pragma once
#include <cuda.h>
#include <stdint.h>

namespace mirai {
int make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t elem_bytes, const void* base,
                 uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                 uint32_t box_outer, CUtensorMapSwizzle swizzle);
}
