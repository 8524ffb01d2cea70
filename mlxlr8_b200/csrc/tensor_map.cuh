// Host-side TMA tensor-map encoding (cuTensorMapEncodeTiled through the
// runtime's driver entry point, so the library links against libcudart only).
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace exlr8 {

// 2-D tiled map over a row-major [rows][inner] array of `type` elements with
// `row_bytes` between rows; boxes of box_inner x box_rows elements, no
// multicast anywhere.  False when the driver entry point is missing or the
// encode rejects the arguments.
bool encode_tiled_2d(CUtensorMap* map, CUtensorMapDataType type, const void* base, uint64_t inner, uint64_t rows,
                     uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swizzle);

}  // namespace exlr8
