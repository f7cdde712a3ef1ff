// tma_host.h -- host-side creation of TMA tensor maps (cuTensorMapEncodeTiled through the
// runtime's driver entry point, so the library does not link libcuda directly).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace dudy {

// 2-D tiled map over a row-major [dim1][dim0] matrix of 16-bit elements.
// swizzle_bytes: 0 (none), 32, 64 or 128. Out-of-bounds reads fill with zero.
// Returns false (with the error recorded) if the driver rejects the map.
bool make_tmap_2d(CUtensorMap *map, const void *base, bool bf16, uint64_t dim0, uint64_t dim1,
                  uint64_t row_stride_bytes, uint32_t box0, uint32_t box1, int swizzle_bytes);

}  // namespace dudy
