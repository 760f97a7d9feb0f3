// Host-side construction of TMA tensor maps (CUtensorMap) for row-major
// 16-bit and 8-bit matrices.  The driver entry point cuTensorMapEncodeTiled is fetched
// through the runtime (cudaGetDriverEntryPoint), so the library does not link
// libcuda directly.
#pragma once

#include <cuda.h>

#include <cstdint>

namespace aotk {

// Encodes a 2-D map over a row-major [rows, cols] matrix of 16-bit elements
// with leading dimension `ld` (elements), box = box_cols x box_rows, 128-byte
// swizzle, zero fill outside the matrix.  Returns AOTK_OK or an error status.
int make_tmap_2d_16bit(CUtensorMap* map, const void* base, bool bf16, uint64_t rows, uint64_t cols,
                       uint64_t ld, uint32_t box_cols, uint32_t box_rows);

// The same for 8-bit elements (fp8 / int8 bytes), 128-byte swizzle.
int make_tmap_2d_8bit(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                      uint32_t box_cols, uint32_t box_rows);

// The same for fp32 elements.
int make_tmap_2d_f32(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                     uint32_t box_cols, uint32_t box_rows);

}  // namespace aotk
