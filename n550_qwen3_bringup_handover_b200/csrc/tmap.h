// TMA tensor-map construction shared by the tcgen05 kernels (internal).
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace n550 {

// 2-D BF16 tensor [rows][cols] with a row stride of ld elements; the box is
// box_rows rows x 64 columns (one 128-byte swizzle row), SWIZZLE_128B,
// out-of-range elements read as zero. Returns N550_OK or an N550_ERR_* code.
int tmap_bf16_sw128(CUtensorMap *tm, const void *ptr, uint64_t rows, uint64_t cols, uint64_t ld,
                    int box_rows);
// 3-D variant [planes][rows][cols] (plane stride plane_ld elements), always a
// rank-3 map -- even for planes == 1 -- for use with tma_load_3d; the box is
// box_rows x 64 of one plane.
int tmap_bf16_sw128_3d(CUtensorMap *tm, const void *ptr, uint64_t rows, uint64_t cols,
                       uint64_t ld, int box_rows, uint64_t planes, uint64_t plane_ld);

}  // namespace n550
