// Tiled TMA loads of row-major matrices (cp.async.bulk.tensor, no multicast).
#pragma once

#include <cuda.h>

#include "bulk.cuh"

namespace wgb {

// Tensor map over a row-major [rows, cols] matrix of `es`-byte elements
// (base and row pitch 16-byte aligned): boxes of 128 bytes of a row
// (128 / es elements) x box_rows rows, 128-byte swizzle (16-byte chunk c of
// box row r lands at chunk c ^ (r % 8); destinations 1024-byte aligned), zero
// fill outside the matrix. Built through the driver entry point (linear_tc.cu);
// false when the driver refuses the map.
bool tma_map_rows(CUtensorMap *tm, const void *base, int es, int rows, int cols, int box_rows);

// The same matrix (cols a multiple of 128 / es) viewed as
// (column % (128 / es), row, column / (128 / es)): a box holds `stages`
// consecutive 128-byte column blocks of box_rows rows, stored block after
// block (each block as one box of tma_map_rows would store it). One box of
// several blocks instead of several boxes: a warp's boxes complete about one
// at a time, so bytes per box set its bandwidth.
bool tma_map_row_stages(CUtensorMap *tm, const void *base, int es, int rows, int cols, int box_rows, int stages);

// Loads the box whose first element is (column x, row y); x * es must be a
// multiple of 16 bytes. Completion is counted on mbarrier bar.
__device__ __forceinline__ void tma_load_box(void *dst, const CUtensorMap *tm, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(tm), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_box3(void *dst, const CUtensorMap *tm, int x, int y, int z, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
            smem_u32(dst)),
        "l"(tm), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

}  // namespace wgb
