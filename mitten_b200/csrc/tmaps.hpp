// Host-side TMA tensor-map helpers shared by the attention kernels.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace mtn {

// Rows of the pool's 2-D [rows, head_dim] view.
int64_t pool_rows(const mtn_kv_layout* pool);

// Cached map over the whole pool: box = box_rows rows x 64 columns, 128B swizzle.  box_rows 0
// means one page of one kv head (page_size rows); num_kv_heads * page_size rows is one page
// of every kv head, which the pool layout keeps contiguous.
int pool_tensor_map(const mtn_kv_layout* pool, CUtensorMap* out, int box_rows = 0);

// Cached map that loads one page of one kv head, all of its head dim, in one box: the 4-D view
// (64 columns, 8 rows, head_dim/64 column blocks, rows/8) lands in shared memory as
// [page_size/8 row groups][head_dim/64 column blocks][8 rows][128 bytes], 128B-swizzled, so
// every 8-row x 64-column atom sits on its own 1024-byte boundary.  Coordinates:
// (0, 0, 0, first_row / 8); page_size must be a multiple of 8.
int pool_tensor_map_paged(const mtn_kv_layout* pool, CUtensorMap* out);

// Map over q [total_q][hq][d] bf16: box = box_rows tokens of one head x 64 columns, 128B swizzle.
int q_tensor_map(const void* q, int64_t total_q, int hq, int d, int box_rows, CUtensorMap* out);

}  // namespace mtn
