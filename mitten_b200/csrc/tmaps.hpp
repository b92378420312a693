// Host-side TMA tensor-map helpers shared by the attention kernels.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace mtn {

// Rows of the pool's 2-D [rows, head_dim] view.
int64_t pool_rows(const mtn_kv_layout* pool);

// Cached map over the whole pool: box = one page of one kv head x 64 columns, 128B swizzle.
int pool_tensor_map(const mtn_kv_layout* pool, CUtensorMap* out);

// Map over q [total_q][hq][d] bf16: box = box_rows tokens of one head x 64 columns, 128B swizzle.
int q_tensor_map(const void* q, int64_t total_q, int hq, int d, int box_rows, CUtensorMap* out);

}  // namespace mtn
