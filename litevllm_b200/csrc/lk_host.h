// Host-side helpers shared by the entry points: error mapping, SM count per
// device, and a cache of TMA tensor maps over KV-cache tensors.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/litekern.h"

namespace lk {

// Number of SMs of the current device (cached per device).
int num_sms();

// Map the last CUDA launch error to an LK code (clears the sticky-free error).
int check_launch();

// Tensor map over a KV cache [num_slots, H_kv, D] (slot = block * block_size +
// offset; the slot stride is H_kv * D elements) viewed as 3-D
// (d, slot, head) so that one box holds `box_heads` heads x `box_slots`
// consecutive slots x 64 values of d, laid out in shared memory as
// [head][slot][64] with 128-byte swizzle. Returns LK_OK or an error; maps are
// cached by (pointer, shape, box) for the life of the process.
int get_kv_tensor_map(CUtensorMap* out, const void* base, int64_t num_slots, int H_kv, int D,
                      int dtype, int box_slots, int box_heads);

inline int dtype_size(int dtype) { return dtype == LK_DTYPE_F32 ? 4 : 2; }

// Shared-prefix attention for lk_paged_decode_shared_prefix (paged_prefill.cu).
int prefix_attention(const void* q, int64_t q_stride, const void* k_cache, const void* v_cache,
                     int64_t num_blocks, const int32_t* block_table_row, int B, int H, int H_kv,
                     int block_size, int prefix_len, int prefix_split, int num_ranges,
                     float scale, float* part_ml, float* part_o, int part_splits, int dtype,
                     int32_t* status, int* zeroed_counter, cudaStream_t s);

}  // namespace lk
