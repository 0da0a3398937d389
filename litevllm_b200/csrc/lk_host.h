// Host-side helpers shared by the entry points: error mapping, SM count per
// device, and a cache of TMA tensor maps over KV-cache tensors.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

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

// Programmatic dependent launch on (LITEKERN_PDL=0 turns it off; read once).
bool pdl_enabled();

// Launch `kernel` so that it may start while the previous kernel in the
// stream is still running (programmatic stream serialization). The kernel
// must call lk::pdl_wait() before it touches memory the previous kernels
// write and before it ends (so that its completion implies theirs). Falls back
// to an ordinary stream-ordered launch when PDL is off.
template <typename... KArgs, typename... Args>
cudaError_t launch_after_previous(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                  cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Shared-prefix attention for lk_paged_decode_shared_prefix (paged_prefill.cu).
int prefix_attention(const void* q, int64_t q_stride, const void* k_cache, const void* v_cache,
                     int64_t num_blocks, const int32_t* block_table_row, int B, int H, int H_kv,
                     int block_size, int prefix_len, int prefix_split, int num_ranges,
                     float scale, float* part_ml, float* part_o, int part_splits, int dtype,
                     int32_t* status, int* zeroed_counter, cudaStream_t s);

// Head of every decode workspace: the status word (padded to 256 B), then the
// split kernel's per-(sequence, head group) counters, which every completed
// call leaves zero and which no other use of the workspace may touch.
constexpr int64_t kDecodeMaxCounters = 65536;
constexpr size_t kDecodeHeadBytes = 256 + kDecodeMaxCounters * 4;

// Decode on the generic CUDA-core kernel (paged_generic.cu) for the shapes
// lk_paged_decode's split kernel does not take; split-KV with a merge launch
// when the workspace has room for the partials (placed after
// kDecodeHeadBytes, so a later split-kernel call on the same workspace finds
// its counters zero). Status bits go to the workspace's first word.
int generic_decode(void* out, int64_t out_token_stride, const void* q, int64_t q_token_stride,
                   const void* k_cache, const void* v_cache, int64_t num_blocks,
                   const int32_t* block_tables, int64_t block_table_stride,
                   const int32_t* context_lens, int B, int H, int H_kv, int D, int block_size,
                   int max_blocks_per_seq, float scale, int dtype, void* workspace,
                   size_t workspace_bytes, void* stream);

}  // namespace lk
