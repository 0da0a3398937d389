// Block copies for copy-on-write forks and swaps. Restates the per-block
// loops of KVCache.swap_in / swap_out (litevllm/cache/kv_cache.py:74-102) and
// the copy that SchedulerOutput.blocks_to_copy (litevllm/engine/scheduler.py:25-27)
// asks for: for every (src, dst) pair and every layer,
//   dst_cache[layer][dst] = src_cache[layer][src]   for K and for V.
// One launch covers all pairs and layers: CTA (pair, cache) streams one
// block (block_size * H_kv * D values, 32 KiB for bf16 Llama-3-8B shapes)
// with 16-byte loads and stores. Source and destination caches are given by
// separate pointer tables, so pinned host caches (unified addressing) and
// device caches mix freely: device -> device for copy-on-write, host -> device
// for swap-in, device -> host for swap-out.
#include "lk_common.cuh"
#include "lk_host.h"

namespace {

constexpr int kCopyThreads = 256;

template <bool VEC>
__global__ void __launch_bounds__(kCopyThreads)
copy_blocks_kernel(const uint64_t* __restrict__ src_ptrs, const uint64_t* __restrict__ dst_ptrs,
                   const int64_t* __restrict__ mapping, int64_t block_bytes, int64_t src_blocks,
                   int64_t dst_blocks, int32_t* __restrict__ status) {
  const int pair = blockIdx.x, cache = blockIdx.y;  // cache = 2 * layer + (0: K, 1: V)
  const int64_t sb = mapping[2 * pair], db = mapping[2 * pair + 1];
  if (sb < 0 || sb >= src_blocks || db < 0 || db >= dst_blocks) {
    if (status != nullptr && threadIdx.x == 0) atomicOr(status, LK_STATUS_BLOCK_OOB);
    return;
  }
  const uint8_t* src = reinterpret_cast<const uint8_t*>(src_ptrs[cache]) + sb * block_bytes;
  uint8_t* dst = reinterpret_cast<uint8_t*>(dst_ptrs[cache]) + db * block_bytes;
  if constexpr (VEC) {
    const int64_t n = block_bytes >> 4;
    constexpr int kU = 4;
    int64_t i = threadIdx.x;
    for (; i + (kU - 1) * kCopyThreads < n; i += kU * kCopyThreads) {
      uint4 v[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) v[u] = reinterpret_cast<const uint4*>(src)[i + u * kCopyThreads];
#pragma unroll
      for (int u = 0; u < kU; ++u) reinterpret_cast<uint4*>(dst)[i + u * kCopyThreads] = v[u];
    }
    for (; i < n; i += kCopyThreads) reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
  } else {
    for (int64_t i = threadIdx.x; i < block_bytes; i += kCopyThreads) dst[i] = src[i];
  }
}

}  // namespace

extern "C" int lk_copy_blocks(const uint64_t* src_cache_ptrs, const uint64_t* dst_cache_ptrs,
                              int32_t num_layers, const int64_t* block_mapping, int32_t num_pairs,
                              int64_t block_bytes, int64_t src_num_blocks, int64_t dst_num_blocks,
                              int32_t* status, void* stream) {
  if (num_layers <= 0 || num_pairs < 0 || block_bytes <= 0 || src_num_blocks <= 0 ||
      dst_num_blocks <= 0)
    return LK_ERR_INVALID_ARG;
  if (num_pairs == 0) return LK_OK;
  if (!src_cache_ptrs || !dst_cache_ptrs || !block_mapping) return LK_ERR_INVALID_ARG;
  if (num_pairs > 0x7fffffff || 2LL * num_layers > 65535) return LK_ERR_INVALID_ARG;
  dim3 grid(num_pairs, 2 * num_layers);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The pointer tables live in device memory; 16-byte vectors need block_bytes
  // and every cache base 16-byte aligned, which the caller asserts by passing
  // block_bytes % 16 == 0 (cache tensors from the CUDA allocator and pinned
  // host allocations are 256-byte aligned).
  if ((block_bytes & 15) == 0)
    copy_blocks_kernel<true><<<grid, kCopyThreads, 0, s>>>(src_cache_ptrs, dst_cache_ptrs,
                                                          block_mapping, block_bytes,
                                                          src_num_blocks, dst_num_blocks, status);
  else
    copy_blocks_kernel<false><<<grid, kCopyThreads, 0, s>>>(src_cache_ptrs, dst_cache_ptrs,
                                                           block_mapping, block_bytes,
                                                           src_num_blocks, dst_num_blocks, status);
  return lk::check_launch();
}

extern "C" int lk_host_device_pointer(const void* host_ptr, uint64_t* device_ptr) {
  if (!host_ptr || !device_ptr) return LK_ERR_INVALID_ARG;
  void* d = nullptr;
  if (cudaHostGetDevicePointer(&d, const_cast<void*>(host_ptr), 0) != cudaSuccess || d == nullptr) {
    cudaGetLastError();  // clear the error of a non-pinned pointer
    return LK_ERR_INVALID_ARG;
  }
  *device_ptr = reinterpret_cast<uint64_t>(d);
  return LK_OK;
}
