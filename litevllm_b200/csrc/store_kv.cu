// KV-cache store: for each token t, copy key[t] / value[t] (H_kv * D values)
// into slot slot_mapping[t] of the paged cache. Restates the advanced-index
// scatter of litevllm/layers/attention.py:79-84 (= PagedAttention.write_to_cache,
// :18-33): key_cache[slot // bs, slot % bs] = key[t]. Because the cache is
// [num_blocks, bs, H_kv, D] contiguous, slot s starts at element s * H_kv * D,
// so the block / offset split is not needed at all.
//
// One CTA per token; its threads stream the K row and the V row with 16-byte
// loads and stores. The work is a pure copy (HBM bound, ~4 KiB per token for
// bf16 Llama-3-8B shapes).
#include "lk_common.cuh"
#include "lk_host.h"

namespace {

constexpr int kStoreThreads = 128;

template <bool VEC>
__global__ void __launch_bounds__(kStoreThreads)
store_kv_kernel(const uint8_t* __restrict__ key, const uint8_t* __restrict__ value,
                uint8_t* __restrict__ k_cache, uint8_t* __restrict__ v_cache,
                const int64_t* __restrict__ slot_mapping, int64_t key_stride_b,
                int64_t value_stride_b, int64_t row_bytes, int64_t num_slots,
                int32_t* __restrict__ status) {
  // The decode step's ordering kernel may start launching now: it waits for
  // this grid to complete before it reads or writes anything.
  lk::pdl_launch_dependents();
  const int t = blockIdx.x;
  const int64_t slot = slot_mapping[t];
  if (slot < 0 || slot >= num_slots) {
    if (slot != -1 && status != nullptr && threadIdx.x == 0) atomicOr(status, LK_STATUS_SLOT_OOB);
    return;
  }
  const uint8_t* ks = key + t * key_stride_b;
  const uint8_t* vs = value + t * value_stride_b;
  uint8_t* kd = k_cache + slot * row_bytes;
  uint8_t* vd = v_cache + slot * row_bytes;
  if constexpr (VEC) {
    const int n16 = static_cast<int>(row_bytes >> 4);
    for (int i = threadIdx.x; i < n16; i += kStoreThreads) {
      const uint4 a = __ldg(reinterpret_cast<const uint4*>(ks) + i);
      const uint4 b = __ldg(reinterpret_cast<const uint4*>(vs) + i);
      reinterpret_cast<uint4*>(kd)[i] = a;
      reinterpret_cast<uint4*>(vd)[i] = b;
    }
  } else {
    const int n2 = static_cast<int>(row_bytes >> 1);  // 16-bit granules (f16/bf16/f32 all even)
    for (int i = threadIdx.x; i < n2; i += kStoreThreads) {
      reinterpret_cast<uint16_t*>(kd)[i] = reinterpret_cast<const uint16_t*>(ks)[i];
      reinterpret_cast<uint16_t*>(vd)[i] = reinterpret_cast<const uint16_t*>(vs)[i];
    }
  }
}

}  // namespace

extern "C" int lk_store_kv(const void* key, const void* value, void* k_cache, void* v_cache,
                           const int64_t* slot_mapping, int32_t num_tokens,
                           int32_t num_kv_heads, int32_t head_dim, int64_t key_token_stride,
                           int64_t value_token_stride, int64_t num_slots, int32_t dtype,
                           int32_t* status, void* stream) {
  if (num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || num_slots < 0)
    return LK_ERR_INVALID_ARG;
  if (dtype != LK_DTYPE_F32 && dtype != LK_DTYPE_F16 && dtype != LK_DTYPE_BF16)
    return LK_ERR_UNSUPPORTED;
  if (num_tokens == 0) return LK_OK;
  if (!key || !value || !k_cache || !v_cache || !slot_mapping) return LK_ERR_INVALID_ARG;
  if (num_tokens > 0x7fffffff) return LK_ERR_INVALID_ARG;
  const int64_t esz = lk::dtype_size(dtype);
  const int64_t row_bytes = static_cast<int64_t>(num_kv_heads) * head_dim * esz;
  const int64_t ksb = key_token_stride * esz, vsb = value_token_stride * esz;
  const bool vec = ((reinterpret_cast<uintptr_t>(key) | reinterpret_cast<uintptr_t>(value) |
                     reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) &
                    15u) == 0 &&
                   (row_bytes & 15) == 0 && (ksb & 15) == 0 && (vsb & 15) == 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const auto* kp = static_cast<const uint8_t*>(key);
  const auto* vp = static_cast<const uint8_t*>(value);
  auto* kc = static_cast<uint8_t*>(k_cache);
  auto* vc = static_cast<uint8_t*>(v_cache);
  if (vec)
    store_kv_kernel<true><<<num_tokens, kStoreThreads, 0, s>>>(kp, vp, kc, vc, slot_mapping, ksb,
                                                               vsb, row_bytes, num_slots, status);
  else
    store_kv_kernel<false><<<num_tokens, kStoreThreads, 0, s>>>(kp, vp, kc, vc, slot_mapping, ksb,
                                                                vsb, row_bytes, num_slots, status);
  return lk::check_launch();
}
