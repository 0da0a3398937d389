// Repetition penalty, fused: restates _apply_repetition_penalty
// (litevllm/layers/sampler.py:190-201) as called from Sampler.sample
// (:168-171):
//   for each row i: ids = unique(past_token_ids[i])
//                   s = logits[i, ids]
//                   logits[i, ids] = s > 0 ? s / penalty : s * penalty
// with torch's arithmetic: the division and product in fp32 (IEEE, the
// penalty as fp32), rounded once to the logits dtype; negative ids index from
// the end of the row, as torch indexing does. Each distinct id is penalised
// once: one CTA per row marks the row's ids in a shared-memory bitmap (V bits)
// and the thread that clears an id's bit applies the penalty to it. Rows whose
// penalty is exactly 1 are left untouched (the reference's call is skipped for
// penalty 1.0). Ids outside [-V, V) are skipped and flagged in *status (the
// reference raises IndexError).
#include "lk_common.cuh"
#include "lk_host.h"

namespace {

constexpr int kPenThreads = 256;

template <typename T> LK_DEVINL T pen_round(float x);
template <> LK_DEVINL float pen_round<float>(float x) { return x; }
template <> LK_DEVINL __nv_bfloat16 pen_round<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <> LK_DEVINL __half pen_round<__half>(float x) { return __float2half_rn(x); }

template <typename T>
__global__ void __launch_bounds__(kPenThreads) repetition_penalty_kernel(
    T* logits, int V, int64_t ld, const int64_t* past, int64_t past_ld, int L,
    const float* penalties, int32_t* status) {
  extern __shared__ uint32_t seen[];  // ceil(V / 32) words
  const int b = blockIdx.x;
  const float pen = penalties[b];
  if (pen == 1.0f) return;
  const int words = (V + 31) >> 5;
  for (int w = threadIdx.x; w < words; w += kPenThreads) seen[w] = 0u;
  __syncthreads();
  const int64_t* prow = past + static_cast<int64_t>(b) * past_ld;
  auto norm = [&](int64_t id) -> int64_t { return id < 0 ? id + V : id; };
  for (int j = threadIdx.x; j < L; j += kPenThreads) {
    const int64_t id = norm(prow[j]);
    if (id < 0 || id >= V) {
      if (status) atomicOr(status, LK_STATUS_TOKEN_OOB);
      continue;
    }
    atomicOr(&seen[id >> 5], 1u << (id & 31));
  }
  __syncthreads();
  T* row = logits + static_cast<int64_t>(b) * ld;
  for (int j = threadIdx.x; j < L; j += kPenThreads) {
    const int64_t id = norm(prow[j]);
    if (id < 0 || id >= V) continue;
    const uint32_t bit = 1u << (id & 31);
    if ((atomicAnd(&seen[id >> 5], ~bit) & bit) == 0u) continue;  // another thread has it
    const float s = lk::Elem<T>::to_f(row[id]);
    row[id] = pen_round<T>(s > 0.f ? __fdiv_rn(s, pen) : __fmul_rn(s, pen));
  }
}

}  // namespace

extern "C" int lk_repetition_penalty(void* logits, int32_t B, int32_t V, int64_t ld,
                                     const int64_t* past_token_ids, int64_t past_ld, int32_t L,
                                     const float* penalties, int32_t* status, int32_t dtype,
                                     void* stream) {
  if (B < 0 || V <= 0 || ld < V || L < 0 || (L > 0 && past_ld < L)) return LK_ERR_INVALID_ARG;
  if (B == 0 || L == 0) return LK_OK;
  if (!logits || !past_token_ids || !penalties || B > 2147483647) return LK_ERR_INVALID_ARG;
  const size_t smem = static_cast<size_t>((V + 31) / 32) * 4;
  if (smem > 227 * 1024) return LK_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto launch = [&](auto* kernel, auto* ptr) -> int {
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return LK_ERR_CUDA;
    kernel<<<B, kPenThreads, smem, s>>>(ptr, V, ld, past_token_ids, past_ld, L, penalties,
                                         status);
    return lk::check_launch();
  };
  switch (dtype) {
    case LK_DTYPE_BF16:
      return launch(repetition_penalty_kernel<__nv_bfloat16>, static_cast<__nv_bfloat16*>(logits));
    case LK_DTYPE_F16:
      return launch(repetition_penalty_kernel<__half>, static_cast<__half*>(logits));
    case LK_DTYPE_F32:
      return launch(repetition_penalty_kernel<float>, static_cast<float*>(logits));
    default:
      return LK_ERR_UNSUPPORTED;
  }
}
