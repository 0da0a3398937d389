// Fused q/k RMSNorm + rotary embedding + KV-cache store: the steps between the
// q/k/v projections and attention in Qwen3Attention.forward
// (litevllm/models/qwen3.py:76-92) and LlamaAttention.forward (no norm):
//   q = q_norm(q); k = k_norm(k)                   LlamaRMSNorm, models/llama.py:18-27
//   q = rope(q, pos); k = rope(k, pos)             apply_rotary_emb, layers/rotary_emb.py:104-117
//   key_cache[slot] = k; value_cache[slot] = v     layers/attention.py:79-84
// with the reference's rounding points: the normalised value is rounded to
// the 16-bit weight dtype, multiplied by the weight in that dtype, the
// rotation is computed in fp32 from the caller's fp32 cos / sin tables (the
// RotaryEmbedding cos_cached / sin_cached buffers) and rounded once when
// stored (and, when the caller asks, written back as the rotated k that an
// attention over the new tokens alone reads). One CTA per token, one warp per head (D = 128): lane l owns the
// rotation pairs (l, l + 64) and (l + 32, l + 96).
#include "lk_common.cuh"
#include "lk_host.h"

namespace {

constexpr int kRopeD = 128;

template <typename T> LK_DEVINL T from_f(float x);
template <> LK_DEVINL __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> LK_DEVINL __half from_f<__half>(float x) { return __float2half_rn(x); }

struct RopeParams {
  void* q;                 // [T, H, D], rotated in place
  int64_t q_stride;
  const void* k;           // [T, H_kv, D]
  int64_t k_stride;
  const void* v;
  int64_t v_stride;
  void* k_out;             // [T, H_kv, D] rotated k, or NULL
  int64_t k_out_stride;
  void* k_cache;           // [num_slots, H_kv, D]
  void* v_cache;
  const int64_t* slot_mapping;
  const int64_t* positions;
  const float* cos;        // [max_pos, D / 2]
  const float* sin;
  int64_t max_pos;
  const void* q_w;         // [D] or NULL (no norm)
  const void* k_w;
  float eps;
  int H, H_kv;
  int64_t num_slots;
  int32_t* status;
};

// Normalise (optional) and rotate one head row in registers: x[0..3] hold
// d = l, l + 32, l + 64, l + 96 of lane l.
template <typename T>
LK_DEVINL void norm_rope(float (&x)[4], const T* w, float eps, const float* cs, const float* sn,
                         int lane) {
  if (w != nullptr) {
    float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float r = rsqrtf(ss / static_cast<float>(kRopeD) + eps);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float n = lk::Elem<T>::to_f(from_f<T>(__fmul_rn(x[i], r)));  // .to(weight dtype)
      const float wi = lk::Elem<T>::to_f(w[lane + 32 * i]);
      x[i] = lk::Elem<T>::to_f(from_f<T>(__fmul_rn(wi, n)));            // weight * x, 16-bit
    }
  }
  // half split: (x1, x2) = (d < 64, d >= 64); pair index p = lane, lane + 32
  const float c0 = cs[lane], s0 = sn[lane], c1 = cs[lane + 32], s1 = sn[lane + 32];
  const float a0 = x[0], a1 = x[1], b0 = x[2], b1 = x[3];
  // separate roundings, as torch evaluates x1 * cos - x2 * sin (no fused multiply-add)
  x[0] = __fsub_rn(__fmul_rn(a0, c0), __fmul_rn(b0, s0));
  x[2] = __fadd_rn(__fmul_rn(b0, c0), __fmul_rn(a0, s0));
  x[1] = __fsub_rn(__fmul_rn(a1, c1), __fmul_rn(b1, s1));
  x[3] = __fadd_rn(__fmul_rn(b1, c1), __fmul_rn(a1, s1));
}

template <typename T>
__global__ void __launch_bounds__(256) rope_store_kernel(const RopeParams p) {
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  int64_t pos = p.positions[t];
  if (pos < 0 || pos >= p.max_pos) {
    if (threadIdx.x == 0 && p.status) atomicOr(p.status, LK_STATUS_CTX_OOB);
    pos = pos < 0 ? 0 : p.max_pos - 1;
  }
  const float* cs = p.cos + pos * (kRopeD / 2);
  const float* sn = p.sin + pos * (kRopeD / 2);
  const int64_t slot = p.slot_mapping ? p.slot_mapping[t] : -1;
  const bool store = slot >= 0 && slot < p.num_slots;
  if (p.slot_mapping && !store && slot != -1 && threadIdx.x == 0 && p.status)
    atomicOr(p.status, LK_STATUS_SLOT_OOB);
  // query heads
  for (int h = warp; h < p.H; h += nwarps) {
    T* row = static_cast<T*>(p.q) + t * p.q_stride + h * kRopeD;
    float x[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = lk::Elem<T>::to_f(row[lane + 32 * i]);
    norm_rope<T>(x, static_cast<const T*>(p.q_w), p.eps, cs, sn, lane);
#pragma unroll
    for (int i = 0; i < 4; ++i) row[lane + 32 * i] = from_f<T>(x[i]);
  }
  // key heads -> cache, value heads -> cache
  for (int h = warp; h < p.H_kv; h += nwarps) {
    const T* krow = static_cast<const T*>(p.k) + t * p.k_stride + h * kRopeD;
    float x[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = lk::Elem<T>::to_f(krow[lane + 32 * i]);
    norm_rope<T>(x, static_cast<const T*>(p.k_w), p.eps, cs, sn, lane);
    if (p.k_out) {
      T* ko = static_cast<T*>(p.k_out) + t * p.k_out_stride + h * kRopeD;
#pragma unroll
      for (int i = 0; i < 4; ++i) ko[lane + 32 * i] = from_f<T>(x[i]);
    }
    if (store) {
      T* kd = static_cast<T*>(p.k_cache) + (slot * p.H_kv + h) * kRopeD;
      T* vd = static_cast<T*>(p.v_cache) + (slot * p.H_kv + h) * kRopeD;
      const T* vrow = static_cast<const T*>(p.v) + t * p.v_stride + h * kRopeD;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        kd[lane + 32 * i] = from_f<T>(x[i]);
        vd[lane + 32 * i] = vrow[lane + 32 * i];
      }
    }
  }
}

}  // namespace

extern "C" int lk_rope_store_kv(void* q, int64_t q_token_stride, const void* k,
                                int64_t k_token_stride, const void* v, int64_t v_token_stride,
                                void* k_out, int64_t k_out_token_stride, void* k_cache, void* v_cache, int64_t num_slots,
                                const int64_t* slot_mapping, const int64_t* positions,
                                const float* cos_cache, const float* sin_cache, int64_t max_pos,
                                const void* q_norm_weight, const void* k_norm_weight, float eps,
                                int32_t num_tokens, int32_t H, int32_t H_kv, int32_t D,
                                int32_t dtype, int32_t* status, void* stream) {
  if (num_tokens < 0 || H <= 0 || H_kv <= 0 || max_pos <= 0) return LK_ERR_INVALID_ARG;
  if (num_tokens == 0) return LK_OK;
  if (D != kRopeD) return LK_ERR_UNSUPPORTED;
  if (dtype != LK_DTYPE_BF16 && dtype != LK_DTYPE_F16) return LK_ERR_UNSUPPORTED;
  if (!q || !k || !v || !positions || !cos_cache || !sin_cache) return LK_ERR_INVALID_ARG;
  if (slot_mapping && (!k_cache || !v_cache)) return LK_ERR_INVALID_ARG;
  RopeParams p;
  p.q = q;
  p.q_stride = q_token_stride;
  p.k = k;
  p.k_stride = k_token_stride;
  p.v = v;
  p.v_stride = v_token_stride;
  p.k_out = k_out;
  p.k_out_stride = k_out_token_stride;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.slot_mapping = slot_mapping;
  p.positions = positions;
  p.cos = cos_cache;
  p.sin = sin_cache;
  p.max_pos = max_pos;
  p.q_w = q_norm_weight;
  p.k_w = k_norm_weight;
  p.eps = eps;
  p.H = H;
  p.H_kv = H_kv;
  p.num_slots = num_slots;
  p.status = status;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == LK_DTYPE_BF16) rope_store_kernel<__nv_bfloat16><<<num_tokens, 256, 0, s>>>(p);
  else rope_store_kernel<__half><<<num_tokens, 256, 0, s>>>(p);
  return lk::check_launch();
}
