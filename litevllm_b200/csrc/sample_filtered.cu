// Fused top-k / top-p sampling. Restates the filtered branch of Sampler.sample
// (litevllm/layers/sampler.py:178-187 with _apply_top_k_top_p, :204-225):
//   p = softmax(x / T)
//   top-k: p[i] = 0 where p[i] < (k-th largest p)           (ties at the cut kept)
//   top-p: sort p descending, drop token j if sum(p before j) > top_p
//          (the sums use the top-k-filtered but not renormalised p)
//   renormalise, draw one token.
// Drawing argmax over the kept tokens of x / T + g, g Gumbel noise, samples the
// renormalised kept distribution exactly, so no probabilities are written.
//
// One CTA (1024 threads) per row. Each logit has an order-preserving integer
// key of its own width (16 bits for bf16 / f16, 32 for fp32), and both cut
// points are found with one 8-bit radix pass per key byte:
//   1. max of y = x / T and Z = sum exp(y - max)
//   2. top-k: radix select of the k-th largest key, high byte first
//   3. top-p: probability mass per key byte among the top-k survivors, scanned
//      from the top, gives the smallest key whose strictly-greater mass is
//      <= top_p, high byte first
//   4. Gumbel-max over keys >= max(both cuts).
// Tokens with equal keys are kept or dropped together (the reference's sort
// breaks such ties in an unspecified order). fp32 logits: distinct logits can
// round to the same probability, and the reference keeps every probability
// equal to the k-th largest; so for fp32 the top-k survivors are the tokens
// whose probability is >= that of the k-th largest key, not only its key and
// above.
#include "lk_common.cuh"
#include "lk_host.h"
#include "lk_philox.cuh"

namespace {

constexpr int kFT = 1024;

LK_DEVINL uint32_t order_key16(uint32_t h) {  // larger float -> larger key
  return (h & 0x8000u) ? (~h & 0xFFFFu) : (h | 0x8000u);
}

struct FilterParams {
  const void* logits;
  int64_t ld;
  int V;
  const float* temps;
  const int32_t* top_k;   // [B] or NULL (<= 0: off)
  const float* top_p;     // [B] or NULL (>= 1: off)
  const float* noise;
  int64_t noise_ld;
  uint32_t off_lo, off_hi;
  lk::PhiloxKey key;  // round keys of the seed
  int64_t* out;
};

// In-kernel noise: the main sampler's Philox stream and u -> Gumbel map
// (lk_philox.cuh), so that the filtered and unfiltered draws share one noise
// stream.
LK_DEVINL float gumbel_at(const FilterParams& p, int b, int v) {
  if (p.noise) return p.noise[static_cast<int64_t>(b) * p.noise_ld + v];
  const lk::U4 r = lk::philox4x32_10(
      lk::U4{static_cast<uint32_t>(v >> 2), static_cast<uint32_t>(b), p.off_lo, p.off_hi}, p.key);
  const uint32_t w = (v & 3) == 0 ? r.x : (v & 3) == 1 ? r.y : (v & 3) == 2 ? r.z : r.w;
  return lk::gumbel_from_bits(w);
}

template <typename T> LK_DEVINL uint32_t bits16(T x);
template <> LK_DEVINL uint32_t bits16<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat16_as_ushort(x); }
template <> LK_DEVINL uint32_t bits16<__half>(__half x) { return __half_as_ushort(x); }

// Order-preserving key of a logit and its width in bytes.
template <typename T> struct Key {
  static constexpr int kBytes = 2;
  LK_DEVINL static uint32_t of(T x) { return order_key16(bits16<T>(x)); }
};
template <> struct Key<float> {
  static constexpr int kBytes = 4;
  LK_DEVINL static uint32_t of(float x) {
    const uint32_t u = __float_as_uint(x);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  }
};

// Block-wide sums / maxima over kFT threads.
LK_DEVINL float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.f;
  for (int w = 0; w < kFT / 32; ++w) s += red[w];
  return s;
}
LK_DEVINL float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = -INFINITY;
  for (int w = 0; w < kFT / 32; ++w) s = fmaxf(s, red[w]);
  return s;
}

template <typename T>
__global__ void __launch_bounds__(kFT) sample_filtered_kernel(const FilterParams p) {
  __shared__ float red[kFT / 32];
  __shared__ float hmass[256];
  __shared__ unsigned int hcount[256];
  __shared__ int s_sel[2];
  __shared__ float s_kv[kFT / 32];
  __shared__ int s_ki[kFT / 32];
  const int b = blockIdx.x;
  const T* row = static_cast<const T*>(p.logits) + static_cast<int64_t>(b) * p.ld;
  const int V = p.V;
  const float temp = p.temps ? p.temps[b] : 0.f;
  const int k = p.top_k ? p.top_k[b] : 0;
  const float top_p = p.top_p ? p.top_p[b] : 1.f;
  const bool sampled = temp > 0.f;

  constexpr int kP = Key<T>::kBytes;
  uint32_t cut = 0;        // top-k: keep keys >= cut
  uint32_t pcut = 0;       // top-p: of the top-k survivors, keep keys >= pcut
  bool tie_rule = false;   // fp32 top-k: also keep probabilities >= p_kth
  float p_kth = 0.f, m = -INFINITY, inv_z = 0.f;
  // survivors of the top-k cut
  auto kept_k = [&](uint32_t key, float x) {
    if (key >= cut) return true;
    return tie_rule && expf(__fdiv_rn(x, temp) - m) * inv_z >= p_kth;
  };
  if (sampled) {
    // ---- 1. max and normaliser of y = x / T
    for (int v = threadIdx.x; v < V; v += kFT) m = fmaxf(m, __fdiv_rn(lk::Elem<T>::to_f(row[v]), temp));
    m = block_max(m, red);
    float z = 0.f;
    for (int v = threadIdx.x; v < V; v += kFT)
      z += expf(__fdiv_rn(lk::Elem<T>::to_f(row[v]), temp) - m);
    z = block_sum(z, red);
    inv_z = 1.f / z;

    // ---- 2. top-k cut: the k-th largest key (radix select, one byte a pass)
    if (k > 0 && k < V) {
      uint32_t prefix = 0;
      int need = k;
      for (int pass = 0; pass < kP; ++pass) {
        const int shift = 8 * (kP - 1 - pass);
        for (int i = threadIdx.x; i < 256; i += kFT) hcount[i] = 0u;
        __syncthreads();
        for (int v = threadIdx.x; v < V; v += kFT) {
          const uint32_t key = Key<T>::of(row[v]);
          // keys whose higher bytes equal the prefix found so far
          const bool in = pass == 0 || (key >> (shift + 8)) == prefix;
          if (in) atomicAdd(&hcount[(key >> shift) & 0xFFu], 1u);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
          int acc = 0, bin = 0;
          for (int i = 255; i >= 0; --i) {
            if (acc + static_cast<int>(hcount[i]) >= need) {
              bin = i;
              break;
            }
            acc += hcount[i];
          }
          s_sel[0] = bin;
          s_sel[1] = need - acc;
        }
        __syncthreads();
        prefix = (prefix << 8) | static_cast<uint32_t>(s_sel[0]);
        need = s_sel[1];
        __syncthreads();
      }
      cut = prefix;
      if constexpr (kP == 4) {
        // the k-th largest logit itself (keys map back one to one)
        const uint32_t u = (cut & 0x80000000u) ? (cut & 0x7FFFFFFFu) : ~cut;
        p_kth = expf(__fdiv_rn(__uint_as_float(u), temp) - m) * inv_z;
        tie_rule = true;
      }
    }
    // ---- 3. top-p cut over the survivors of top-k. A key v is kept iff the
    // mass of survivors with keys strictly above v is <= top_p. Each pass
    // finds, inside the bytes fixed so far, the byte where the running mass
    // (from the top) crosses top_p: keys in higher bytes are kept, lower ones
    // dropped.
    if (top_p < 1.f) {
      float above = 0.f;
      uint32_t prefix = 0;
      for (int pass = 0; pass < kP; ++pass) {
        const int shift = 8 * (kP - 1 - pass);
        for (int i = threadIdx.x; i < 256; i += kFT) hmass[i] = 0.f;
        __syncthreads();
        for (int v = threadIdx.x; v < V; v += kFT) {
          const T raw = row[v];
          const uint32_t key = Key<T>::of(raw);
          const float x = lk::Elem<T>::to_f(raw);
          if (!kept_k(key, x)) continue;
          if (pass > 0 && (key >> (shift + 8)) != prefix) continue;
          const float pv = expf(__fdiv_rn(x, temp) - m) * inv_z;
          atomicAdd(&hmass[(key >> shift) & 0xFFu], pv);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
          int bin = -1;
          float acc = above;
          for (int i = 255; i >= 0; --i) {
            if (hmass[i] > 0.f && acc + hmass[i] > top_p) {
              bin = i;
              break;
            }
            acc += hmass[i];
          }
          s_sel[0] = bin;
          red[0] = acc;
        }
        __syncthreads();
        const int bin = s_sel[0];
        const float acc = red[0];
        __syncthreads();
        if (bin < 0) {
          // pass 0: all survivors fit within top_p, no cut. A later pass
          // only if the lower-byte sums rounded differently from the
          // enclosing byte's sum: keep that whole byte.
          if (pass > 0) pcut = prefix << (shift + 8);
          break;
        }
        prefix = (prefix << 8) | static_cast<uint32_t>(bin);
        above = acc;
        if (pass == kP - 1) pcut = prefix;
      }
    }
  }

  // ---- 4. argmax of y + g over the kept keys (greedy rows: argmax x)
  float best = -INFINITY;
  int besti = 0x7fffffff;
  for (int v = threadIdx.x; v < V; v += kFT) {
    const T raw = row[v];
    const float x = lk::Elem<T>::to_f(raw);
    float key;
    if (!sampled) {
      key = x;
    } else {
      const uint32_t kx = Key<T>::of(raw);
      if (kx < pcut || !kept_k(kx, x)) continue;
      key = __fadd_rn(__fdiv_rn(x, temp), gumbel_at(p, b, v));
    }
    if (key > best || (key != key && best == best)) {
      best = key;
      besti = v;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float k2 = __shfl_xor_sync(0xffffffffu, best, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, besti, o);
    const bool n1 = best != best, n2 = k2 != k2;
    const bool take = (n2 != n1) ? n2 : (n2 ? i2 < besti : (k2 > best || (k2 == best && i2 < besti)));
    if (take) {
      best = k2;
      besti = i2;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    s_kv[threadIdx.x >> 5] = best;
    s_ki[threadIdx.x >> 5] = besti;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float kb = s_kv[0];
    int ib = s_ki[0];
    for (int w = 1; w < kFT / 32; ++w) {
      const float k2 = s_kv[w];
      const int i2 = s_ki[w];
      const bool n1 = kb != kb, n2 = k2 != k2;
      const bool take = (n2 != n1) ? n2 : (n2 ? i2 < ib : (k2 > kb || (k2 == kb && i2 < ib)));
      if (take) {
        kb = k2;
        ib = i2;
      }
    }
    p.out[b] = ib == 0x7fffffff ? 0 : ib;
  }
}

}  // namespace

extern "C" int lk_sample_filtered(int64_t* out_ids, const void* logits, int32_t B, int32_t V,
                                  int64_t ld, const float* temperatures, const int32_t* top_k,
                                  const float* top_p, const float* noise, int64_t noise_ld,
                                  uint64_t seed, uint64_t offset, int32_t dtype, void* stream) {
  if (B < 0 || V <= 0 || ld < V) return LK_ERR_INVALID_ARG;
  if (B == 0) return LK_OK;
  if (!out_ids || !logits || B > 0x7fffffff) return LK_ERR_INVALID_ARG;
  if (noise && noise_ld < V) return LK_ERR_INVALID_ARG;
  if (dtype != LK_DTYPE_BF16 && dtype != LK_DTYPE_F16 && dtype != LK_DTYPE_F32)
    return LK_ERR_UNSUPPORTED;
  FilterParams p;
  p.logits = logits;
  p.ld = ld;
  p.V = V;
  p.temps = temperatures;
  p.top_k = top_k;
  p.top_p = top_p;
  p.noise = noise;
  p.noise_ld = noise_ld;
  p.key = lk::philox_key(seed);
  p.off_lo = static_cast<uint32_t>(offset);
  p.off_hi = static_cast<uint32_t>(offset >> 32);
  p.out = out_ids;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == LK_DTYPE_BF16) sample_filtered_kernel<__nv_bfloat16><<<B, kFT, 0, s>>>(p);
  else if (dtype == LK_DTYPE_F16) sample_filtered_kernel<__half><<<B, kFT, 0, s>>>(p);
  else sample_filtered_kernel<float><<<B, kFT, 0, s>>>(p);
  return lk::check_launch();
}
