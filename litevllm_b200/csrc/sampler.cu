// Vocab-wide sampler: one pass over each logits row picks
//   greedy rows (T == 0):  argmax_v float(x[v])
//   sampled rows (T > 0):  argmax_v float(x[v]) / T + g[v]     (Gumbel-max)
// Restates Sampler.sample, litevllm/layers/sampler.py:147-187: the greedy
// branch (_triton_argmax / _argmax_kernel, :60-84, :111-124: fp32 compare,
// first index wins ties) and the temperature branch (:178, :187,
// softmax(x / T) then a categorical draw). Gumbel-max draws from exactly
// softmax(x / T); the draw is a pure function of the noise g, so it is
// reproducible from a noise tensor, which torch.multinomial's is not.
//
// B200 design: the vocabulary of each row is cut into chunks, one CTA per
// (chunk, row). Each thread streams 16-byte vectors (8 16-bit logits) with
// several loads in flight, keeps a running (key, index) best, and the CTA
// reduces with warp shuffles then shared memory. The last CTA of a row to
// finish (atomic counter, no waiting) reduces the per-chunk winners and
// writes the int64 token id; all-greedy rows with 2-8 chunks merge inside a
// thread-block cluster instead. Three kernels share this frame:
//   argmax_kernel  all-greedy 16-bit rows, HBM bound: few long chunks
//                  (ceil(SMs / B) per row);
//   gumbel_kernel  in-kernel-noise 16-bit rows, bound by instruction issue:
//                  max(4, ceil(256 / B)) equal chunks per row; vectors whose
//                  key bound cannot beat the CTA's best key are skipped
//                  (exactly), most of them right after their Philox words;
//   sample_kernel  everything else (a noise tensor, fp32 logits, unaligned
//                  rows), one wave of chunks.
//
// In-kernel noise (lk_philox.cuh): u = ((r >> 9) + 0.5) * 2^-23 with r from
// Philox4x32-10 keyed by the 64-bit seed, counter (v / 4, b, offset_lo,
// offset_hi); word v % 4 of the block feeds element v; g = -ln(-ln u) from
// hardware base-2 logarithms (within 5e-7 relative of the exact value).
#include "lk_common.cuh"
#include "lk_host.h"
#include "lk_philox.cuh"

#include <cooperative_groups.h>
#include <stdlib.h>

#include <mutex>
#include <type_traits>

namespace cg = cooperative_groups;

namespace {

constexpr int kSampThreads = 256;
constexpr int kVec = 8;  // elements per 16-byte vector of 16-bit logits
constexpr int kSampCtasPerSm = 6;
constexpr int kGumbelCtasPerSm = 4;

struct SampleParams {
  const void* logits;
  int64_t ld;
  int V;
  int chunk;      // elements per CTA (multiple of kVec)
  int nchunks;
  const float* temps;
  const float* noise;
  int64_t noise_ld;
  uint32_t off_lo, off_hi;
  lk::PhiloxKey key;  // round keys of the seed
  float* noise_dump;
  int64_t* out;
  float* part_key;   // [B][nchunks]
  int32_t* part_idx; // [B][nchunks]
  int32_t* counters; // [B]
  int nv;             // whole 16-byte vectors per row
  int gumbel;         // 1: gumbel_kernel takes the call
};

using lk::U4;

// ---------------------------------------------------------- comparisons ---
// a beats the current best (b) if it is larger, or NaN where b is not; the
// caller visits indices in increasing order so equal keys keep the earlier.
LK_DEVINL bool beats_later(float a, float b) {
  return a > b || (a != a && b == b);
}
// NaN-propagating fp32 max.
LK_DEVINL float fmax_nan(float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}
// Full comparison for merging two candidates with explicit indices.
LK_DEVINL bool beats(float ka, int ia, float kb, int ib) {
  const bool na = ka != ka, nb = kb != kb;
  if (na != nb) return na;
  if (na) return ia < ib;
  return ka > kb || (ka == kb && ia < ib);
}

template <typename T> struct Load16;
template <> struct Load16<__nv_bfloat16> {
  LK_DEVINL static void cvt(const uint4& v, float (&f)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
};
template <> struct Load16<__half> {
  LK_DEVINL static void cvt(const uint4& v, float (&f)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      float2 t = __half22float2(h);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
};
template <> struct Load16<float> {};

template <typename T, bool VEC, int MODE>  // MODE 0 greedy, 1 noise tensor, 2 in-kernel RNG
LK_DEVINL void scan_chunk(const SampleParams& p, int b, int v0, int v1, float temp, float& best,
                          int& besti) {
  const T* row = static_cast<const T*>(p.logits) + static_cast<int64_t>(b) * p.ld;
  const float* nrow = MODE == 1 ? p.noise + static_cast<int64_t>(b) * p.noise_ld : nullptr;
  float* drow = (MODE == 2 && p.noise_dump) ? p.noise_dump + static_cast<int64_t>(b) * p.V : nullptr;

  auto visit = [&](float x, int v, float g) {
    float key;
    if constexpr (MODE == 0) key = x;
    else key = __fadd_rn(__fdiv_rn(x, temp), g);
    if (beats_later(key, best)) {
      best = key;
      besti = v;
    }
  };

  int vs = v0;
  if constexpr (VEC && !std::is_same<T, float>::value) {
    const int vend = v0 + ((min(v1, p.V) - v0) / kVec) * kVec;
    constexpr int kU = 4;
    // One 16-byte vector of logits at element vv (its noise loaded or drawn here).
    auto process = [&](const uint4& raw, int vv) {
      float f[8];
      Load16<T>::cvt(raw, f);
      float g[8];
      if constexpr (MODE == 1) {
        const float4 a = __ldcs(reinterpret_cast<const float4*>(nrow + vv));
        const float4 c = __ldcs(reinterpret_cast<const float4*>(nrow + vv + 4));
        g[0] = a.x; g[1] = a.y; g[2] = a.z; g[3] = a.w;
        g[4] = c.x; g[5] = c.y; g[6] = c.z; g[7] = c.w;
      } else if constexpr (MODE == 2) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const U4 r = lk::philox4x32_10(U4{static_cast<uint32_t>((vv >> 2) + h),
                                            static_cast<uint32_t>(b), p.off_lo, p.off_hi},
                                         p.key);
          g[4 * h + 0] = lk::gumbel_from_bits(r.x);
          g[4 * h + 1] = lk::gumbel_from_bits(r.y);
          g[4 * h + 2] = lk::gumbel_from_bits(r.z);
          g[4 * h + 3] = lk::gumbel_from_bits(r.w);
        }
        if (drow) {
          reinterpret_cast<float4*>(drow + vv)[0] = make_float4(g[0], g[1], g[2], g[3]);
          reinterpret_cast<float4*>(drow + vv)[1] = make_float4(g[4], g[5], g[6], g[7]);
        }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) visit(f[e], vv + e, MODE == 0 ? 0.f : g[e]);
    };
    constexpr int kS = kSampThreads * kVec;
    int v = v0 + threadIdx.x * kVec;
    for (; v + (kU - 1) * kS < vend; v += kU * kS) {
      uint4 raw[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) raw[u] = __ldcs(reinterpret_cast<const uint4*>(row + v + u * kS));
      if constexpr (MODE == 2) {
        // in-kernel noise is compute-bound: one copy of the (large) body keeps
        // the loop in the instruction cache
#pragma unroll 1
        for (int u = 0; u < kU; ++u) process(raw[u], v + u * kS);
      } else {
#pragma unroll
        for (int u = 0; u < kU; ++u) process(raw[u], v + u * kS);
      }
    }
    if (v < vend) {  // fewer than kU vectors left: one predicated batch
      uint4 raw[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u)
        if (v + u * kS < vend) raw[u] = __ldcs(reinterpret_cast<const uint4*>(row + v + u * kS));
      if constexpr (MODE == 2) {
#pragma unroll 1
        for (int u = 0; u < kU; ++u)
          if (v + u * kS < vend) process(raw[u], v + u * kS);
      } else {
#pragma unroll
        for (int u = 0; u < kU; ++u)
          if (v + u * kS < vend) process(raw[u], v + u * kS);
      }
    }
    vs = vend;
  }
  // Scalar path: unaligned rows, fp32 logits, and the ragged tail.
  const int vend = min(v1, p.V);
  for (int v = vs + threadIdx.x; v < vend; v += kSampThreads) {
    const float x = lk::Elem<T>::to_f(row[v]);
    float g = 0.f;
    if constexpr (MODE == 1) {
      g = nrow[v];
    } else if constexpr (MODE == 2) {
      const U4 r = lk::philox4x32_10(U4{static_cast<uint32_t>(v >> 2), static_cast<uint32_t>(b),
                                        p.off_lo, p.off_hi},
                                     p.key);
      const uint32_t w = (v & 3) == 0 ? r.x : (v & 3) == 1 ? r.y : (v & 3) == 2 ? r.z : r.w;
      g = lk::gumbel_from_bits(w);
      if (drow) drow[v] = g;
    }
    visit(x, v, g);
  }
}

LK_DEVINL void reduce_pair(float& k, int& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float k2 = __shfl_xor_sync(0xffffffffu, k, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, i, o);
    if (beats(k2, i2, k, i)) {
      k = k2;
      i = i2;
    }
  }
}

// Block-wide (key, index) reduction; result valid in thread 0.
LK_DEVINL void block_reduce(float& k, int& i) {
  __shared__ float sk[kSampThreads / 32];
  __shared__ int si[kSampThreads / 32];
  reduce_pair(k, i);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    sk[w] = k;
    si[w] = i;
  }
  __syncthreads();
  if (w == 0) {
    k = l < kSampThreads / 32 ? sk[l] : -INFINITY;
    i = l < kSampThreads / 32 ? si[l] : 0x7fffffff;
    reduce_pair(k, i);
  }
}

// Block winner -> row result: a one-chunk row writes its id; otherwise the
// chunk's winner goes to the workspace and the row's last CTA to finish
// (atomic counter, no waiting) reduces the winners and resets the counter.
LK_DEVINL void finish_row(const SampleParams& p, int b, int ch, float best, int besti) {
  block_reduce(best, besti);
  if (p.nchunks == 1) {
    if (threadIdx.x == 0) p.out[b] = besti == 0x7fffffff ? 0 : besti;
    return;
  }
  __shared__ int s_last;
  if (threadIdx.x == 0) {
    p.part_key[static_cast<int64_t>(b) * p.nchunks + ch] = best;
    p.part_idx[static_cast<int64_t>(b) * p.nchunks + ch] = besti;
    __threadfence();
    const int prev = atomicAdd(p.counters + b, 1);
    s_last = prev == p.nchunks - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  float k = -INFINITY;
  int i = 0x7fffffff;
  for (int c = threadIdx.x; c < p.nchunks; c += kSampThreads) {
    const float k2 = __ldcg(p.part_key + static_cast<int64_t>(b) * p.nchunks + c);
    const int i2 = __ldcg(p.part_idx + static_cast<int64_t>(b) * p.nchunks + c);
    if (beats(k2, i2, k, i)) {
      k = k2;
      i = i2;
    }
  }
  block_reduce(k, i);
  if (threadIdx.x == 0) {
    p.out[b] = i == 0x7fffffff ? 0 : i;
    p.counters[b] = 0;
  }
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(kSampThreads, kSampCtasPerSm) sample_kernel(const SampleParams p) {
  lk::pdl_wait();  // launched to overlap the kernel ahead of it: wait for it before reading
  // a kernel launched after this one may place its CTAs in the SM slots this grid
  // leaves free (it still waits for this grid to complete before reading)
  lk::pdl_launch_dependents();
  const int ch = blockIdx.x, b = blockIdx.y;
  const float temp = p.temps ? p.temps[b] : 0.f;
  const int v0 = ch * p.chunk, v1 = min(p.V, v0 + p.chunk);
  float best = -INFINITY;
  int besti = 0x7fffffff;
  if (!(temp > 0.f)) scan_chunk<T, VEC, 0>(p, b, v0, v1, temp, best, besti);
  else if (p.noise) scan_chunk<T, VEC, 1>(p, b, v0, v1, temp, best, besti);
  else scan_chunk<T, VEC, 2>(p, b, v0, v1, temp, best, besti);
  finish_row(p, b, ch, best, besti);
}

// In-kernel-noise rows of 16-bit logits (16-byte aligned rows, gumbel_kernel
// below): the sampled path of config 4 / 5. It is bound by instruction issue, not HBM: per
// element a quarter Philox block, and for the few vectors whose key bound can
// beat the CTA's best (gumbel_segment) two hardware logarithms and the
// division, so every step here is trimmed to few instructions:
//  * Philox round keys arrive as kernel parameters (constant operands);
//  * x / T is the IEEE quotient computed as in Markstein's theorem (P.
//    Markstein, "Computation of elementary functions on the IBM RISC
//    System/6000 processor", IBM J. Res. Dev. 34(1), 1990): with y = RN(1/T)
//    and q0 = RN(x y), r = x - q0 T is exact and RN(q0 + r y) is the
//    correctly rounded x / T when nothing underflows or overflows. Vectors
//    with an element outside [xlo, xhi] (zeros, infinities, NaN, tiny or
//    huge values for this T) take __fdiv_rn instead; tested against IEEE
//    division over every 16-bit value;
//  * the running best is compared once per 8-element vector (NaN-propagating
//    max of its keys); only a vector that improves it is searched for the
//    element, which after the first few vectors is rare.
struct FastDiv {
  float t, y, xlo, xhi;
  LK_DEVINL static FastDiv make(float temp) {
    FastDiv d;
    d.t = temp;
    d.y = __frcp_rn(temp);
    // |x| in [xlo, xhi] keeps q0, r and the result normal and finite
    const bool ok = temp >= 0x1p-60f && temp <= 0x1p60f;
    d.xlo = ok ? 0x1p-98f * fmaxf(1.f, temp) : INFINITY;
    d.xhi = ok ? 0x1p98f * fminf(1.f, temp) : 0.f;
    return d;
  }
  LK_DEVINL bool in_range(float x) const { return fabsf(x) >= xlo && fabsf(x) <= xhi; }
  LK_DEVINL float fast(float x) const {
    const float q0 = __fmul_rn(x, y);
    const float r = fmaf(-q0, t, x);
    return fmaf(r, y, q0);
  }
};

// The 8 keys of one 16-byte vector from its logits f and its two Philox
// blocks r (words 0-3: elements vv..vv+3, 4-7: vv+4..vv+7).
LK_DEVINL void gumbel_keys(const FastDiv& dv, int vv, const float (&f)[8], const U4 (&r)[2],
                           float (&key)[8], float* drow) {
  float g[8];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    g[4 * h + 0] = lk::gumbel_from_bits(r[h].x);
    g[4 * h + 1] = lk::gumbel_from_bits(r[h].y);
    g[4 * h + 2] = lk::gumbel_from_bits(r[h].z);
    g[4 * h + 3] = lk::gumbel_from_bits(r[h].w);
  }
  if (drow) {
    reinterpret_cast<float4*>(drow + vv)[0] = make_float4(g[0], g[1], g[2], g[3]);
    reinterpret_cast<float4*>(drow + vv)[1] = make_float4(g[4], g[5], g[6], g[7]);
  }
  bool fast = true;
#pragma unroll
  for (int e = 0; e < 8; ++e) fast = fast && dv.in_range(f[e]);
  float q[8];
  if (fast) {
#pragma unroll
    for (int e = 0; e < 8; ++e) q[e] = dv.fast(f[e]);
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) q[e] = __fdiv_rn(f[e], dv.t);
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) key[e] = __fadd_rn(q[e], g[e]);
}

// fp32 <-> int with the same order (for atomicMax on keys); NaN (positive
// sign bit clear) maps above +infinity.
LK_DEVINL int float_to_ordered(float x) {
  const int i = __float_as_int(x);
  return i >= 0 ? i : i ^ 0x7fffffff;
}
LK_DEVINL float ordered_to_float(int i) { return __int_as_float(i >= 0 ? i : i ^ 0x7fffffff); }

// Margin added to the vector bound's Gumbel value: the map is within 2e-5
// of the exact, monotone -ln(-ln u) everywhere (tested over all uniforms),
// so g(u_e) <= g(u_max) + 4e-5 for every element of the vector.
constexpr float kGumbelBoundMargin = 1e-3f;

// ---------------------------------------------------- softmax(x / T) ---
template <typename T>
__global__ void __launch_bounds__(kSampThreads)
softmax_temp_kernel(float* __restrict__ probs, int64_t probs_ld, const T* __restrict__ logits,
                    int V, int64_t ld, const float* __restrict__ temps) {
  const int b = blockIdx.x;
  const T* row = logits + static_cast<int64_t>(b) * ld;
  const float t = temps ? temps[b] : 1.f;
  float m = -INFINITY, s = 0.f;
  for (int v = threadIdx.x; v < V; v += kSampThreads) {
    const float x = __fdiv_rn(lk::Elem<T>::to_f(row[v]), t);
    if (x > m) {
      s = s * __expf(m - x) + 1.f;
      m = x;
    } else {
      s += __expf(x - m);
    }
  }
  __shared__ float sm[kSampThreads / 32], ss[kSampThreads / 32];
  __shared__ float gm, gs;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    const float mm = fmaxf(m, m2);
    s = (m == -INFINITY ? 0.f : s * __expf(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mm));
    m = mm;
  }
  if ((threadIdx.x & 31) == 0) {
    sm[threadIdx.x >> 5] = m;
    ss[threadIdx.x >> 5] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = -INFINITY;
    for (int w = 0; w < kSampThreads / 32; ++w) M = fmaxf(M, sm[w]);
    float S = 0.f;
    for (int w = 0; w < kSampThreads / 32; ++w)
      S += sm[w] == -INFINITY ? 0.f : ss[w] * __expf(sm[w] - M);
    gm = M;
    gs = S;
  }
  __syncthreads();
  const float M = gm, inv = 1.f / gs;
  float* prow = probs + static_cast<int64_t>(b) * probs_ld;
  for (int v = threadIdx.x; v < V; v += kSampThreads)
    prow[v] = __expf(__fdiv_rn(lk::Elem<T>::to_f(row[v]), t) - M) * inv;
}


// ---------------------------------------------------- greedy-only kernel ---
// All rows greedy (temperatures == NULL), 16-bit logits, 16-byte aligned
// rows: the vector max of 8 values is taken with packed NaN-propagating
// max instructions, and the first index of that max is searched only when
// it beats the thread's running best, so the common path is three packed
// max operations per 8 logits.
// Packed NaN-propagating max of two 16-bit pairs, and NaN-propagating fp32 max.
template <typename T> LK_DEVINL uint32_t pmax_nan(uint32_t a, uint32_t b);
template <> LK_DEVINL uint32_t pmax_nan<__nv_bfloat16>(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
template <> LK_DEVINL uint32_t pmax_nan<__half>(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.NaN.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
template <typename T> LK_DEVINL float half_lo(uint32_t w);
template <typename T> LK_DEVINL float half_hi(uint32_t w);
template <> LK_DEVINL float half_lo<__nv_bfloat16>(uint32_t w) { return __uint_as_float(w << 16); }
template <> LK_DEVINL float half_hi<__nv_bfloat16>(uint32_t w) {
  return __uint_as_float(w & 0xffff0000u);
}
template <> LK_DEVINL float half_lo<__half>(uint32_t w) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xffffu)));
}
template <> LK_DEVINL float half_hi<__half>(uint32_t w) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16)));
}

// Bits of a 16-bit float that compare equal to vm, and the NaN test, in the
// raw 16-bit encoding (exact: vm came from one of these values).
template <typename T> LK_DEVINL uint32_t to_bits16(float vm);
template <> LK_DEVINL uint32_t to_bits16<__nv_bfloat16>(float vm) {
  return __float_as_uint(vm) >> 16;
}
template <> LK_DEVINL uint32_t to_bits16<__half>(float vm) {
  return __half_as_ushort(__float2half_rn(vm));
}
template <typename T> LK_DEVINL bool is_nan16(uint32_t h);
template <> LK_DEVINL bool is_nan16<__nv_bfloat16>(uint32_t h) { return (h & 0x7fffu) > 0x7f80u; }
template <> LK_DEVINL bool is_nan16<__half>(uint32_t h) { return (h & 0x7fffu) > 0x7c00u; }

// The vector holds a new running best: index (0..7) of its first occurrence.
// +0 and -0 compare equal, as in the fp32 comparison.
template <typename T>
LK_DEVINL int first_index_of(const uint4& raw, float vm) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
  const bool want_nan = vm != vm;
  const uint32_t hv = to_bits16<T>(vm);
  int e = 8;
#pragma unroll
  for (int k = 7; k >= 0; --k) {
    const uint32_t h = (k & 1) ? (w[k >> 1] >> 16) : (w[k >> 1] & 0xffffu);
    const bool hit = want_nan ? is_nan16<T>(h) : (h == hv || ((h | hv) & 0x7fffu) == 0u);
    e = hit ? k : e;
  }
  return e;
}

// Running best over 16-byte vectors: the value, the START of the first
// vector that holds it (strict comparison, increasing order) and that vector
// itself; the element inside it is found once, at the end, by resolve_index.
// Searching it on every improvement costs more than the whole scan: the
// compiler if-converts the search into every iteration.
template <typename T>
LK_DEVINL void argmax_vec(const uint4& raw, int base, float& best, int& besti, uint4& braw) {
  const uint32_t m = pmax_nan<T>(pmax_nan<T>(raw.x, raw.y), pmax_nan<T>(raw.z, raw.w));
  const float vm = fmax_nan(half_lo<T>(m), half_hi<T>(m));
  if (beats_later(vm, best)) {
    besti = base;
    best = vm;
    braw = raw;
  }
}

// Vector start -> index of the first element equal to best.
template <typename T>
LK_DEVINL void resolve_index(const uint4& braw, float best, int& besti) {
  if (besti == 0x7fffffff) return;
  besti += first_index_of<T>(braw, best);
}

template <typename T, int kU, int kMinBlocks, bool kCluster>
__global__ void __launch_bounds__(kSampThreads, kMinBlocks) argmax_kernel(const SampleParams p) {
  lk::pdl_wait();  // launched to overlap the kernel ahead of it: wait for it before reading
  // a kernel launched after this one may place its CTAs in the SM slots this grid
  // leaves free (it still waits for this grid to complete before reading)
  lk::pdl_launch_dependents();
  const int ch = blockIdx.x, b = blockIdx.y;
  const int v0 = ch * p.chunk, v1 = min(p.V, v0 + p.chunk);
  const T* row = static_cast<const T*>(p.logits) + static_cast<int64_t>(b) * p.ld;
  float best = -INFINITY;
  int besti = 0x7fffffff;
  uint4 braw = make_uint4(0u, 0u, 0u, 0u);
  const int vend = v0 + ((v1 - v0) / kVec) * kVec;
  constexpr int kStride = kSampThreads * kVec;
  int v = v0 + threadIdx.x * kVec;
  for (; v + (kU - 1) * kStride < vend; v += kU * kStride) {
    uint4 raw[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) raw[u] = __ldcs(reinterpret_cast<const uint4*>(row + v + u * kStride));
#pragma unroll
    for (int u = 0; u < kU; ++u) argmax_vec<T>(raw[u], v + u * kStride, best, besti, braw);
  }
  if (v < vend) {
    // fewer than kU vectors left for this thread: one predicated batch, all
    // loads in flight together (a one-load-per-iteration loop here costs a
    // memory round trip per vector)
    uint4 raw[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u)
      if (v + u * kStride < vend)
        raw[u] = __ldcs(reinterpret_cast<const uint4*>(row + v + u * kStride));
#pragma unroll
    for (int u = 0; u < kU; ++u)
      if (v + u * kStride < vend) argmax_vec<T>(raw[u], v + u * kStride, best, besti, braw);
  }
  resolve_index<T>(braw, best, besti);
  for (int t = vend + threadIdx.x; t < v1; t += kSampThreads) {
    const float x = lk::Elem<T>::to_f(row[t]);
    if (beats_later(x, best)) {
      best = x;
      besti = t;
    }
  }
  block_reduce(best, besti);
  if constexpr (kCluster) {
    // The row's chunks form one thread-block cluster: every CTA publishes
    // its winner in its own shared memory and rank 0 reads them all through
    // distributed shared memory. The second cluster barrier keeps each CTA's
    // shared memory alive until rank 0 has read it.
    __shared__ float c_key;
    __shared__ int c_idx;
    cg::cluster_group cluster = cg::this_cluster();
    if (threadIdx.x == 0) {
      c_key = best;
      c_idx = besti;
    }
    cluster.sync();
    if (cluster.block_rank() == 0 && threadIdx.x < 32) {
      float k = -INFINITY;
      int i = 0x7fffffff;
      for (int r = threadIdx.x; r < static_cast<int>(cluster.num_blocks()); r += 32) {
        const float k2 = *cluster.map_shared_rank(&c_key, r);
        const int i2 = *cluster.map_shared_rank(&c_idx, r);
        if (beats(k2, i2, k, i)) {
          k = k2;
          i = i2;
        }
      }
      reduce_pair(k, i);
      if (threadIdx.x == 0) p.out[b] = i == 0x7fffffff ? 0 : i;
    }
    cluster.sync();
    return;
  }
  if (p.nchunks == 1) {
    if (threadIdx.x == 0) p.out[b] = besti == 0x7fffffff ? 0 : besti;
    return;
  }
  __shared__ int s_last;
  if (threadIdx.x == 0) {
    p.part_key[static_cast<int64_t>(b) * p.nchunks + ch] = best;
    p.part_idx[static_cast<int64_t>(b) * p.nchunks + ch] = besti;
    __threadfence();
    s_last = atomicAdd(p.counters + b, 1) == p.nchunks - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  float k = -INFINITY;
  int i = 0x7fffffff;
  for (int c = threadIdx.x; c < p.nchunks; c += kSampThreads) {
    const float k2 = __ldcg(p.part_key + static_cast<int64_t>(b) * p.nchunks + c);
    const int i2 = __ldcg(p.part_idx + static_cast<int64_t>(b) * p.nchunks + c);
    if (beats(k2, i2, k, i)) {
      k = k2;
      i = i2;
    }
  }
  block_reduce(k, i);
  if (threadIdx.x == 0) {
    p.out[b] = i == 0x7fffffff ? 0 : i;
    p.counters[b] = 0;
  }
}


// Greedy rows streamed through shared memory: thread 0 keeps a ring of kNS
// 16 KiB tiles filled with 1-D bulk async copies (the copy engine holds up to
// kNS * 16 KiB in flight per CTA without tying up registers); all threads
// reduce each tile from shared memory.
constexpr int kTileVec = 1024;  // 16-byte vectors per tile (16 KiB)
constexpr int kNS = 4;
constexpr int kBulkSmem = kNS * kTileVec * 16;

template <typename T>
__global__ void __launch_bounds__(kSampThreads) argmax_bulk_kernel(const SampleParams p) {
  extern __shared__ __align__(128) uint4 ring[];
  __shared__ __align__(8) uint64_t full[kNS];
  const int ch = blockIdx.x, b = blockIdx.y;
  const int v0 = ch * p.chunk, v1 = min(p.V, v0 + p.chunk);
  const T* row = static_cast<const T*>(p.logits) + static_cast<int64_t>(b) * p.ld;
  const int vend = v0 + ((v1 - v0) / kVec) * kVec;
  const int nvec = (vend - v0) / kVec;
  const int tiles = (nvec + kTileVec - 1) / kTileVec;
  auto issue = [&](int t, int s) {
    const int nv = min(kTileVec, nvec - t * kTileVec);
    const uint32_t bytes = static_cast<uint32_t>(nv) * 16u;
    lk::mbar_arrive_expect_tx(&full[s], bytes);
    lk::bulk_load(ring + s * kTileVec, row + v0 + static_cast<int64_t>(t) * kTileVec * kVec, bytes,
                  &full[s]);
  };
  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < kNS; ++s) lk::mbar_init(&full[s], 1);
    lk::fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0)
    for (int t = 0; t < kNS && t < tiles; ++t) issue(t, t);
  float best = -INFINITY;
  int besti = 0x7fffffff;
  uint4 braw = make_uint4(0u, 0u, 0u, 0u);
  for (int t = 0; t < tiles; ++t) {
    const int s = t % kNS;
    if (!lk::mbar_wait(&full[s], (t / kNS) & 1)) break;  // bounded; never expected
    const int nv = min(kTileVec, nvec - t * kTileVec);
    const uint4* tile = ring + s * kTileVec;
    const int vbase = v0 + t * kTileVec * kVec;
#pragma unroll 4
    for (int i = threadIdx.x; i < nv; i += kSampThreads)
      argmax_vec<T>(tile[i], vbase + i * kVec, best, besti, braw);
    __syncthreads();
    if (threadIdx.x == 0 && t + kNS < tiles) {
      lk::fence_proxy_async();
      issue(t + kNS, s);
    }
  }
  resolve_index<T>(braw, best, besti);
  for (int t = vend + threadIdx.x; t < v1; t += kSampThreads) {
    const float x = lk::Elem<T>::to_f(row[t]);
    if (beats_later(x, best)) {
      best = x;
      besti = t;
    }
  }
  block_reduce(best, besti);
  if (p.nchunks == 1) {
    if (threadIdx.x == 0) p.out[b] = besti == 0x7fffffff ? 0 : besti;
    return;
  }
  __shared__ int s_last;
  if (threadIdx.x == 0) {
    p.part_key[static_cast<int64_t>(b) * p.nchunks + ch] = best;
    p.part_idx[static_cast<int64_t>(b) * p.nchunks + ch] = besti;
    __threadfence();
    s_last = atomicAdd(p.counters + b, 1) == p.nchunks - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  float k = -INFINITY;
  int i = 0x7fffffff;
  for (int c = threadIdx.x; c < p.nchunks; c += kSampThreads) {
    const float k2 = __ldcg(p.part_key + static_cast<int64_t>(b) * p.nchunks + c);
    const int i2 = __ldcg(p.part_idx + static_cast<int64_t>(b) * p.nchunks + c);
    if (beats(k2, i2, k, i)) {
      k = k2;
      i = i2;
    }
  }
  block_reduce(k, i);
  if (threadIdx.x == 0) {
    p.out[b] = i == 0x7fffffff ? 0 : i;
    p.counters[b] = 0;
  }
}

// One row segment [j0, j1) of 16-byte vectors (plus, with tail, the row's
// V % 8 ragged elements) of an in-kernel-noise row.
//
// Without a noise dump, most vectors need no keys: each key fl(fl(x / T) + g)
// is at most fl(fl(x_max / T) + h(u_max) + margin), where h(u) = -ln(1 - u)
// >= g(u) = -ln(-ln u) (as -ln u >= 1 - u; one logarithm instead of the
// map's two and its polynomial, and within 0.05 of g for the u_max near 0.9
// that the largest of 8 uniforms usually is), and x_max / T is taken as
// x_max RN(1/T) widened by 2^-22, which is at least the IEEE quotient. That,
// h and rounding are monotone, and the errors of g and h are far below the
// margin, so a vector whose bound is below a key already reached in this CTA
// cannot hold the row's winner (nor tie it) and is skipped after its Philox
// words. x_max is taken with packed 16-bit max instructions; a vector is
// widened to fp32 only when its keys are computed. A NaN logit makes the
// bound NaN: its vector is always computed (a NaN key wins). With a noise
// dump every key is computed.
template <typename T>
LK_DEVINL void gumbel_segment(const SampleParams& p, int b, int j0, int j1, bool tail, float temp,
                              float& best, int& besti) {
  const T* row = static_cast<const T*>(p.logits) + static_cast<int64_t>(b) * p.ld;
  const int nv = p.nv;
  float* drow = p.noise_dump ? p.noise_dump + static_cast<int64_t>(b) * p.V : nullptr;
  const FastDiv dv = FastDiv::make(temp);
  const uint4* rowv = reinterpret_cast<const uint4*>(row);
  // The CTA's best key so far, as an order-preserving int (a NaN key maps
  // above every number).
  __shared__ int s_best;
  if (threadIdx.x == 0) s_best = float_to_ordered(-INFINITY);
  __syncthreads();

  // the largest noise the map gives (every bit set), plus the margin
  const float g_cap = lk::gumbel_from_bits(0xffffffffu) + kGumbelBoundMargin;

  // a vector's 8 keys: the best of them against the thread's best
  auto keys = [&](int vv, const float (&f)[8], const U4 (&r)[2]) {
    float k[8];
    gumbel_keys(dv, vv, f, r, k, drow);
    const float m = fmax_nan(fmax_nan(fmax_nan(k[0], k[1]), fmax_nan(k[2], k[3])),
                             fmax_nan(fmax_nan(k[4], k[5]), fmax_nan(k[6], k[7])));
    const bool want_nan = m != m;
    int e = 7;
#pragma unroll
    for (int qq = 7; qq >= 0; --qq) e = (want_nan ? k[qq] != k[qq] : k[qq] == m) ? qq : e;
    if (beats(m, vv + e, best, besti)) {
      best = m;
      besti = vv + e;
      if (!drow) atomicMax(&s_best, float_to_ordered(m));
    }
  };
  auto philox = [&](int vv, int h) {
    return lk::philox4x32_10(
        U4{static_cast<uint32_t>((vv >> 2) + h), static_cast<uint32_t>(b), p.off_lo, p.off_hi},
        p.key);
  };

  if (drow) {  // every key, with the noise written out
    for (int j = j0 + threadIdx.x; j < j1; j += kSampThreads) {
      float f[8];
      Load16<T>::cvt(__ldcs(rowv + j), f);
      const U4 r[2] = {philox(j * kVec, 0), philox(j * kVec, 1)};
      keys(j * kVec, f, r);
    }
  } else {
    // Each vector's load is issued one step ahead, so the check that reads
    // it (before the Philox blocks) does not wait on memory. Measured from a
    // CUDA graph at 128 / 256 rows: 34.7 / 59.1 us loading in the step, 32.7 /
    // 51.6 us one step ahead; two steps ahead 33.6 / 53.0; two vectors a step
    // (4 Philox blocks in flight) 34.6 / 54.3 (registers spill at 4 CTAs/SM).
    // The one-logarithm bound and the packed x_max then took 33.7 -> 32.0 us
    // at 128 rows (same box, identical ids).
    const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
    uint4 nxt = j0 + static_cast<int>(threadIdx.x) < j1 ? __ldcs(rowv + j0 + threadIdx.x) : zero;
    for (int j = j0 + threadIdx.x; j < j1; j += kSampThreads) {
      const uint4 raw = nxt;
      nxt = j + kSampThreads < j1 ? __ldcs(rowv + j + kSampThreads) : zero;
      const uint32_t pm = pmax_nan<T>(pmax_nan<T>(raw.x, raw.y), pmax_nan<T>(raw.z, raw.w));
      const float xm = fmax_nan(half_lo<T>(pm), half_hi<T>(pm));
      // an upper bound of fl(x_max / T) is all the bound needs: x_max RN(1/T)
      // is within 2^-23 of the quotient, so widening it by 2^-22 covers that
      const float q0 = xm * dv.y;
      const float qm = fmaf(fabsf(q0), 2.384185791015625e-07f, q0);
      const float thr = fmaxf(best, ordered_to_float(*static_cast<volatile int*>(&s_best)));
      // logits alone: even the largest noise cannot lift this vector to the
      // best key, so its Philox blocks are not needed either
      if (__fadd_rn(qm, g_cap) < thr) continue;
      const U4 r[2] = {philox(j * kVec, 0), philox(j * kVec, 1)};
      const uint32_t rm = max(max(max(r[0].x, r[0].y), max(r[0].z, r[0].w)),
                              max(max(r[1].x, r[1].y), max(r[1].z, r[1].w)));
      {  // g(u) <= -ln(1 - u) (since -ln u >= 1 - u): one logarithm
        const float one_k = __uint_as_float(0x3f800000u | (rm >> 9));
        const float t = __fsub_rn(1.f, __fsub_rn(one_k, 0.99999994039535522f));
        const float gb = -0.693147180559945309f * lk::lg2_approx(t);
        if (__fadd_rn(qm, gb + kGumbelBoundMargin) < thr) continue;
      }
      float f[8];
      Load16<T>::cvt(raw, f);
      keys(j * kVec, f, r);
    }
  }
  if (tail) {  // the row's ragged tail (indices above every vector's)
    for (int t = nv * kVec + threadIdx.x; t < p.V; t += kSampThreads) {
      const U4 r = lk::philox4x32_10(
          U4{static_cast<uint32_t>(t >> 2), static_cast<uint32_t>(b), p.off_lo, p.off_hi}, p.key);
      const uint32_t w = (t & 3) == 0 ? r.x : (t & 3) == 1 ? r.y : (t & 3) == 2 ? r.z : r.w;
      const float g = lk::gumbel_from_bits(w);
      if (drow) drow[t] = g;
      const float key = __fadd_rn(__fdiv_rn(lk::Elem<T>::to_f(row[t]), temp), g);
      if (beats(key, t, best, besti)) {
        best = key;
        besti = t;
      }
    }
  }
}

// Grid (chunk, row): each CTA takes one of the row's equal chunks of vectors
// (the last chunk also the ragged tail); gumbel_chunks sets how many. Long
// chunks let the CTA's running best skip more vectors, so large batches take
// 4 chunks a row (under one wave); small ones take more to reach the SMs.
// Measured slower: a static cut of the batch into one equal range per
// resident slot, crossing row boundaries (the SMs' speeds differ on this
// compute-bound loop), and a persistent grid pulling items from a counter.
template <typename T>
__global__ void __launch_bounds__(kSampThreads, kGumbelCtasPerSm) gumbel_kernel(const SampleParams p) {
  lk::pdl_wait();  // launched to overlap the kernel ahead of it: wait for it before reading
  // a kernel launched after this one may place its CTAs in the SM slots this grid
  // leaves free (it still waits for this grid to complete before reading)
  lk::pdl_launch_dependents();
  const int ch = blockIdx.x, b = blockIdx.y;
  const float temp = p.temps[b];
  const int cv = p.chunk / kVec;  // vectors per chunk
  const int j0 = ch * cv, j1 = min(p.nv, j0 + cv);
  const bool tail = ch == p.nchunks - 1;
  float best = -INFINITY;
  int besti = 0x7fffffff;
  if (temp > 0.f) {
    gumbel_segment<T>(p, b, j0, j1, tail, temp, best, besti);
  } else {  // a greedy row inside a sampled batch
    scan_chunk<T, true, 0>(p, b, j0 * kVec, tail ? p.V : j1 * kVec, temp, best, besti);
  }
  finish_row(p, b, ch, best, besti);
}

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// Workspace layout: [counters: 65536 int32 — a fixed region, so that calls
// with different B find it where the previous call left it zeroed]
// [part_key: B*chunks f32][part_idx: B*chunks int32]
constexpr size_t kCounterBytes = 65536 * 4;

// Loads in flight per thread of the greedy kernel and the CTAs per SM that
// its registers allow: 4 -> 6, 8 -> 4, 16 -> 2. LITEKERN_SAMPLE_UNROLL (read
// once) selects one; the grid is sized for one full wave of it.
int sample_unroll() {
  static int u = [] {
    const char* e = getenv("LITEKERN_SAMPLE_UNROLL");
    const int v = e ? atoi(e) : 8;
    return (v == 0 || v == 4 || v == 8 || v == 16) ? v : 8;
  }();
  return u;
}
int ctas_per_sm() {
  switch (sample_unroll()) {
    case 4: return 6;
    case 8: return 4;
    case 16: return 2;
    default: return 3;  // bulk kernel: 64 KiB ring per CTA
  }
}

// LITEKERN_SAMPLE_CLUSTER=0 (read once): all-greedy rows merge their chunks
// through the workspace (last CTA of the row) instead of a cluster.
bool sample_cluster() {
  static bool c = [] {
    const char* e = getenv("LITEKERN_SAMPLE_CLUSTER");
    return !(e && atoi(e) == 0);
  }();
  return c;
}

int chunk_override() {
  static int c = [] {
    const char* e = getenv("LITEKERN_SAMPLE_CHUNKS");
    return e ? atoi(e) : 0;
  }();
  return c;
}

int choose_chunks(int B, int V) {
  if (chunk_override() > 0) return chunk_override();
  // One full wave: kSampCtasPerSm CTAs per SM over the whole batch (rounded
  // down so the grid never spills into a second wave), chunks of at least
  // 2048 elements.
  const int64_t target = static_cast<int64_t>(ctas_per_sm()) * lk::num_sms();
  int64_t n = target / B;
  const int64_t maxn = (V + 2047) / 2048;
  if (n > maxn) n = maxn;
  if (n < 1) n = 1;
  if (n > 1024) n = 1024;
  return static_cast<int>(n);
}

// LITEKERN_GUMBEL_GENERIC=1 (read once) sends in-kernel-noise rows to the
// general sample_kernel instead of gumbel_kernel (the earlier path).
bool gumbel_generic() {
  static bool g = [] {
    const char* e = getenv("LITEKERN_GUMBEL_GENERIC");
    return e && atoi(e) != 0;
  }();
  return g;
}


constexpr int kMaxCluster = 8;  // portable cluster size

template <typename K>
cudaError_t launch_cluster(K kernel, const cudaLaunchConfig_t& cfg, const SampleParams& p) {
  return cudaLaunchKernelEx(&cfg, kernel, p);
}

template <typename T>
int launch_sample(const SampleParams& p, int B, bool vec, cudaStream_t s) {
  dim3 grid(p.nchunks, B);
  if constexpr (!std::is_same<T, float>::value) {
    if (vec && p.temps == nullptr && sample_unroll() != 0) {
      if (p.nchunks > 1 && p.nchunks <= kMaxCluster && sample_cluster()) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = grid;
        cfg.blockDim = dim3(kSampThreads);
        cfg.dynamicSmemBytes = 0;
        cfg.stream = s;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = p.nchunks;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        // may start while the kernel ahead of it runs; waits for it first thing
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = lk::pdl_enabled() ? 2 : 1;
        cudaError_t e;
        switch (sample_unroll()) {
          case 4: e = launch_cluster(argmax_kernel<T, 4, 6, true>, cfg, p); break;
          case 16: e = launch_cluster(argmax_kernel<T, 16, 2, true>, cfg, p); break;
          default: e = launch_cluster(argmax_kernel<T, 8, 4, true>, cfg, p); break;
        }
        return e == cudaSuccess ? LK_OK : LK_ERR_CUDA;
      }
      cudaError_t e;
      switch (sample_unroll()) {
        case 4:
          e = lk::launch_after_previous(argmax_kernel<T, 4, 6, false>, grid, dim3(kSampThreads), 0,
                                        s, p);
          break;
        case 16:
          e = lk::launch_after_previous(argmax_kernel<T, 16, 2, false>, grid, dim3(kSampThreads),
                                        0, s, p);
          break;
        default:
          e = lk::launch_after_previous(argmax_kernel<T, 8, 4, false>, grid, dim3(kSampThreads), 0,
                                        s, p);
          break;
      }
      return e == cudaSuccess ? LK_OK : LK_ERR_CUDA;
    }
  }
  if constexpr (!std::is_same<T, float>::value) {
    if (vec && p.temps == nullptr) {
      static int configured[64] = {0};
      int dev = 0;
      cudaGetDevice(&dev);
      if (dev >= 0 && dev < 64 && !configured[dev]) {
        if (cudaFuncSetAttribute(argmax_bulk_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kBulkSmem) != cudaSuccess)
          return LK_ERR_CUDA;
        configured[dev] = 1;
      }
      argmax_bulk_kernel<T><<<grid, kSampThreads, kBulkSmem, s>>>(p);
      return lk::check_launch();
    }
  }
  if constexpr (!std::is_same<T, float>::value) {
    if (p.gumbel) {
      const cudaError_t e =
          lk::launch_after_previous(gumbel_kernel<T>, grid, dim3(kSampThreads), 0, s, p);
      return e == cudaSuccess ? LK_OK : LK_ERR_CUDA;
    }
  }
  const cudaError_t e =
      vec ? lk::launch_after_previous(sample_kernel<T, true>, grid, dim3(kSampThreads), 0, s, p)
          : lk::launch_after_previous(sample_kernel<T, false>, grid, dim3(kSampThreads), 0, s, p);
  return e == cudaSuccess ? LK_OK : LK_ERR_CUDA;
}

// gumbel_kernel's chunks per row; the row's vectors are split evenly over
// them. Long chunks let a CTA's running best skip more vectors; small batches
// still need enough CTAs to reach the SMs. The rule: at least 4 chunks a row
// and about 256 CTAs in all, no chunk under one vector per thread. Measured
// from a CUDA graph at V = 151936, T = 0.7, best count per batch (us): B = 1
// 74 chunks (5.5), 16 16 (9.7), 32 8 (13.0), 64 4 (20.9; 9 chunks 20.0),
// 128 4 (33.1; 6 chunks 32.8), 256 4 (52.3); 2 chunks or 16+ chunks at
// B >= 128 were 3-40 % slower. LITEKERN_GUMBEL_CHUNKS (read once) fixes it.
int gumbel_chunks_env() {
  static int v = [] {
    const char* e = getenv("LITEKERN_GUMBEL_CHUNKS");
    const int x = e ? atoi(e) : 0;
    return x >= 1 && x <= 4096 ? x : 0;
  }();
  return v;
}
bool use_gumbel(int V, bool vec, bool rng) { return rng && vec && V >= kVec && !gumbel_generic(); }
int gumbel_chunks(int B, int V) {
  const int64_t nvr = V / kVec;
  int64_t n = gumbel_chunks_env();
  if (n == 0) {
    n = std::max<int64_t>(4, (256 + B - 1) / B);
    n = std::min<int64_t>(n, std::max<int64_t>(1, nvr / kSampThreads));
  }
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(n, nvr)));
}

// Chunks (CTAs) per row for one call: all-greedy 16-bit rows reduce their
// chunks inside one cluster (at most kMaxCluster); in-kernel-noise 16-bit
// rows take gumbel_kernel's chunks; everything else one wave.
int chunks_for(int B, int V, bool vec, bool greedy_only, bool rng) {
  if (greedy_only && vec && sample_unroll() != 0) {
    if (chunk_override() > 0) return chunk_override();
    // Few, long chunks: just enough CTAs to give every SM one (ceil(SMs / B)
    // per row). Each thread then keeps several batches of loads in flight
    // over its chunk; measured from a CUDA graph at 256 x 128256, 1 chunk per
    // row ran 12.7 us, 2 (a cluster pair) 13.7 us, 8 chunks 22.6 us (the
    // per-CTA ramp and merge dominate short chunks); at 64 rows 3 chunks 7.4
    // us, 1 chunk 9.3 us.
    const int64_t maxn = std::max<int64_t>(1, (V + 2047) / 2048);
    int64_t n = (lk::num_sms() + B - 1) / B;
    n = std::min<int64_t>(n, maxn);
    if (sample_cluster()) n = std::min<int64_t>(n, kMaxCluster);
    return static_cast<int>(std::max<int64_t>(1, n));
  }
  if (use_gumbel(V, vec, rng)) return gumbel_chunks(B, V);
  return choose_chunks(B, V);
}

// Validates the arguments and fills everything but the scratch pointers;
// returns LK_OK or an error code. Shared by lk_sample and lk_sample_noalloc.
int prepare(SampleParams& p, bool& vec, int64_t* out_ids, const void* logits, int32_t B,
            int32_t V, int64_t ld, const float* temperatures, const float* noise,
            int64_t noise_ld, uint64_t seed, uint64_t offset, float* noise_dump, int32_t dtype,
            int64_t max_partials = INT64_MAX) {
  if (B < 0 || V <= 0 || ld < V) return LK_ERR_INVALID_ARG;
  if (B == 0) return LK_OK;
  if (!out_ids || !logits || B > 65535) return LK_ERR_INVALID_ARG;
  if (noise && noise_ld < V) return LK_ERR_INVALID_ARG;
  if (dtype != LK_DTYPE_F32 && dtype != LK_DTYPE_F16 && dtype != LK_DTYPE_BF16)
    return LK_ERR_UNSUPPORTED;
  const int esz = lk::dtype_size(dtype);
  vec = dtype != LK_DTYPE_F32 &&
        (reinterpret_cast<uintptr_t>(logits) & 15u) == 0 && ((ld * esz) & 15) == 0 &&
        (!noise || (((reinterpret_cast<uintptr_t>(noise) & 15u) == 0) &&
                    ((noise_ld * 4) & 15) == 0)) &&
        (!noise_dump || ((reinterpret_cast<uintptr_t>(noise_dump) & 15u) == 0 &&
                         ((static_cast<int64_t>(V) * 4) & 15) == 0));
  p.logits = logits;
  p.ld = ld;
  p.V = V;
  p.nchunks = chunks_for(B, V, vec, temperatures == nullptr,
                         temperatures != nullptr && noise == nullptr);
  if (use_gumbel(V, vec, temperatures != nullptr && noise == nullptr)) {
    // whole vectors per chunk; the ragged tail joins the last chunk
    const int64_t nvr = V / kVec;
    const int64_t nmax = std::max<int64_t>(1, max_partials / B);
    const int64_t n = std::min<int64_t>(gumbel_chunks(B, V), nmax);
    const int64_t cv = (nvr + n - 1) / n;  // even split; the last chunk may be shorter
    p.chunk = static_cast<int>(cv * kVec);
    p.nchunks = static_cast<int>((nvr + cv - 1) / cv);
    p.gumbel = 1;
  } else {
    const int64_t per = (static_cast<int64_t>(V) + p.nchunks - 1) / p.nchunks;
    p.chunk = static_cast<int>(((per + kVec - 1) / kVec) * kVec);
    p.nchunks = static_cast<int>((V + static_cast<int64_t>(p.chunk) - 1) / p.chunk);
    p.gumbel = 0;
  }
  p.nv = V / kVec;
  p.temps = temperatures;
  p.noise = noise;
  p.noise_ld = noise_ld;
  p.key = lk::philox_key(seed);
  p.off_lo = static_cast<uint32_t>(offset);
  p.off_hi = static_cast<uint32_t>(offset >> 32);
  p.noise_dump = noise_dump;
  p.out = out_ids;
  p.counters = nullptr;
  p.part_key = nullptr;
  p.part_idx = nullptr;
  return LK_OK;
}

int launch(const SampleParams& p, int B, bool vec, int32_t dtype, cudaStream_t s) {
  switch (dtype) {
    case LK_DTYPE_BF16: return launch_sample<__nv_bfloat16>(p, B, vec, s);
    case LK_DTYPE_F16: return launch_sample<__half>(p, B, vec, s);
    default: return launch_sample<float>(p, B, false, s);
  }
}

// Largest chunk count any call shape (B, V) can take: the workspace covers it.
int max_chunks(int B, int V) { return std::max(choose_chunks(B, V), gumbel_chunks(B, V)); }

}  // namespace

extern "C" size_t lk_sample_workspace_bytes(int32_t B, int32_t V) {
  if (B <= 0 || V <= 0) return 0;
  return kCounterBytes + 2 * align256(static_cast<size_t>(B) * max_chunks(B, V) * 4);
}

extern "C" int lk_sample(int64_t* out_ids, const void* logits, int32_t B, int32_t V, int64_t ld,
                         const float* temperatures, const float* noise, int64_t noise_ld,
                         uint64_t seed, uint64_t offset, float* noise_dump, void* workspace,
                         size_t workspace_bytes, int32_t dtype, void* stream) {
  SampleParams p;
  bool vec = false;
  const int rc = prepare(p, vec, out_ids, logits, B, V, ld, temperatures, noise, noise_ld, seed,
                         offset, noise_dump, dtype);
  if (rc != LK_OK || B == 0) return rc;
  if (p.nchunks > 1) {
    const size_t need = lk_sample_workspace_bytes(B, V);
    if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255u))
      return LK_ERR_WORKSPACE;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const size_t kb = align256(static_cast<size_t>(B) * max_chunks(B, V) * 4);
    p.counters = reinterpret_cast<int32_t*>(ws);
    p.part_key = reinterpret_cast<float*>(ws + kCounterBytes);
    p.part_idx = reinterpret_cast<int32_t*>(ws + kCounterBytes + kb);
  }
  return launch(p, B, vec, dtype, static_cast<cudaStream_t>(stream));
}

// ------------------------------------------------------------ self-tests ---
namespace {

__global__ void selftest_div_kernel(float* out, const float* x, int n, const float* temps, int nt) {
  const int j = blockIdx.y;
  const FastDiv dv = FastDiv::make(temps[j]);
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    out[static_cast<int64_t>(j) * n + i] = dv.in_range(x[i]) ? dv.fast(x[i]) : __fdiv_rn(x[i], dv.t);
}

__global__ void selftest_gumbel_kernel(float* out, const uint32_t* bits, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    out[i] = lk::gumbel_from_bits(bits[i]);
}

}  // namespace

extern "C" int lk_selftest_sampler_div(float* out, const float* x, int32_t n, const float* temps,
                                       int32_t nt, void* stream) {
  if (!out || !x || !temps || n <= 0 || nt <= 0 || nt > 65535) return LK_ERR_INVALID_ARG;
  selftest_div_kernel<<<dim3(64, nt), 256, 0, static_cast<cudaStream_t>(stream)>>>(out, x, n,
                                                                                  temps, nt);
  return lk::check_launch();
}

extern "C" int lk_selftest_gumbel(float* out, const uint32_t* bits, int32_t n, void* stream) {
  if (!out || !bits || n <= 0) return LK_ERR_INVALID_ARG;
  selftest_gumbel_kernel<<<4 * lk::num_sms(), 256, 0, static_cast<cudaStream_t>(stream)>>>(out, bits,
                                                                                          n);
  return lk::check_launch();
}

extern "C" int lk_softmax_temp(float* probs, int64_t probs_ld, const void* logits, int32_t B,
                               int32_t V, int64_t ld, const float* temperatures, int32_t dtype,
                               void* stream) {
  if (B < 0 || V <= 0 || ld < V || probs_ld < V) return LK_ERR_INVALID_ARG;
  if (B == 0) return LK_OK;
  if (!probs || !logits) return LK_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case LK_DTYPE_BF16:
      softmax_temp_kernel<__nv_bfloat16><<<B, kSampThreads, 0, s>>>(
          probs, probs_ld, static_cast<const __nv_bfloat16*>(logits), V, ld, temperatures);
      break;
    case LK_DTYPE_F16:
      softmax_temp_kernel<__half><<<B, kSampThreads, 0, s>>>(
          probs, probs_ld, static_cast<const __half*>(logits), V, ld, temperatures);
      break;
    case LK_DTYPE_F32:
      softmax_temp_kernel<float><<<B, kSampThreads, 0, s>>>(
          probs, probs_ld, static_cast<const float*>(logits), V, ld, temperatures);
      break;
    default: return LK_ERR_UNSUPPORTED;
  }
  return lk::check_launch();
}

// ------------------------------------------------ allocation-free variant ---
// lk_sample_noalloc: the same kernel, with its cross-CTA scratch (per-row
// counters and per-chunk winners) in a file-scope __device__ array instead of
// a caller workspace, for callers that cannot allocate device memory.
namespace {

constexpr int kNoAllocMaxRows = 8192;
constexpr int kNoAllocMaxPartials = 16384;
constexpr size_t kNoAllocCounterBytes = kNoAllocMaxRows * 4;
constexpr size_t kNoAllocBytes = kNoAllocCounterBytes + 2 * kNoAllocMaxPartials * 4;  // 160 KiB

static __device__ __align__(256) unsigned char g_sample_scratch[kNoAllocBytes];

// Device address of g_sample_scratch per device, looked up once with that
// device current. In host code the symbol is only a host-side stand-in.
std::mutex g_scratch_mu;
void* g_scratch_ptr[64] = {nullptr};

int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return LK_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_sample_scratch) != cudaSuccess || p == nullptr)
      return LK_ERR_CUDA;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return LK_OK;
}

}  // namespace

extern "C" int lk_sample_noalloc(int64_t* out_ids, const void* logits, int32_t B, int32_t V,
                                 int64_t ld, const float* temperatures, const float* noise,
                                 int64_t noise_ld, uint64_t seed, uint64_t offset,
                                 float* noise_dump, int32_t dtype, void* stream) {
  SampleParams p;
  bool vec = false;
  const int rc0 = prepare(p, vec, out_ids, logits, B, V, ld, temperatures, noise, noise_ld, seed,
                          offset, noise_dump, dtype, kNoAllocMaxPartials);
  if (rc0 != LK_OK || B == 0) return rc0;
  if (B > kNoAllocMaxRows || static_cast<int64_t>(B) * p.nchunks > kNoAllocMaxPartials)
    return LK_ERR_TOO_LARGE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (p.nchunks > 1) {
    void* base = nullptr;
    const int rc = scratch_address(&base);
    if (rc != LK_OK) return rc;
    uint8_t* ws = static_cast<uint8_t*>(base);
    p.counters = reinterpret_cast<int32_t*>(ws);
    p.part_key = reinterpret_cast<float*>(ws + kNoAllocCounterBytes);
    p.part_idx = reinterpret_cast<int32_t*>(ws + kNoAllocCounterBytes + kNoAllocMaxPartials * 4);
    // The counters must start at zero; clear the rows this call uses.
    if (cudaMemsetAsync(p.counters, 0, static_cast<size_t>(B) * 4, s) != cudaSuccess)
      return LK_ERR_CUDA;
  }
  return launch(p, B, vec, dtype, s);
}
