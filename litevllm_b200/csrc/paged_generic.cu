// Generic paged attention on the CUDA cores: the shapes the tuned kernels do
// not take. Those kernels (paged_decode.cu, paged_prefill.cu) want 16-bit
// caches, head_dim 128, block sizes that are multiples of 16 and, for
// prefill, G in {1, 2, 4, 8}. A model that runs in fp32 (the reference's CPU
// configuration), a Llama with head_dim 64 (Llama-3.2-1B, TinyLlama), or a
// cache with 8-slot blocks calls the same entry points and lands here.
//
// One kernel serves decode and prefill: query token i of sequence b sits at
// absolute position prior_b + i, prior_b = context_lens[b] - q_len_b, and
// attends keys j <= prior_b + i (decode: q_len 1, so every key < context_len;
// the reference's Attention._decode_fast, litevllm/layers/attention.py:91-139;
// prefill: the causal chunk over prior paged context, Attention._prefill
// :141-151 at prior 0). Scores, softmax and the PV sum are fp32 whatever the
// storage type; GQA maps query head h to KV head h / G (attention.py:124).
//
// Layout: CTA = (KV head, tile of query tokens, sequence), 128 threads. The
// tile's G * QT query rows (QT = 32 / G tokens) sit in shared memory as fp32;
// 32-token K and V tiles are gathered through the block table into shared
// memory (coalesced along d, 16-byte loads when the caches are 16-byte
// aligned) and converted to fp32. Each warp owns up to 8
// rows: lane j scores key j of the tile against a row, a warp max / sum gives
// the online-softmax update, and lane l accumulates output elements
// l, l + 32, ... of the row (D / 32 per lane) in registers.
#include <algorithm>
#include <mutex>

#include "lk_common.cuh"
#include "lk_host.h"

namespace {

constexpr int kGThreads = 128;
constexpr int kGWarps = kGThreads / 32;
constexpr int kGRows = 32;                 // query rows (token x head) per CTA
constexpr int kGRowsPerWarp = kGRows / kGWarps;
constexpr int kGKeys = 32;                 // keys per shared-memory tile

struct GenericParams {
  void* out;
  int64_t out_stride;  // elements between query tokens of out
  const void* q;
  int64_t q_stride;    // elements between query tokens of q
  const void* k;
  const void* v;
  int64_t num_slots;   // slots in the cache (paged) or key rows (contiguous)
  int64_t num_blocks;
  const int32_t* block_tables;  // NULL: contiguous keys, slot = cu_seqlens_q[b] + j
  int64_t bt_stride;
  const int32_t* cu_seqlens_q;  // NULL: one query per sequence (decode), row b
  const int32_t* context_lens;  // NULL: prior 0 (context = the chunk)
  int32_t* status;
  int H, H_kv, G, bs;
  int max_keys;        // > 0: context_lens beyond it are flagged and clamped
  int qt;              // query tokens per CTA
  float scale_log2;
  // Split-KV (decode only): blockIdx.y is the split; split s covers keys
  // [s * split_keys, (s + 1) * split_keys) and writes its (max, sum) and
  // unnormalised output to part_ml / part_o for generic_merge_kernel.
  int nsplit;          // 1: no split, the kernel writes out itself
  int split_keys;
  float* part_ml;      // [B * H][nsplit][2]
  float* part_o;       // [B * H][nsplit][D]
};

template <typename T>
__device__ __forceinline__ float ld_f(const T* p) {
  return lk::Elem<T>::to_f(*p);
}

template <typename T>
__device__ __forceinline__ void st_f(T* p, float x);
template <>
__device__ __forceinline__ void st_f<float>(float* p, float x) { *p = x; }
template <>
__device__ __forceinline__ void st_f<__half>(__half* p, float x) { *p = __float2half_rn(x); }
template <>
__device__ __forceinline__ void st_f<__nv_bfloat16>(__nv_bfloat16* p, float x) {
  *p = __float2bfloat16_rn(x);
}

// 16 bytes of T at src (16-byte aligned) -> 16 / sizeof(T) floats.
template <typename T>
__device__ __forceinline__ void load16_f(const T* src, float* dst);
template <>
__device__ __forceinline__ void load16_f<float>(const float* src, float* dst) {
  const float4 v = *reinterpret_cast<const float4*>(src);
  dst[0] = v.x; dst[1] = v.y; dst[2] = v.z; dst[3] = v.w;
}
template <>
__device__ __forceinline__ void load16_f<__nv_bfloat16>(const __nv_bfloat16* src, float* dst) {
  const uint4 v = *reinterpret_cast<const uint4*>(src);
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
    dst[2 * i] = f.x;
    dst[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void load16_f<__half>(const __half* src, float* dst) {
  const uint4 v = *reinterpret_cast<const uint4*>(src);
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    dst[2 * i] = f.x;
    dst[2 * i + 1] = f.y;
  }
}

// VEC: the caches are 16-byte aligned, so every (slot, head, d multiple of
// 16 / sizeof(T)) address is too and the tiles move in 16-byte loads.
// RPW: query rows per warp (the CTA holds 4 * RPW rows).
template <typename T, int D, bool VEC, int RPW>
__global__ void __launch_bounds__(kGThreads) generic_attn_kernel(GenericParams p) {
  constexpr int DV = D / 32;                    // output elements per lane and row
  constexpr int ROWS = kGWarps * RPW;
  constexpr int VE = VEC ? 16 / sizeof(T) : 1;  // elements per load
  constexpr int NV = D / VE;                    // loads per key row
  constexpr int PER = kGKeys * NV / kGThreads;  // loads per thread per tile, K or V
  // With few loads per thread, the next tile is held in registers while the
  // current one is computed, so its global latency overlaps the math.
  constexpr bool PF = VEC && PER <= 4;
  extern __shared__ float gsm[];
  float* Qs = gsm;                          // [ROWS][D]
  float* Ks = Qs + ROWS * D;                // [kGKeys][D + 1] (padded: lane j reads row j)
  float* Vs = Ks + kGKeys * (D + 1);        // [kGKeys][D]
  int* slots = reinterpret_cast<int*>(Vs + kGKeys * D);  // [2][kGKeys], -1 = zeros

  const int kvh = blockIdx.x, b = blockIdx.z;
  const int tile = p.nsplit > 1 ? 0 : blockIdx.y, sp = p.nsplit > 1 ? blockIdx.y : 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.G;

  int q_start, q_len;
  if (p.cu_seqlens_q) {
    q_start = p.cu_seqlens_q[b];
    q_len = p.cu_seqlens_q[b + 1] - q_start;
  } else {
    q_start = b;
    q_len = 1;
  }
  const int i0 = tile * p.qt;
  if (i0 >= q_len) return;
  const int ntok = min(p.qt, q_len - i0);
  const int nrows = ntok * G;  // <= ROWS (the host picks RPW so)

  int ctx = p.context_lens ? p.context_lens[b] : q_len;
  if (p.max_keys > 0 && ctx > p.max_keys) {
    if (threadIdx.x == 0 && tile == 0 && kvh == 0 && p.status)
      atomicOr(p.status, LK_STATUS_CTX_OOB);
    ctx = p.max_keys;
  }
  int prior = ctx - q_len;
  if (prior < 0) {
    // A decode row with context 0 has no keys (its output is NaN, as the
    // reference's softmax over an all -inf row); a prefill chunk longer than
    // its context is malformed.
    if (p.cu_seqlens_q && threadIdx.x == 0 && tile == 0 && kvh == 0 && p.status)
      atomicOr(p.status, LK_STATUS_CTX_OOB);
    prior = p.cu_seqlens_q ? 0 : -1;
  }
  // keys [0, kv_end) feed this tile's rows; this CTA takes [kv_beg, kv_stop)
  const int kv_end = max(0, prior + i0 + ntok);
  // split bounds in 64 bits: near INT_MAX keys the last split's end would
  // overflow; a split that starts past kv_end is empty
  const int64_t beg64 = static_cast<int64_t>(sp) * p.split_keys;
  const int kv_beg = static_cast<int>(min(beg64, static_cast<int64_t>(kv_end)));
  const int kv_stop = p.nsplit > 1
                          ? static_cast<int>(min(static_cast<int64_t>(kv_end), beg64 + p.split_keys))
                          : kv_end;

  // Q rows of the tile: row r = (token i0 + r / G, head kvh * G + r % G).
  const T* q = static_cast<const T*>(p.q);
  for (int e = threadIdx.x; e < nrows * D; e += kGThreads) {
    const int r = e / D, d = e - r * D;
    const int tok = q_start + i0 + r / G, h = kvh * G + r % G;
    Qs[e] = ld_f(q + tok * p.q_stride + static_cast<int64_t>(h) * D + d);
  }

  const T* kc = static_cast<const T*>(p.k);
  const T* vc = static_cast<const T*>(p.v);
  const int64_t slot_stride = static_cast<int64_t>(p.H_kv) * D;
  const int32_t* bt = p.block_tables ? p.block_tables + b * p.bt_stride : nullptr;

  // Cache slot of key j (-1: past the keys, or an out-of-range block: zeros).
  auto slot_of = [&](int j) -> int {
    if (j >= kv_stop) return -1;
    if (bt) {
      const int blk = bt[j / p.bs];
      if (blk < 0 || blk >= p.num_blocks) {
        if (p.status) atomicOr(p.status, LK_STATUS_BLOCK_OOB);
        return -1;
      }
      return blk * p.bs + j % p.bs;
    }
    const int64_t s = static_cast<int64_t>(q_start) + j;
    if (s < p.num_slots) return static_cast<int>(s);
    if (p.status) atomicOr(p.status, LK_STATUS_BLOCK_OOB);
    return -1;
  };

  // slots of tile 0 in buffer 0; warp 0 keeps tile 1's in a register
  int pend = -1;
  if (warp == 0) {
    slots[lane] = slot_of(kv_beg + lane);
    pend = slot_of(kv_beg + kGKeys + lane);
  }
  __syncthreads();

  uint4 kreg[PF ? PER : 1], vreg[PF ? PER : 1];
  auto prefetch = [&](const int* sl) {
    if constexpr (PF) {
#pragma unroll
      for (int v = 0; v < PER; ++v) {
        const int e = threadIdx.x + v * kGThreads;
        const int jj = e / NV, d = (e - jj * NV) * VE;
        const int slot = sl[jj];
        if (slot >= 0) {
          const int64_t off = slot * slot_stride + static_cast<int64_t>(kvh) * D + d;
          kreg[v] = *reinterpret_cast<const uint4*>(kc + off);
          vreg[v] = *reinterpret_cast<const uint4*>(vc + off);
        } else {
          kreg[v] = make_uint4(0u, 0u, 0u, 0u);
          vreg[v] = make_uint4(0u, 0u, 0u, 0u);
        }
      }
    }
  };
  prefetch(slots);

  float m[RPW], l[RPW], o[RPW][DV];
#pragma unroll
  for (int k = 0; k < RPW; ++k) {
    m[k] = -INFINITY;
    l[k] = 0.f;
#pragma unroll
    for (int t = 0; t < DV; ++t) o[k][t] = 0.f;
  }

  for (int j0 = kv_beg, buf = 0; j0 < kv_stop; j0 += kGKeys, buf ^= 1) {
    int* cur = slots + buf * kGKeys;
    int* nxt = slots + (buf ^ 1) * kGKeys;
    // 1. tile j0 into shared memory as fp32
    if constexpr (PF) {
#pragma unroll
      for (int v = 0; v < PER; ++v) {
        const int e = threadIdx.x + v * kGThreads;
        const int jj = e / NV, d = (e - jj * NV) * VE;
        float kx[VE], vx[VE];
        load16_f<T>(reinterpret_cast<const T*>(&kreg[v]), kx);
        load16_f<T>(reinterpret_cast<const T*>(&vreg[v]), vx);
#pragma unroll
        for (int i = 0; i < VE; ++i) {
          Ks[jj * (D + 1) + d + i] = kx[i];
          Vs[jj * D + d + i] = vx[i];
        }
      }
    } else {
      for (int e = threadIdx.x; e < kGKeys * NV; e += kGThreads) {
        const int jj = e / NV, d = (e - jj * NV) * VE;
        const int slot = cur[jj];
        float kx[VE], vx[VE];
        if (slot >= 0) {
          const int64_t off = slot * slot_stride + static_cast<int64_t>(kvh) * D + d;
          if constexpr (VEC) {
            load16_f<T>(kc + off, kx);
            load16_f<T>(vc + off, vx);
          } else {
            kx[0] = ld_f(kc + off);
            vx[0] = ld_f(vc + off);
          }
        } else {
#pragma unroll
          for (int i = 0; i < VE; ++i) kx[i] = vx[i] = 0.f;
        }
#pragma unroll
        for (int i = 0; i < VE; ++i) {
          Ks[jj * (D + 1) + d + i] = kx[i];
          Vs[jj * D + d + i] = vx[i];
        }
      }
    }
    // 2. publish the next tile's slots; fetch the block-table entries of the
    //    one after it
    if (warp == 0) {
      nxt[lane] = pend;
      pend = slot_of(j0 + 2 * kGKeys + lane);
    }
    __syncthreads();
    // 3. the next tile's loads fly while this tile is computed
    if (j0 + kGKeys < kv_stop) prefetch(nxt);

    // 4. scores, online softmax and PV for this warp's rows
#pragma unroll
    for (int k = 0; k < RPW; ++k) {
      const int r = warp + k * kGWarps;
      if (r < nrows) {
        const int pos = prior + i0 + r / G;  // this row's last visible key
        const int j = j0 + lane;
        const float4* qr = reinterpret_cast<const float4*>(Qs + r * D);
        const float* kr = Ks + lane * (D + 1);
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll 8
        for (int d4 = 0; d4 < D / 4; ++d4) {
          const float4 qv = qr[d4];
          s0 = fmaf(qv.x, kr[4 * d4], s0);
          s1 = fmaf(qv.y, kr[4 * d4 + 1], s1);
          s2 = fmaf(qv.z, kr[4 * d4 + 2], s2);
          s3 = fmaf(qv.w, kr[4 * d4 + 3], s3);
        }
        float s = (s0 + s1) + (s2 + s3);
        const bool valid = j <= pos && j < kv_stop;
        s = valid ? s * p.scale_log2 : -INFINITY;
        float mt = s;
#pragma unroll
        for (int w = 16; w > 0; w >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, w));
        const float mn = fmaxf(m[k], mt);
        if (mn != -INFINITY) {  // the row has a visible key by now
          const float alpha = exp2f(m[k] - mn);
          const float pj = valid ? exp2f(s - mn) : 0.f;
          float ps = pj;
#pragma unroll
          for (int w = 16; w > 0; w >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, w);
          l[k] = l[k] * alpha + ps;
#pragma unroll
          for (int t = 0; t < DV; ++t) o[k][t] *= alpha;
#pragma unroll 4
          for (int jj = 0; jj < kGKeys; ++jj) {
            const float pb = __shfl_sync(0xffffffffu, pj, jj);
            const float* vr = Vs + jj * D + lane;
#pragma unroll
            for (int t = 0; t < DV; ++t) o[k][t] = fmaf(pb, vr[32 * t], o[k][t]);
          }
          m[k] = mn;
        }
      }
    }
    __syncthreads();  // Ks / Vs and this tile's slots are free again
  }

  if (p.nsplit > 1) {  // decode split: one query token, rows = heads
#pragma unroll
    for (int k = 0; k < RPW; ++k) {
      const int r = warp + k * kGWarps;
      if (r < nrows) {
        const int64_t idx = (static_cast<int64_t>(b) * p.H + kvh * G + r) * p.nsplit + sp;
        if (lane == 0) {
          p.part_ml[2 * idx] = m[k];
          p.part_ml[2 * idx + 1] = l[k];
        }
        float* po = p.part_o + idx * D;
#pragma unroll
        for (int t = 0; t < DV; ++t) po[lane + 32 * t] = o[k][t];
      }
    }
    return;
  }
  T* out = static_cast<T*>(p.out);
#pragma unroll
  for (int k = 0; k < RPW; ++k) {
    const int r = warp + k * kGWarps;
    if (r < nrows) {
      const int tok = q_start + i0 + r / G, h = kvh * G + r % G;
      const float inv = l[k] > 0.f ? 1.f / l[k] : __int_as_float(0x7fc00000);  // no key: NaN
      T* orow = out + tok * p.out_stride + static_cast<int64_t>(h) * D;
#pragma unroll
      for (int t = 0; t < DV; ++t) st_f<T>(orow + lane + 32 * t, o[k][t] * inv);
    }
  }
}

// Merge of the decode splits: one warp per (sequence, query head). Weights
// exp2(m_s - M) with M the largest split max; a row with no key is NaN.
template <typename T, int D>
__global__ void __launch_bounds__(128) generic_merge_kernel(GenericParams p, int rows) {
  constexpr int DV = D / 32;
  const int row = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int b = row / p.H, h = row - b * p.H;
  const float* ml = p.part_ml + static_cast<int64_t>(row) * p.nsplit * 2;
  const float* po = p.part_o + static_cast<int64_t>(row) * p.nsplit * D;
  float M = -INFINITY;
  for (int s = 0; s < p.nsplit; ++s) M = fmaxf(M, ml[2 * s]);
  float L = 0.f, o[DV];
#pragma unroll
  for (int t = 0; t < DV; ++t) o[t] = 0.f;
  if (M != -INFINITY) {
    for (int s = 0; s < p.nsplit; ++s) {
      const float w = exp2f(ml[2 * s] - M);  // 0 for an empty split
      L = fmaf(ml[2 * s + 1], w, L);
#pragma unroll
      for (int t = 0; t < DV; ++t) o[t] = fmaf(po[s * D + lane + 32 * t], w, o[t]);
    }
  }
  const float inv = L > 0.f ? 1.f / L : __int_as_float(0x7fc00000);  // no key: NaN
  T* orow = static_cast<T*>(p.out) + b * p.out_stride + static_cast<int64_t>(h) * D;
#pragma unroll
  for (int t = 0; t < DV; ++t) st_f<T>(orow + lane + 32 * t, o[t] * inv);
}

size_t generic_smem_bytes(int D, int rpw) {
  return (static_cast<size_t>(kGWarps) * rpw * D + static_cast<size_t>(kGKeys) * (D + 1) +
          static_cast<size_t>(kGKeys) * D) * sizeof(float) + 2 * kGKeys * sizeof(int);
}

template <typename T, int D, bool VEC, int RPW>
int launch_generic_r(const GenericParams& p, int num_seqs, int max_q_len, cudaStream_t s) {
  auto kern = generic_attn_kernel<T, D, VEC, RPW>;
  const size_t smem = generic_smem_bytes(D, RPW);
  // Shared memory above 48 KB is opted into once per device (and instantiation).
  static std::mutex mu;
  static bool done[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return LK_ERR_CUDA;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!done[dev]) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(smem)) != cudaSuccess)
        return LK_ERR_CUDA;
      done[dev] = true;
    }
  }
  dim3 grid(p.H_kv, p.nsplit > 1 ? p.nsplit : (max_q_len + p.qt - 1) / p.qt, num_seqs);
  kern<<<grid, kGThreads, smem, s>>>(p);
  if (p.nsplit > 1) {
    const int rows = num_seqs * p.H;
    generic_merge_kernel<T, D><<<(rows + 3) / 4, 128, 0, s>>>(p, rows);
  }
  return lk::check_launch();
}

template <typename T, int D, bool VEC>
int launch_generic_d(GenericParams p, int num_seqs, int max_q_len, cudaStream_t s) {
  // Rows per warp: the fewest that hold the tile's query rows (decode: the
  // G heads of one token; prefill: up to 32 rows, 32 / G tokens).
  const int want = std::min(max_q_len, std::max(1, kGRows / p.G)) * p.G;
  const int rpw = want <= kGWarps ? 1 : want <= 2 * kGWarps ? 2 : want <= 4 * kGWarps ? 4 : 8;
  p.qt = std::max(1, kGWarps * rpw / p.G);
  switch (rpw) {
    case 1: return launch_generic_r<T, D, VEC, 1>(p, num_seqs, max_q_len, s);
    case 2: return launch_generic_r<T, D, VEC, 2>(p, num_seqs, max_q_len, s);
    case 4: return launch_generic_r<T, D, VEC, 4>(p, num_seqs, max_q_len, s);
    default: return launch_generic_r<T, D, VEC, 8>(p, num_seqs, max_q_len, s);
  }
}

template <typename T, bool VEC>
int launch_generic_v(const GenericParams& p, int D, int num_seqs, int max_q_len, cudaStream_t s) {
  switch (D) {
    case 32: return launch_generic_d<T, 32, VEC>(p, num_seqs, max_q_len, s);
    case 64: return launch_generic_d<T, 64, VEC>(p, num_seqs, max_q_len, s);
    case 96: return launch_generic_d<T, 96, VEC>(p, num_seqs, max_q_len, s);
    case 128: return launch_generic_d<T, 128, VEC>(p, num_seqs, max_q_len, s);
    case 256: return launch_generic_d<T, 256, VEC>(p, num_seqs, max_q_len, s);
    default: return LK_ERR_UNSUPPORTED;
  }
}

template <typename T>
int launch_generic(const GenericParams& p, int D, int num_seqs, int max_q_len, cudaStream_t s) {
  const bool vec =
      ((reinterpret_cast<uintptr_t>(p.k) | reinterpret_cast<uintptr_t>(p.v)) & 15u) == 0;
  return vec ? launch_generic_v<T, true>(p, D, num_seqs, max_q_len, s)
             : launch_generic_v<T, false>(p, D, num_seqs, max_q_len, s);
}

}  // namespace

namespace {

// Splits of a decode whose contexts reach max_keys: about 512 keys (16
// tiles) per split CTA, at most 64.
int generic_decode_splits(int64_t max_keys) {
  return static_cast<int>(std::min<int64_t>(64, std::max<int64_t>(1, (max_keys + 511) / 512)));
}

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// Decode workspace with split partials: the decode head (status word and the
// split kernel's counters, left untouched here), then (max, sum) and output
// partials.
size_t generic_split_bytes(int64_t rows, int D, int ns) {
  return lk::kDecodeHeadBytes + align256(static_cast<size_t>(rows) * ns * 2 * 4) +
         align256(static_cast<size_t>(rows) * ns * D * 4);
}

int check_generic_args(int num_seqs, int max_q_len, int H, int H_kv, int D, int64_t num_blocks,
                       int max_blocks_per_seq, int dtype) {
  if (num_seqs < 0 || max_q_len < 0 || H <= 0 || H_kv <= 0 || H % H_kv != 0 || num_blocks <= 0 ||
      max_blocks_per_seq < 0)
    return LK_ERR_INVALID_ARG;
  if (dtype != LK_DTYPE_F32 && dtype != LK_DTYPE_F16 && dtype != LK_DTYPE_BF16)
    return LK_ERR_UNSUPPORTED;
  if (H / H_kv > kGRows || (D != 32 && D != 64 && D != 96 && D != 128 && D != 256))
    return LK_ERR_UNSUPPORTED;
  if (num_seqs > 65535 || H_kv > 65535) return LK_ERR_INVALID_ARG;
  return LK_OK;
}

GenericParams make_params(void* out, int64_t out_token_stride, const void* q,
                          int64_t q_token_stride, const void* k_cache, const void* v_cache,
                          int64_t num_blocks, int64_t num_slots, const int32_t* block_tables,
                          int64_t block_table_stride, const int32_t* cu_seqlens_q,
                          const int32_t* context_lens, int H, int H_kv, int block_size,
                          int64_t max_keys, float scale, int32_t* status) {
  GenericParams p;
  p.out = out;
  p.out_stride = out_token_stride;
  p.q = q;
  p.q_stride = q_token_stride;
  p.k = k_cache;
  p.v = v_cache;
  p.num_slots = num_slots;
  p.num_blocks = block_tables ? num_blocks : 0;
  p.block_tables = block_tables;
  p.bt_stride = block_table_stride;
  p.cu_seqlens_q = cu_seqlens_q;
  p.context_lens = block_tables ? context_lens : nullptr;  // contiguous mode: prior 0
  p.status = status;
  p.H = H;
  p.H_kv = H_kv;
  p.G = H / H_kv;
  p.bs = block_size;
  p.max_keys = static_cast<int>(max_keys);
  p.qt = kGRows / p.G;  // refined with the rows per warp at launch
  p.scale_log2 = scale * 1.4426950408889634f;
  p.nsplit = 1;
  p.split_keys = 0;
  p.part_ml = nullptr;
  p.part_o = nullptr;
  return p;
}

int run_generic(const GenericParams& p, int D, int dtype, int num_seqs, int max_q_len,
                void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case LK_DTYPE_BF16: return launch_generic<__nv_bfloat16>(p, D, num_seqs, max_q_len, s);
    case LK_DTYPE_F16: return launch_generic<__half>(p, D, num_seqs, max_q_len, s);
    default: return launch_generic<float>(p, D, num_seqs, max_q_len, s);
  }
}

bool aligned_to(const void* a, const void* b, const void* c, const void* d, int esz) {
  return ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
           reinterpret_cast<uintptr_t>(c) | reinterpret_cast<uintptr_t>(d)) &
          static_cast<uintptr_t>(esz - 1)) == 0;
}

}  // namespace

extern "C" size_t lk_paged_attention_generic_workspace_bytes(int32_t B, int32_t H, int32_t D,
                                                             int32_t max_blocks_per_seq,
                                                             int32_t block_size) {
  if (B <= 0 || H <= 0 || D <= 0 || max_blocks_per_seq <= 0 || block_size <= 0) return 256;
  const int ns = generic_decode_splits(static_cast<int64_t>(max_blocks_per_seq) * block_size);
  return ns > 1 ? generic_split_bytes(static_cast<int64_t>(B) * H, D, ns) : 256;
}

namespace lk {

int generic_decode(void* out, int64_t out_token_stride, const void* q, int64_t q_token_stride,
                   const void* k_cache, const void* v_cache, int64_t num_blocks,
                   const int32_t* block_tables, int64_t block_table_stride,
                   const int32_t* context_lens, int B, int H, int H_kv, int D, int block_size,
                   int max_blocks_per_seq, float scale, int dtype, void* workspace,
                   size_t workspace_bytes, void* stream) {
  int rc = check_generic_args(B, 1, H, H_kv, D, num_blocks, max_blocks_per_seq, dtype);
  if (rc != LK_OK) return rc;
  if (B == 0) return LK_OK;
  if (!out || !q || !k_cache || !v_cache || !block_tables || !context_lens || block_size <= 0 ||
      max_blocks_per_seq <= 0)
    return LK_ERR_INVALID_ARG;
  if (!workspace || workspace_bytes < 4 || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return LK_ERR_WORKSPACE;
  const int64_t num_slots = num_blocks * block_size;
  const int64_t max_keys = static_cast<int64_t>(max_blocks_per_seq) * block_size;
  if (num_slots > 0x7fffffffLL || max_keys > 0x7fffffffLL) return LK_ERR_UNSUPPORTED;
  if (!aligned_to(q, out, k_cache, v_cache, lk::dtype_size(dtype))) return LK_ERR_ALIGNMENT;
  GenericParams p = make_params(out, out_token_stride, q, q_token_stride, k_cache, v_cache,
                                num_blocks, num_slots, block_tables, block_table_stride, nullptr,
                                context_lens, H, H_kv, block_size, max_keys, scale,
                                static_cast<int32_t*>(workspace));
  // As many splits as the workspace holds, up to generic_decode_splits.
  const int64_t rows = static_cast<int64_t>(B) * H;
  int ns = generic_decode_splits(max_keys);
  while (ns > 1 && generic_split_bytes(rows, D, ns) > workspace_bytes) --ns;
  if (ns > 1) {
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    p.nsplit = ns;
    p.split_keys = static_cast<int>((((max_keys + ns - 1) / ns) + kGKeys - 1) / kGKeys * kGKeys);
    p.part_ml = reinterpret_cast<float*>(ws + lk::kDecodeHeadBytes);
    p.part_o = reinterpret_cast<float*>(ws + lk::kDecodeHeadBytes +
                                        align256(static_cast<size_t>(rows) * ns * 8));
  }
  return run_generic(p, D, dtype, B, 1, stream);
}

}  // namespace lk

extern "C" int lk_paged_attention_generic(
    void* out, int64_t out_token_stride, const void* q, int64_t q_token_stride,
    const void* k_cache, const void* v_cache, int64_t num_blocks, const int32_t* block_tables,
    int64_t block_table_stride, const int32_t* cu_seqlens_q, const int32_t* context_lens,
    int32_t num_seqs, int32_t max_q_len, int32_t H, int32_t H_kv, int32_t D, int32_t block_size,
    int32_t max_blocks_per_seq, float scale, int32_t dtype, int32_t* status, void* stream) {
  int rc = check_generic_args(num_seqs, max_q_len, H, H_kv, D, num_blocks, max_blocks_per_seq,
                              dtype);
  if (rc != LK_OK) return rc;
  if (num_seqs == 0 || max_q_len == 0) return LK_OK;
  if (!out || !q || !k_cache || !v_cache) return LK_ERR_INVALID_ARG;
  if (!cu_seqlens_q && max_q_len != 1) return LK_ERR_INVALID_ARG;
  if (!block_tables && !cu_seqlens_q) return LK_ERR_INVALID_ARG;
  int64_t num_slots;
  if (block_tables) {
    if (block_size <= 0) return LK_ERR_INVALID_ARG;
    num_slots = num_blocks * block_size;
  } else {
    num_slots = num_blocks;
  }
  if (num_slots > 0x7fffffffLL) return LK_ERR_UNSUPPORTED;
  const int64_t max_keys =
      block_tables && max_blocks_per_seq > 0 ? static_cast<int64_t>(max_blocks_per_seq) * block_size : 0;
  if (max_keys > 0x7fffffffLL) return LK_ERR_UNSUPPORTED;
  if (!aligned_to(q, out, k_cache, v_cache, lk::dtype_size(dtype))) return LK_ERR_ALIGNMENT;
  const GenericParams p = make_params(out, out_token_stride, q, q_token_stride, k_cache, v_cache,
                                      num_blocks, num_slots, block_tables, block_table_stride,
                                      cu_seqlens_q, context_lens, H, H_kv, block_size, max_keys,
                                      scale, status);
  return run_generic(p, D, dtype, num_seqs, max_q_len, stream);
}
