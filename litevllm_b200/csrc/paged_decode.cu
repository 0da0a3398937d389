// Paged decode attention (one query token per sequence) over the block-table
// KV cache. Restates Attention._decode_fast, litevllm/layers/attention.py:91-139:
//   out[b, h] = softmax_s(scale * q[b,h] . K[b,s,h/G]) V[b,s,h/G],  s < ctx[b]
// with the GQA mapping h -> h / G of attention.py:124.
//
// B200 design
//  * Work unit = (sequence, KV-head group of HPC heads, split of the context).
//    A CTA streams its split's 16-token stages of K and V with TMA
//    (cp.async.bulk.tensor, 3-D map (d, slot, head), 128-byte swizzle) into an
//    NST-deep shared-memory ring; one producer warp walks the block table and
//    issues the loads, HPC consumer warps (one per KV head) compute.
//  * The G query heads that share a KV head share every K/V tile: each
//    consumer warp computes S^T = K Q^T (16 tokens x 8 query columns) and
//    O^T += V^T P^T with mma.sync m16n8k16 (fp32 accumulate); P^T is moved
//    from accumulator layout to operand layout with movmatrix. Online softmax
//    (running max / sum) uses warp shuffles.
//  * Split-KV: each split writes (m, l, o) partials to the workspace; the last
//    CTA of a (sequence, head group) to finish (atomic counter, no waiting)
//    merges them with a log-sum-exp reduction and resets the counter.
#include "lk_common.cuh"
#include "lk_host.h"

namespace {

constexpr int kD = 128;          // head_dim
constexpr int kTok = 16;         // tokens per stage (mma M)

struct DecodeParams {
  void* out;
  int64_t out_stride;  // elements between tokens (rows) of out
  const void* q;
  int64_t q_stride;
  const int32_t* block_tables;
  int64_t bt_stride;
  const int32_t* context_lens;
  int64_t num_blocks;
  int H, G, bs, max_blocks;
  float scale_log2;       // scale * log2(e)
  int stages_per_split;
  int num_splits;
  int num_groups;         // H_kv / HPC
  int32_t* counters;      // [B * num_groups]
  int32_t* status;
  float* part_ml;         // [B][num_splits][H][2]  (m in log2 domain, l)
  float* part_o;          // [B][num_splits][H][D]
};

template <int HPC, int NST> struct DecodeShape {
  static constexpr int kBoxBytes = HPC * kTok * 128;  // HPC heads x 16 slots x 64 values
  static constexpr int kStageBytes = 4 * kBoxBytes;   // K lo/hi, V lo/hi
  static constexpr int kThreads = (HPC + 1) * 32;
  static constexpr int kSmem = NST * kStageBytes + 1024;
};

template <typename T>
LK_DEVINL void store_out(T* p, float v);
template <> LK_DEVINL void store_out<__nv_bfloat16>(__nv_bfloat16* p, float v) {
  *p = __float2bfloat16_rn(v);
}
template <> LK_DEVINL void store_out<__half>(__half* p, float v) { *p = __float2half_rn(v); }

template <typename T, int HPC, int NST>
__global__ void __launch_bounds__((HPC + 1) * 32, 1)
paged_decode_kernel(const __grid_constant__ CUtensorMap kmap,
                    const __grid_constant__ CUtensorMap vmap, const DecodeParams p) {
  using Shape = DecodeShape<HPC, NST>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[NST];
  __shared__ __align__(8) uint64_t empty_bar[NST];
  __shared__ int s_last;
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

  const int sp = blockIdx.x, hg = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.G;

  int ctx = p.context_lens[b];
  const int cap = p.max_blocks * p.bs;
  if (ctx > cap) {
    if (threadIdx.x == 0 && sp == 0) atomicOr(p.status, LK_STATUS_CTX_OOB);
    ctx = cap;
  }
  if (ctx < 0) ctx = 0;
  const int nst = (ctx + kTok - 1) / kTok;
  const int spp = p.stages_per_split;
  const int nsp = nst == 0 ? 1 : (nst + spp - 1) / spp;
  if (sp >= nsp) return;

  T* out = static_cast<T*>(p.out) + static_cast<int64_t>(b) * p.out_stride;
  if (nst == 0) {
    // softmax over an all -inf row is NaN in the reference; reproduce it.
    const int nq = HPC * G;
    for (int i = threadIdx.x; i < nq * kD; i += Shape::kThreads)
      store_out<T>(out + (hg * nq) * kD + i, __int_as_float(0x7fc00000));
    return;
  }
  const int st0 = sp * spp;
  const int st1 = min(nst, st0 + spp);

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < NST; ++s) {
      lk::mbar_init(&full_bar[s], 1);
      lk::mbar_init(&empty_bar[s], HPC);
    }
    lk::fence_barrier_init();
  }
  __syncthreads();

  if (warp == HPC) {
    // ------------------------------------------------------- producer ---
    if (lane == 0) {
      lk::prefetch_tensormap(&kmap);
      lk::prefetch_tensormap(&vmap);
    }
    const int32_t* bt = p.block_tables + static_cast<int64_t>(b) * p.bt_stride;
    const int64_t num_slots = p.num_blocks * p.bs;
    bool ok = true;
    int it = 0;
    for (int base = st0; base < st1 && ok; base += 32) {
      // Each lane resolves one stage's starting slot ahead of time so the
      // block-table reads overlap instead of serialising the TMA issue.
      int slot0 = 0;
      const int st = base + lane;
      if (st < st1) {
        const int pos = st * kTok;
        const int blk = __ldg(bt + pos / p.bs);
        if (blk < 0 || blk >= p.num_blocks) {
          atomicOr(p.status, LK_STATUS_BLOCK_OOB);
          slot0 = static_cast<int>(num_slots < 0x7fffffffLL ? num_slots : 0x7fffffffLL);  // past the end: TMA reads zeros
        } else {
          slot0 = blk * p.bs + (pos % p.bs);
        }
      }
      const int n = min(32, st1 - base);
      for (int i = 0; i < n; ++i, ++it) {
        const int slot = __shfl_sync(0xffffffffu, slot0, i);
        if (lane == 0) {
          const int s = it % NST;
          const uint32_t ph = ((it / NST) & 1) ^ 1;
          if (!lk::mbar_wait(&empty_bar[s], ph)) {
            atomicOr(p.status, LK_STATUS_WAIT_TIMEOUT);
            ok = false;
          } else {
            lk::mbar_arrive_expect_tx(&full_bar[s], Shape::kStageBytes);
            uint8_t* dst = smem + s * Shape::kStageBytes;
            const int h0 = hg * HPC;
            lk::tma_load_3d(dst, &kmap, &full_bar[s], 0, slot, h0);
            lk::tma_load_3d(dst + Shape::kBoxBytes, &kmap, &full_bar[s], 64, slot, h0);
            lk::tma_load_3d(dst + 2 * Shape::kBoxBytes, &vmap, &full_bar[s], 0, slot, h0);
            lk::tma_load_3d(dst + 3 * Shape::kBoxBytes, &vmap, &full_bar[s], 64, slot, h0);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
      }
    }
  } else {
    // ------------------------------------------------------- consumers ---
    const int g = lane >> 2, c = lane & 3;
    const int kvh = hg * HPC + warp;
    const int qh0 = kvh * G;
    // Q^T as the mma B operand: column n = query head qh0 + n (n < G),
    // k = head_dim index. Columns n >= G are zero.
    uint32_t qb[8][2];
    {
      const T* qrow = static_cast<const T*>(p.q) + static_cast<int64_t>(b) * p.q_stride +
                      static_cast<int64_t>(qh0 + g) * kD;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        if (g < G) {
          qb[ks][0] = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 2 * c);
          qb[ks][1] = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 8 + 2 * c);
        } else {
          qb[ks][0] = 0u;
          qb[ks][1] = 0u;
        }
      }
    }
    float o[8][4];
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    const float sl2 = p.scale_log2;
    const uint32_t smem_base = lk::smem_u32(smem) + warp * (kTok * 128);
    const int j = lane >> 3;

    int it = 0;
    for (int st = st0; st < st1; ++st, ++it) {
      const int s = it % NST;
      if (!lk::mbar_wait(&full_bar[s], (it / NST) & 1)) {
        if (lane == 0) atomicOr(p.status, LK_STATUS_WAIT_TIMEOUT);
        break;
      }
      const uint32_t kb = smem_base + s * Shape::kStageBytes;
      const uint32_t vb = kb + 2 * Shape::kBoxBytes;
      // S^T[token][query column] = K Q^T
      float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t row = (lane & 7) + ((j & 1) << 3);
        const uint32_t chunk = ((ks & 3) << 1) + (j >> 1);
        uint32_t a[4];
        lk::ldsm_x4(kb + (ks >> 2) * Shape::kBoxBytes + lk::swz128(row, chunk), a[0], a[1], a[2],
                    a[3]);
        lk::mma16816<T>(sc, a, qb[ks][0], qb[ks][1]);
      }
      const int pos = st * kTok + g;
      float x0 = sc[0] * sl2, x1 = sc[1] * sl2, x2 = sc[2] * sl2, x3 = sc[3] * sl2;
      if (pos >= ctx) x0 = x1 = -INFINITY;
      if (pos + 8 >= ctx) x2 = x3 = -INFINITY;
      float mx0 = fmaxf(x0, x2), mx1 = fmaxf(x1, x3);
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
      }
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float al0 = exp2f(m0 - mn0), al1 = exp2f(m1 - mn1);
      const float p0 = exp2f(x0 - mn0), p1 = exp2f(x1 - mn1);
      const float p2 = exp2f(x2 - mn0), p3 = exp2f(x3 - mn1);
      l0 = l0 * al0 + p0 + p2;
      l1 = l1 * al1 + p1 + p3;
      m0 = mn0;
      m1 = mn1;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        o[mt][0] *= al0;
        o[mt][1] *= al1;
        o[mt][2] *= al0;
        o[mt][3] *= al1;
      }
      const uint32_t pb0 = lk::movmatrix_t(lk::pack2<T>(p0, p1));
      const uint32_t pb1 = lk::movmatrix_t(lk::pack2<T>(p2, p3));
      // O^T[d][query column] += V^T P^T
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const uint32_t tok = (lane & 7) + ((j >> 1) << 3);
        const uint32_t chunk = ((mt & 3) << 1) + (j & 1);
        uint32_t a[4];
        lk::ldsm_x4_t(vb + (mt >> 2) * Shape::kBoxBytes + lk::swz128(tok, chunk), a[0], a[1],
                      a[2], a[3]);
        lk::mma16816<T>(o[mt], a, pb0, pb1);
      }
      __syncwarp();
      if (lane == 0) lk::mbar_arrive(&empty_bar[s]);
    }
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, off);
      l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
    const int n0 = 2 * c, n1 = 2 * c + 1;
    if (nsp == 1) {
      const float r0 = 1.f / l0, r1 = 1.f / l1;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int d = mt * 16 + g;
        if (n0 < G) {
          store_out<T>(out + (qh0 + n0) * kD + d, o[mt][0] * r0);
          store_out<T>(out + (qh0 + n0) * kD + d + 8, o[mt][2] * r0);
        }
        if (n1 < G) {
          store_out<T>(out + (qh0 + n1) * kD + d, o[mt][1] * r1);
          store_out<T>(out + (qh0 + n1) * kD + d + 8, o[mt][3] * r1);
        }
      }
    } else {
      const int64_t prow = (static_cast<int64_t>(b) * p.num_splits + sp) * p.H;
      float* po = p.part_o + prow * kD;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int d = mt * 16 + g;
        if (n0 < G) {
          po[(qh0 + n0) * kD + d] = o[mt][0];
          po[(qh0 + n0) * kD + d + 8] = o[mt][2];
        }
        if (n1 < G) {
          po[(qh0 + n1) * kD + d] = o[mt][1];
          po[(qh0 + n1) * kD + d + 8] = o[mt][3];
        }
      }
      if (g == 0) {
        float* pml = p.part_ml + prow * 2;
        if (n0 < G) {
          pml[(qh0 + n0) * 2] = m0;
          pml[(qh0 + n0) * 2 + 1] = l0;
        }
        if (n1 < G) {
          pml[(qh0 + n1) * 2] = m1;
          pml[(qh0 + n1) * 2 + 1] = l1;
        }
      }
    }
  }

  if (nsp == 1) return;
  // ---------------------------------------------- split-KV merge (last CTA) ---
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(p.counters + b * p.num_groups + hg, 1);
    s_last = (prev == nsp - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int nq = HPC * G;
  const int qbase = hg * nq;
  const int64_t rowb = static_cast<int64_t>(b) * p.num_splits;
  for (int i = threadIdx.x; i < nq * kD; i += Shape::kThreads) {
    const int qh = qbase + i / kD, d = i % kD;
    float M = -INFINITY;
    for (int s = 0; s < nsp; ++s) M = fmaxf(M, __ldcg(p.part_ml + ((rowb + s) * p.H + qh) * 2));
    float L = 0.f, acc = 0.f;
    for (int s = 0; s < nsp; ++s) {
      const float* ml = p.part_ml + ((rowb + s) * p.H + qh) * 2;
      const float w = exp2f(__ldcg(ml) - M);
      L += __ldcg(ml + 1) * w;
      acc += __ldcg(p.part_o + ((rowb + s) * p.H + qh) * kD + d) * w;
    }
    store_out<T>(out + qh * kD + d, acc / L);
  }
  if (threadIdx.x == 0) p.counters[b * p.num_groups + hg] = 0;
}

// Workspace layout: [status: int32, padded to 256 B][counters: kMaxCounters
// int32, a fixed region so that calls with different B find it where the
// previous call left it zeroed][part_ml: B*splits*H*2 f32][part_o: B*splits*H*D f32]
constexpr int64_t kMaxCounters = 65536;
constexpr size_t kHeadBytes = 256 + kMaxCounters * 4;
size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

int heads_per_cta(int H_kv) {
  if (H_kv % 8 == 0) return 8;
  if (H_kv % 4 == 0) return 4;
  if (H_kv % 2 == 0) return 2;
  return 1;
}

template <typename T, int HPC, int NST>
int launch_decode(const CUtensorMap& km, const CUtensorMap& vm, const DecodeParams& p, int B,
                  cudaStream_t s) {
  using Shape = DecodeShape<HPC, NST>;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(paged_decode_kernel<T, HPC, NST>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Shape::kSmem) != cudaSuccess)
      return LK_ERR_CUDA;
    configured[dev] = 1;
  }
  dim3 grid(p.num_splits, p.num_groups, B);
  paged_decode_kernel<T, HPC, NST><<<grid, Shape::kThreads, Shape::kSmem, s>>>(km, vm, p);
  return lk::check_launch();
}

template <typename T>
int dispatch_decode(int hpc, const CUtensorMap& km, const CUtensorMap& vm, const DecodeParams& p,
                    int B, cudaStream_t s) {
  switch (hpc) {
    case 8: return launch_decode<T, 8, 3>(km, vm, p, B, s);
    case 4: return launch_decode<T, 4, 6>(km, vm, p, B, s);
    case 2: return launch_decode<T, 2, 8>(km, vm, p, B, s);
    default: return launch_decode<T, 1, 8>(km, vm, p, B, s);
  }
}

}  // namespace

extern "C" int lk_paged_decode_num_splits(int32_t B, int32_t H_kv, int32_t max_blocks_per_seq,
                                          int32_t block_size) {
  if (B <= 0 || H_kv <= 0 || max_blocks_per_seq <= 0 || block_size <= 0) return 1;
  const int groups = H_kv / heads_per_cta(H_kv);
  const int64_t max_stages = (static_cast<int64_t>(max_blocks_per_seq) * block_size + 15) / 16;
  const int64_t units = static_cast<int64_t>(B) * groups;
  // Enough CTAs to cover every SM twice even if all sequences were long,
  // no split shorter than 8 stages (128 tokens), and no split longer than
  // 32 stages (512 tokens, 2 MiB of bf16 K+V) so that long sequences do not
  // leave a tail on a few SMs.
  int64_t splits = (2 * lk::num_sms() + units - 1) / units;
  splits = std::min<int64_t>(splits, (max_stages + 7) / 8);
  splits = std::max<int64_t>(splits, (max_stages + 31) / 32);
  splits = std::max<int64_t>(1, std::min<int64_t>(splits, max_stages));
  return static_cast<int>(std::min<int64_t>(splits, 65535));
}

extern "C" size_t lk_paged_decode_workspace_bytes(int32_t B, int32_t H, int32_t H_kv, int32_t D,
                                                  int32_t num_splits) {
  if (B <= 0 || H <= 0 || H_kv <= 0 || D <= 0) return 0;
  const int groups = H_kv / heads_per_cta(H_kv);
  (void)groups;
  size_t bytes = kHeadBytes;
  if (num_splits > 1) {
    bytes += align256(static_cast<size_t>(B) * num_splits * H * 2 * 4);
    bytes += align256(static_cast<size_t>(B) * num_splits * H * D * 4);
  }
  return bytes;
}

extern "C" int lk_paged_decode(void* out, int64_t out_token_stride, const void* q,
                               int64_t q_token_stride, const void* k_cache, const void* v_cache,
                               int64_t num_blocks, const int32_t* block_tables,
                               int64_t block_table_stride, const int32_t* context_lens, int32_t B,
                               int32_t H, int32_t H_kv, int32_t D, int32_t block_size,
                               int32_t max_blocks_per_seq, float scale, int32_t num_splits,
                               void* workspace, size_t workspace_bytes, int32_t dtype,
                               void* stream) {
  if (B < 0 || H <= 0 || H_kv <= 0 || H % H_kv != 0 || num_blocks <= 0 || block_size <= 0 ||
      max_blocks_per_seq < 0)
    return LK_ERR_INVALID_ARG;
  if (B == 0) return LK_OK;
  if (!out || !q || !k_cache || !v_cache || !block_tables || !context_lens)
    return LK_ERR_INVALID_ARG;
  if (dtype != LK_DTYPE_BF16 && dtype != LK_DTYPE_F16) return LK_ERR_UNSUPPORTED;
  if (D != kD || block_size % kTok != 0 || H / H_kv > 8) return LK_ERR_UNSUPPORTED;
  if (B > 65535 || max_blocks_per_seq == 0) return LK_ERR_INVALID_ARG;
  if (static_cast<int64_t>(B) * (H_kv / heads_per_cta(H_kv)) > kMaxCounters)
    return LK_ERR_UNSUPPORTED;
  if (num_blocks * block_size > 0x7fffffffLL) return LK_ERR_UNSUPPORTED;
  if (((reinterpret_cast<uintptr_t>(q) & 3u) != 0) || (q_token_stride & 1) != 0)
    return LK_ERR_ALIGNMENT;
  if (num_splits <= 0)
    num_splits = lk_paged_decode_num_splits(B, H_kv, max_blocks_per_seq, block_size);
  const size_t need = lk_paged_decode_workspace_bytes(B, H, H_kv, D, num_splits);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return LK_ERR_WORKSPACE;

  const int hpc = heads_per_cta(H_kv);
  const int64_t num_slots = num_blocks * block_size;
  CUtensorMap km, vm;
  int rc = lk::get_kv_tensor_map(&km, k_cache, num_slots, H_kv, D, dtype, kTok, hpc);
  if (rc != LK_OK) return rc;
  rc = lk::get_kv_tensor_map(&vm, v_cache, num_slots, H_kv, D, dtype, kTok, hpc);
  if (rc != LK_OK) return rc;

  const int64_t max_stages = (static_cast<int64_t>(max_blocks_per_seq) * block_size + 15) / 16;
  DecodeParams p;
  p.out = out;
  p.out_stride = out_token_stride;
  p.q = q;
  p.q_stride = q_token_stride;
  p.block_tables = block_tables;
  p.bt_stride = block_table_stride;
  p.context_lens = context_lens;
  p.num_blocks = num_blocks;
  p.H = H;
  p.G = H / H_kv;
  p.bs = block_size;
  p.max_blocks = max_blocks_per_seq;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.num_splits = num_splits;
  p.stages_per_split = static_cast<int>((max_stages + num_splits - 1) / num_splits);
  p.num_groups = H_kv / hpc;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const size_t cnt_bytes = kHeadBytes;
  p.status = reinterpret_cast<int32_t*>(ws);
  p.counters = reinterpret_cast<int32_t*>(ws + 256);
  p.part_ml = reinterpret_cast<float*>(ws + cnt_bytes);
  p.part_o = reinterpret_cast<float*>(
      ws + cnt_bytes + align256(static_cast<size_t>(B) * num_splits * H * 2 * 4));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == LK_DTYPE_BF16) return dispatch_decode<__nv_bfloat16>(hpc, km, vm, p, B, s);
  return dispatch_decode<__half>(hpc, km, vm, p, B, s);
}

extern "C" int lk_paged_decode_status(const void* workspace, void* stream) {
  if (!workspace) return LK_ERR_INVALID_ARG;
  int32_t v = 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(&v, workspace, sizeof(v), cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return LK_ERR_CUDA;
  if (cudaStreamSynchronize(s) != cudaSuccess) return LK_ERR_CUDA;
  return v;
}
