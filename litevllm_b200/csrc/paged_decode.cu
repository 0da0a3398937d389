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

#include <stdlib.h>

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
  int prefetch;           // stages prefetched into L2 ahead of the ring (0 = off)
  int stages_per_split;
  int num_splits;
  int num_groups;         // H_kv / HPC
  int32_t* counters;      // [B * num_groups]
  int32_t* status;
  float* part_ml;         // [B][num_splits][H][2]  (m in log2 domain, l)
  float* part_o;          // [B][num_splits][H][D]
  const int2* order;      // [B * num_splits]: (b * num_splits + split, ctx), longest first
  int* work;              // streaming kernel's unit counter (zeroed by the ordering kernel)
  int first_stage;        // shared-prefix mode: stages before it are covered by prefix partials
  int part_offset;        // ... which fill partial slots [0, part_offset) of each row
};

// Launch order of the split kernel's (sequence, split) units: longest first.
// The hardware hands CTAs to SMs in blockIdx order; with units of up to 64
// stages (4 MB of K/V) dispatched in sequence order, the last wave leaves
// SMs idle for tens of microseconds. One CTA buckets the units by stage
// count (64 buckets, longest bucket first, empty contexts last) and writes
// the list; CTA i of the decode kernel takes entry i. Order within a bucket
// is arbitrary; results do not depend on it (each unit's partial has a fixed
// slot and the merge reads them in split order).
constexpr int kOrderBuckets = 64;

__global__ void __launch_bounds__(1024) decode_order_kernel(const int32_t* context_lens, int B,
                                                            int cap, int spp, int num_splits,
                                                            int2* order, int* work, int first,
                                                            int* work2) {
  static_assert(kOrderBuckets + 1 <= 96, "one warp scans the buckets, three per lane");
  // Launched with lk::launch_after_previous: let the split kernel start
  // launching, then wait for the previous kernel (the step's KV store) before
  // touching memory, so this grid's completion implies the store's.
  lk::pdl_launch_dependents();
  lk::pdl_wait();
  if (threadIdx.x == 0 && work) *work = 0;
  if (threadIdx.x == 0 && work2) *work2 = 0;
  __shared__ int hist[96];
  __shared__ int cursor[96];
  __shared__ int total;
  const int tid = threadIdx.x;
  if (tid < 96) hist[tid] = 0;
  auto bucket = [&](int n) {
    return n <= 0 ? kOrderBuckets
                  : (kOrderBuckets - 1) -
                        static_cast<int>(static_cast<int64_t>(n - 1) * kOrderBuckets / spp);
  };
  auto stages = [&](int ctx) {  // stages this kernel's units cover (past `first`)
    ctx = ctx < 0 ? 0 : (ctx > cap ? cap : ctx);
    const int n = (ctx + kTok - 1) / kTok - first;
    return n < 0 ? 0 : n;
  };
  // Each thread's first sequence stays in registers between the passes
  // (one global read for B <= 1024).
  const int ctx0 = tid < B ? context_lens[tid] : 0;
  __syncthreads();
  for (int b = tid; b < B; b += blockDim.x) {
    const int nst = stages(b == tid ? ctx0 : context_lens[b]);
    const int nsp = nst == 0 ? 1 : (nst + spp - 1) / spp;
    for (int sp = 0; sp < nsp; ++sp)
      atomicAdd(&hist[bucket(nst == 0 ? 0 : min(spp, nst - sp * spp))], 1);
  }
  __syncthreads();
  if (tid < 32) {  // exclusive scan of the 65 buckets: three per lane
    const int h0 = hist[3 * tid], h1 = hist[3 * tid + 1], h2 = hist[3 * tid + 2];
    int x = h0 + h1 + h2;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (tid >= o) x += y;
    }
    const int base = x - (h0 + h1 + h2);
    cursor[3 * tid] = base;
    cursor[3 * tid + 1] = base + h0;
    cursor[3 * tid + 2] = base + h0 + h1;
    if (tid == 31) total = x;
  }
  __syncthreads();
  for (int b = tid; b < B; b += blockDim.x) {
    const int ctx_raw = b == tid ? ctx0 : context_lens[b];
    const int nst = stages(ctx_raw);
    const int nsp = nst == 0 ? 1 : (nst + spp - 1) / spp;
    for (int sp = 0; sp < nsp; ++sp) {
      const int pos = atomicAdd(&cursor[bucket(nst == 0 ? 0 : min(spp, nst - sp * spp))], 1);
      order[pos] = make_int2(b * num_splits + sp, ctx_raw);
    }
  }
  for (int i = total + tid; i < B * num_splits; i += blockDim.x) order[i] = make_int2(-1, 0);
}

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

  // Launched with lk::launch_after_previous after the ordering kernel: wait
  // for it (and through it for the KV store) before reading anything. The
  // kernel after this one (the sampler) may then start launching: its blocks
  // wait for this grid to complete, and take SMs as the last wave drains.
  // Shared-prefix mode (part_offset > 0): the grid ahead is the prefix kernel,
  // a plain launch behind the ordering kernel and the store, so everything
  // but the prefix partials is complete once this grid starts; the wait
  // moves to the merge, which reads those partials.
  if (p.part_offset == 0) lk::pdl_wait();
  lk::pdl_launch_dependents();
  int2 unit;
  if (p.order != nullptr) {
    unit = p.order[blockIdx.x];
    if (unit.x < 0) return;
  } else {
    const int bb = blockIdx.x / p.num_splits;
    unit = make_int2(blockIdx.x, p.context_lens[bb]);
  }
  const int sp = unit.x % p.num_splits, hg = blockIdx.y, b = unit.x / p.num_splits;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.G;

  int ctx = unit.y;
  const int cap = p.max_blocks * p.bs;
  if (ctx > cap) {
    if (threadIdx.x == 0 && sp == 0) atomicOr(p.status, LK_STATUS_CTX_OOB);
    ctx = cap;
  }
  if (ctx < 0) ctx = 0;
  const int nst = (ctx + kTok - 1) / kTok;
  const int spp = p.stages_per_split;
  // Units cover the stages past first_stage (0 unless a shared prefix's
  // partials already fill slots [0, part_offset)); nsp = this kernel's splits
  // of the row, nparts = all partial slots the merge combines.
  if (p.part_offset > 0 && ctx < p.first_stage * kTok && sp == 0 && hg == 0 &&
      threadIdx.x == 0)
    atomicOr(p.status, LK_STATUS_CTX_OOB);  // shared prefix longer than this row's context
  const int sst = nst > p.first_stage ? nst - p.first_stage : 0;
  const int nsp = sst == 0 ? 1 : (sst + spp - 1) / spp;
  const int nparts = p.part_offset + nsp;
  if (sp >= nsp) return;

  T* out = static_cast<T*>(p.out) + static_cast<int64_t>(b) * p.out_stride;
  if (nst == 0 && p.part_offset == 0) {
    // softmax over an all -inf row is NaN in the reference; reproduce it.
    const int nq = HPC * G;
    for (int i = threadIdx.x; i < nq * kD; i += Shape::kThreads)
      store_out<T>(out + (hg * nq) * kD + i, __int_as_float(0x7fc00000));
    return;
  }
  const int st0 = p.first_stage + sp * spp;
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
    // Each lane resolves one stage's starting slot ahead of time so the
    // block-table reads overlap instead of serialising the TMA issue; the
    // next 32 stages are resolved one batch early so that L2 prefetches can
    // run `prefetch` stages ahead of the shared-memory ring.
    const int oob = static_cast<int>(num_slots < 0x7fffffffLL ? num_slots : 0x7fffffffLL);
    auto lookup = [&](int st) -> int {
      if (st >= st1) return -1;
      const int pos = st * kTok;
      const int blk = __ldg(bt + pos / p.bs);
      if (blk < 0 || blk >= p.num_blocks) {
        atomicOr(p.status, LK_STATUS_BLOCK_OOB);
        return oob;  // past the end: TMA reads zeros
      }
      return blk * p.bs + (pos % p.bs);
    };
    const int PF = p.prefetch;
    const int h0 = hg * HPC;
    int nxt = lookup(st0 + lane);
    {
      // warm-up prefetches for the first PF stages
      for (int i = 0; i < PF && i < 32; ++i) {
        const int sl = __shfl_sync(0xffffffffu, nxt, i);
        if (lane == 0 && sl >= 0) {
          lk::tma_prefetch_3d(&kmap, 0, sl, h0);
          lk::tma_prefetch_3d(&kmap, 64, sl, h0);
          lk::tma_prefetch_3d(&vmap, 0, sl, h0);
          lk::tma_prefetch_3d(&vmap, 64, sl, h0);
        }
      }
    }
    for (int base = st0; base < st1 && ok; base += 32) {
      const int cur = nxt;
      nxt = lookup(base + 32 + lane);
      const int n = min(32, st1 - base);
      for (int i = 0; i < n; ++i, ++it) {
        const int slot = __shfl_sync(0xffffffffu, cur, i);
        int pslot = -1;
        if (PF > 0) {
          const int j = i + PF;
          const int a = __shfl_sync(0xffffffffu, cur, j & 31);
          const int c = __shfl_sync(0xffffffffu, nxt, j & 31);
          pslot = j < 32 ? a : c;
        }
        if (lane == 0) {
          const int s = it % NST;
          const uint32_t ph = ((it / NST) & 1) ^ 1;
          if (pslot >= 0) {
            lk::tma_prefetch_3d(&kmap, 0, pslot, h0);
            lk::tma_prefetch_3d(&kmap, 64, pslot, h0);
            lk::tma_prefetch_3d(&vmap, 0, pslot, h0);
            lk::tma_prefetch_3d(&vmap, 64, pslot, h0);
          }
          if (!lk::mbar_wait(&empty_bar[s], ph)) {
            atomicOr(p.status, LK_STATUS_WAIT_TIMEOUT);
            ok = false;
          } else {
            lk::mbar_arrive_expect_tx(&full_bar[s], Shape::kStageBytes);
            uint8_t* dst = smem + s * Shape::kStageBytes;
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
    if (nparts == 1) {
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
      const int64_t prow = (static_cast<int64_t>(b) * p.num_splits + p.part_offset + sp) * p.H;
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

  if (nparts == 1) return;
  // ---------------------------------------------- split-KV merge (last CTA) ---
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(p.counters + b * p.num_groups + hg, 1);
    s_last = (prev == nsp - 1);
  }
  __syncthreads();
  if (!s_last) return;
  if (p.part_offset > 0) lk::pdl_wait();  // the prefix kernel's partials
  __threadfence();
  const int nq = HPC * G;
  const int qbase = hg * nq;
  const int64_t rowb = static_cast<int64_t>(b) * p.num_splits;
  if (nq * nparts * 4 <= Shape::kSmem - 1024) {
    // Weights w[q][s] = exp2(m_s - M) / L into the (idle) ring once, then
    // every split's partial rows as float4 with all loads of a thread in
    // flight together: the merge is a few L2 round trips, not one per output.
    float* w = reinterpret_cast<float*>(smem);
    for (int q = threadIdx.x; q < nq; q += Shape::kThreads) {
      const float* ml = p.part_ml + (rowb * p.H + qbase + q) * 2;
      float M = -INFINITY;
      for (int s2 = 0; s2 < nparts; ++s2) M = fmaxf(M, __ldcg(ml + s2 * p.H * 2));
      float L = 0.f;
      for (int s2 = 0; s2 < nparts; ++s2) {
        const float e = exp2f(__ldcg(ml + s2 * p.H * 2) - M);
        w[q * nparts + s2] = e;
        L += __ldcg(ml + s2 * p.H * 2 + 1) * e;
      }
      const float inv = 1.f / L;
      for (int s2 = 0; s2 < nparts; ++s2) w[q * nparts + s2] *= inv;
    }
    __syncthreads();
    constexpr int kU = 4;
    const int n4 = nq * kD / 4;
    const float4* po4 = reinterpret_cast<const float4*>(p.part_o + (rowb * p.H + qbase) * kD);
    const int64_t sstride4 = static_cast<int64_t>(p.H) * kD / 4;
    for (int i0 = threadIdx.x; i0 < n4; i0 += kU * Shape::kThreads) {
      float4 acc[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
      for (int s2 = 0; s2 < nparts; ++s2) {
        float4 v[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int i = i0 + u * Shape::kThreads;
          v[u] = i < n4 ? __ldcg(po4 + s2 * sstride4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int i = i0 + u * Shape::kThreads;
          const float wt = i < n4 ? w[(i * 4 / kD) * nparts + s2] : 0.f;
          acc[u].x += v[u].x * wt;
          acc[u].y += v[u].y * wt;
          acc[u].z += v[u].z * wt;
          acc[u].w += v[u].w * wt;
        }
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int i = i0 + u * Shape::kThreads;
        if (i < n4) {
          T* o = out + qbase * kD + i * 4;
          store_out<T>(o, acc[u].x);
          store_out<T>(o + 1, acc[u].y);
          store_out<T>(o + 2, acc[u].z);
          store_out<T>(o + 3, acc[u].w);
        }
      }
    }
  } else {
    for (int i = threadIdx.x; i < nq * kD; i += Shape::kThreads) {
      const int qh = qbase + i / kD, d = i % kD;
      float M = -INFINITY;
      for (int s = 0; s < nparts; ++s) M = fmaxf(M, __ldcg(p.part_ml + ((rowb + s) * p.H + qh) * 2));
      float L = 0.f, acc = 0.f;
      for (int s = 0; s < nparts; ++s) {
        const float* ml = p.part_ml + ((rowb + s) * p.H + qh) * 2;
        const float wt = exp2f(__ldcg(ml) - M);
        L += __ldcg(ml + 1) * wt;
        acc += __ldcg(p.part_o + ((rowb + s) * p.H + qh) * kD + d) * wt;
      }
      store_out<T>(out + qh * kD + d, acc / L);
    }
  }
  if (threadIdx.x == 0) p.counters[b * p.num_groups + hg] = 0;
}

// ------------------------------------------------------------------------
// Persistent, stage-balanced decode.
//
// The (unit, stage) space — unit u = b * groups + hg, nst(u) = ceil(ctx_b/16)
// stages of 16 tokens — is flattened in unit order and cut into gridDim.x
// equal contiguous ranges, one per CTA (grid = number of SMs, one CTA per
// SM). The producer streams TMA loads across unit boundaries without
// draining the ring; every stage carries a small descriptor (unit, stage,
// flags) in shared memory. A unit split across CTAs (at most two partial
// segments per CTA: its first and its last) writes (m, l, o) partials into
// slot (cta, 0|1); each consumer warp counts the segments of its own
// (sequence, KV head) with an atomic and the last one merges. No CTA ever
// waits on another.
struct DecodeState {
  float o[8][4];
  float m0, m1, l0, l1;
};

template <typename T, int kBoxBytes>
LK_DEVINL void decode_stage(DecodeState& st, const uint32_t (&qb)[8][2], uint32_t kb,
                            uint32_t vb, int pos0, int ctx, float sl2, int lane) {
  const int g = lane >> 2, j = lane >> 3;
  float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    const uint32_t row = (lane & 7) + ((j & 1) << 3);
    const uint32_t chunk = ((ks & 3) << 1) + (j >> 1);
    uint32_t a[4];
    lk::ldsm_x4(kb + (ks >> 2) * kBoxBytes + lk::swz128(row, chunk), a[0], a[1], a[2], a[3]);
    lk::mma16816<T>(sc, a, qb[ks][0], qb[ks][1]);
  }
  const int pos = pos0 + g;
  float x0 = sc[0] * sl2, x1 = sc[1] * sl2, x2 = sc[2] * sl2, x3 = sc[3] * sl2;
  if (pos >= ctx) x0 = x1 = -INFINITY;
  if (pos + 8 >= ctx) x2 = x3 = -INFINITY;
  float mx0 = fmaxf(x0, x2), mx1 = fmaxf(x1, x3);
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
  }
  const float mn0 = fmaxf(st.m0, mx0), mn1 = fmaxf(st.m1, mx1);
  const float al0 = exp2f(st.m0 - mn0), al1 = exp2f(st.m1 - mn1);
  const float p0 = exp2f(x0 - mn0), p1 = exp2f(x1 - mn1);
  const float p2 = exp2f(x2 - mn0), p3 = exp2f(x3 - mn1);
  st.l0 = st.l0 * al0 + p0 + p2;
  st.l1 = st.l1 * al1 + p1 + p3;
  st.m0 = mn0;
  st.m1 = mn1;
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    st.o[mt][0] *= al0;
    st.o[mt][1] *= al1;
    st.o[mt][2] *= al0;
    st.o[mt][3] *= al1;
  }
  const uint32_t pb0 = lk::movmatrix_t(lk::pack2<T>(p0, p1));
  const uint32_t pb1 = lk::movmatrix_t(lk::pack2<T>(p2, p3));
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    const uint32_t tok = (lane & 7) + ((j >> 1) << 3);
    const uint32_t chunk = ((mt & 3) << 1) + (j & 1);
    uint32_t a[4];
    lk::ldsm_x4_t(vb + (mt >> 2) * kBoxBytes + lk::swz128(tok, chunk), a[0], a[1], a[2], a[3]);
    lk::mma16816<T>(st.o[mt], a, pb0, pb1);
  }
}

// CTA that owns flattened stage s when S stages are cut into n ranges
// [floor(i*S/n), floor((i+1)*S/n)).
LK_DEVINL int stage_owner(int64_t s, int64_t S, int n) {
  return static_cast<int>(((s + 1) * n - 1) / S);
}

// Whether CTA c's range is non-empty (S < n leaves some CTAs without stages;
// such CTAs hold no segment of any unit).
LK_DEVINL bool range_nonempty(int c, int64_t S, int n) {
  return (S * (c + 1)) / n > (S * c) / n;
}

constexpr int kFirst = 1, kLast = 2;

template <typename T, int HPC, int NST>
__global__ void __launch_bounds__((HPC + 1) * 32, 1)
paged_decode_persistent_kernel(const __grid_constant__ CUtensorMap kmap,
                               const __grid_constant__ CUtensorMap vmap, const DecodeParams p,
                               int num_units) {
  using Shape = DecodeShape<HPC, NST>;
  constexpr int kThreads = Shape::kThreads;
  constexpr int kWarps = HPC + 1;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[NST];
  __shared__ __align__(8) uint64_t empty_bar[NST];
  __shared__ int meta[NST][6];  // unit, stage-in-unit, ctx, flags, P lo, P hi
  __shared__ long long s_red[kWarps];
  __shared__ long long s_scan[kWarps];
  __shared__ long long s_P0;
  __shared__ int s_u0;
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int cta = blockIdx.x, nctas = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.G, groups = p.num_groups;
  const int cap = p.max_blocks * p.bs;

  // ---- pass 1: total stages; NaN rows for empty contexts
  long long local = 0;
  for (int u = threadIdx.x; u < num_units; u += kThreads) {
    const int b = u / groups;
    int ctx = p.context_lens[b];
    if (ctx > cap) {
      if (cta == 0) atomicOr(p.status, LK_STATUS_CTX_OOB);
      ctx = cap;
    }
    const int n = ctx > 0 ? (ctx + kTok - 1) / kTok : 0;
    local += n;
    if (n == 0 && (u % nctas) == cta) {
      // softmax over an all -inf row is NaN in the reference; reproduce it.
      T* out = static_cast<T*>(p.out) + static_cast<int64_t>(b) * p.out_stride;
      const int nq = HPC * G, hg = u % groups;
      for (int i = 0; i < nq * kD; ++i)
        store_out<T>(out + (hg * nq) * kD + i, __int_as_float(0x7fc00000));
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) local += __shfl_xor_sync(0xffffffffu, local, off);
  if (lane == 0) s_red[warp] = local;
  if (threadIdx.x == 0) s_u0 = -1;
  __syncthreads();
  long long S = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) S += s_red[w];
  const long long start = S * cta / nctas, end = S * (cta + 1) / nctas;
  if (start >= end) return;

  // ---- pass 2: first unit u0 with P(u0) <= start < P(u0) + nst(u0)
  long long base = 0;
  for (int c0 = 0; c0 < num_units; c0 += kThreads) {
    const int u = c0 + threadIdx.x;
    int n = 0;
    if (u < num_units) {
      const int ctx = min(p.context_lens[u / groups], cap);
      n = ctx > 0 ? (ctx + kTok - 1) / kTok : 0;
    }
    long long incl = n;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const long long v = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += v;
    }
    if (lane == 31) s_scan[warp] = incl;
    __syncthreads();
    long long woff = 0, tot = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      if (w < warp) woff += s_scan[w];
      tot += s_scan[w];
    }
    const long long P = base + woff + incl - n;
    if (n > 0 && P <= start && start < P + n) {
      s_u0 = u;
      s_P0 = P;
    }
    __syncthreads();
    if (s_u0 >= 0) break;
    base += tot;
  }
  const int u0 = s_u0;
  const long long P0 = s_P0;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < NST; ++s) {
      lk::mbar_init(&full_bar[s], 1);
      lk::mbar_init(&empty_bar[s], HPC);
    }
    lk::fence_barrier_init();
  }
  __syncthreads();
  const int total = static_cast<int>(end - start);

  if (warp == HPC) {
    // ------------------------------------------------------- producer ---
    if (lane == 0) {
      lk::prefetch_tensormap(&kmap);
      lk::prefetch_tensormap(&vmap);
    }
    const int64_t num_slots = p.num_blocks * p.bs;
    const int oob = static_cast<int>(num_slots < 0x7fffffffLL ? num_slots : 0x7fffffffLL);
    bool ok = true;
    int it = 0;
    long long P = P0;
    for (int u = u0; u < num_units && P < end && ok; ++u) {
      const int b = u / groups, hg = u % groups;
      const int ctx = min(p.context_lens[b], cap);
      const int n = ctx > 0 ? (ctx + kTok - 1) / kTok : 0;
      const int lo = static_cast<int>((start > P ? start : P) - P);
      const int hi = static_cast<int>(((P + n) < end ? (P + n) : end) - P);
      const int32_t* bt = p.block_tables + static_cast<int64_t>(b) * p.bt_stride;
      const int h0 = hg * HPC;
      const int PF = p.prefetch;
      auto lookup = [&](int t) -> int {
        if (t >= hi) return -1;
        const int pos = t * kTok;
        const int blk = __ldg(bt + pos / p.bs);
        if (blk < 0 || blk >= p.num_blocks) {
          atomicOr(p.status, LK_STATUS_BLOCK_OOB);
          return oob;
        }
        return blk * p.bs + (pos % p.bs);
      };
      int nxt = lookup(lo + lane);
      for (int i = 0; i < PF && i < 32; ++i) {
        const int sl = __shfl_sync(0xffffffffu, nxt, i);
        if (lane == 0 && sl >= 0) {
          lk::tma_prefetch_3d(&kmap, 0, sl, h0);
          lk::tma_prefetch_3d(&kmap, 64, sl, h0);
          lk::tma_prefetch_3d(&vmap, 0, sl, h0);
          lk::tma_prefetch_3d(&vmap, 64, sl, h0);
        }
      }
      for (int t0 = lo; t0 < hi && ok; t0 += 32) {
        const int cur = nxt;
        nxt = lookup(t0 + 32 + lane);
        const int cnt = min(32, hi - t0);
        for (int i = 0; i < cnt; ++i, ++it) {
          const int slot = __shfl_sync(0xffffffffu, cur, i);
          int pslot = -1;
          if (PF > 0) {
            const int j = i + PF;
            const int a = __shfl_sync(0xffffffffu, cur, j & 31);
            const int c = __shfl_sync(0xffffffffu, nxt, j & 31);
            pslot = j < 32 ? a : c;
          }
          if (lane == 0) {
            const int s = it % NST;
            if (pslot >= 0) {
              lk::tma_prefetch_3d(&kmap, 0, pslot, h0);
              lk::tma_prefetch_3d(&kmap, 64, pslot, h0);
              lk::tma_prefetch_3d(&vmap, 0, pslot, h0);
              lk::tma_prefetch_3d(&vmap, 64, pslot, h0);
            }
            if (!lk::mbar_wait(&empty_bar[s], ((it / NST) & 1) ^ 1)) {
              atomicOr(p.status, LK_STATUS_WAIT_TIMEOUT);
              ok = false;
            } else {
              const int tt = t0 + i;
              meta[s][0] = u;
              meta[s][1] = tt;
              meta[s][2] = ctx;
              meta[s][3] = (tt == lo ? kFirst : 0) | (tt == hi - 1 ? kLast : 0);
              meta[s][4] = static_cast<int>(P & 0xffffffffLL);
              meta[s][5] = static_cast<int>(P >> 32);
              lk::mbar_arrive_expect_tx(&full_bar[s], Shape::kStageBytes);
              uint8_t* dst = smem + s * Shape::kStageBytes;
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
      P += n;
    }
    return;
  }

  // --------------------------------------------------------- consumers ---
  const int g = lane >> 2, c = lane & 3;
  const int n0 = 2 * c, n1 = 2 * c + 1;
  const float sl2 = p.scale_log2;
  const uint32_t smem_base = lk::smem_u32(smem) + warp * (kTok * 128);
  DecodeState st;
  uint32_t qb[8][2];
  for (int it = 0; it < total; ++it) {
    const int s = it % NST;
    if (!lk::mbar_wait(&full_bar[s], (it / NST) & 1)) {
      if (lane == 0) atomicOr(p.status, LK_STATUS_WAIT_TIMEOUT);
      break;
    }
    const int u = meta[s][0], t = meta[s][1], ctx = meta[s][2], flags = meta[s][3];
    const long long P = (static_cast<long long>(meta[s][5]) << 32) |
                        static_cast<unsigned int>(meta[s][4]);
    const int b = u / groups, hg = u % groups;
    const int kvh = hg * HPC + warp;
    const int qh0 = kvh * G;
    if (flags & kFirst) {
      const T* qrow = static_cast<const T*>(p.q) + static_cast<int64_t>(b) * p.q_stride +
                      static_cast<int64_t>(qh0 + g) * kD;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        qb[ks][0] = g < G ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 2 * c) : 0u;
        qb[ks][1] = g < G ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 8 + 2 * c) : 0u;
      }
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) st.o[mt][0] = st.o[mt][1] = st.o[mt][2] = st.o[mt][3] = 0.f;
      st.m0 = st.m1 = -INFINITY;
      st.l0 = st.l1 = 0.f;
    }
    const uint32_t kb = smem_base + s * Shape::kStageBytes;
    decode_stage<T, Shape::kBoxBytes>(st, qb, kb, kb + 2 * Shape::kBoxBytes, t * kTok, ctx, sl2,
                                      lane);
    __syncwarp();
    if (lane == 0) lk::mbar_arrive(&empty_bar[s]);
    if (!(flags & kLast)) continue;

    // ---- segment finished: final output, or partial + merge by the last segment
    float l0 = st.l0, l1 = st.l1;
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, off);
      l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
    const int nst = (ctx + kTok - 1) / kTok;
    const int c0 = stage_owner(P, S, nctas), c1 = stage_owner(P + nst - 1, S, nctas);
    T* out = static_cast<T*>(p.out) + static_cast<int64_t>(b) * p.out_stride;
    if (c0 == c1) {
      const float r0 = 1.f / l0, r1 = 1.f / l1;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int d = mt * 16 + g;
        if (n0 < G) {
          store_out<T>(out + (qh0 + n0) * kD + d, st.o[mt][0] * r0);
          store_out<T>(out + (qh0 + n0) * kD + d + 8, st.o[mt][2] * r0);
        }
        if (n1 < G) {
          store_out<T>(out + (qh0 + n1) * kD + d, st.o[mt][1] * r1);
          store_out<T>(out + (qh0 + n1) * kD + d + 8, st.o[mt][3] * r1);
        }
      }
      continue;
    }
    const int slot = cta * 2 + (cta == c0 ? 1 : 0);
    const int64_t prow = static_cast<int64_t>(slot) * p.H;
    float* po = p.part_o + prow * kD;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      const int d = mt * 16 + g;
      if (n0 < G) {
        po[(qh0 + n0) * kD + d] = st.o[mt][0];
        po[(qh0 + n0) * kD + d + 8] = st.o[mt][2];
      }
      if (n1 < G) {
        po[(qh0 + n1) * kD + d] = st.o[mt][1];
        po[(qh0 + n1) * kD + d + 8] = st.o[mt][3];
      }
    }
    if (g == 0) {
      float* pml = p.part_ml + prow * 2;
      if (n0 < G) {
        pml[(qh0 + n0) * 2] = st.m0;
        pml[(qh0 + n0) * 2 + 1] = l0;
      }
      if (n1 < G) {
        pml[(qh0 + n1) * 2] = st.m1;
        pml[(qh0 + n1) * 2 + 1] = l1;
      }
    }
    __threadfence();
    __syncwarp();
    int prev = 0;
    int32_t* counter = p.counters + static_cast<int64_t>(b) * (groups * HPC) + kvh;
    if (lane == 0) prev = atomicAdd(counter, 1);
    prev = __shfl_sync(0xffffffffu, prev, 0);
    int nseg = 0;
    for (int cc = c0; cc <= c1; ++cc) nseg += range_nonempty(cc, S, nctas) ? 1 : 0;
    if (prev != nseg - 1) continue;
    __threadfence();
    for (int i = lane; i < G * kD; i += 32) {
      const int qh = qh0 + i / kD, d = i % kD;
      float M = -INFINITY;
      for (int cc = c0; cc <= c1; ++cc) {
        if (!range_nonempty(cc, S, nctas)) continue;
        const int sl = cc * 2 + (cc == c0 ? 1 : 0);
        M = fmaxf(M, __ldcg(p.part_ml + (static_cast<int64_t>(sl) * p.H + qh) * 2));
      }
      float L = 0.f, acc = 0.f;
      for (int cc = c0; cc <= c1; ++cc) {
        if (!range_nonempty(cc, S, nctas)) continue;
        const int sl = cc * 2 + (cc == c0 ? 1 : 0);
        const float* ml = p.part_ml + (static_cast<int64_t>(sl) * p.H + qh) * 2;
        const float w = exp2f(__ldcg(ml) - M);
        L += __ldcg(ml + 1) * w;
        acc += __ldcg(p.part_o + (static_cast<int64_t>(sl) * p.H + qh) * kD + d) * w;
      }
      store_out<T>(out + qh * kD + d, acc / L);
    }
    __syncwarp();
    if (lane == 0) *counter = 0;
  }
}

// Workspace layout: [status: int32, padded to 256 B][counters: kMaxCounters
// int32, a fixed region so that calls with different B find it where the
// previous call left it zeroed][part_ml: B*splits*H*2 f32][part_o: B*splits*H*D f32]
constexpr int64_t kMaxCounters = lk::kDecodeMaxCounters;
constexpr size_t kHeadBytes = lk::kDecodeHeadBytes;
size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// ------------------------------------------------------------------------
// Streaming split decode (the default): one CTA per SM takes (sequence,
// split, head group) units, longest first, from the list decode_order_kernel
// writes, through a counter that kernel zeroes. The producer warp publishes
// each unit to the consumer warps through a 4-deep descriptor ring and keeps
// the TMA stage ring streaming across unit boundaries, so a unit's block-table
// reads and first loads overlap the previous unit's last stages: no CTA launch,
// barrier setup or pipeline refill per unit. Splits write (m, l, o) partials and
// the consumer warps of the last unit of a (sequence, head group) to finish
// merge them, as in the split kernel (weights in shared memory, float4 loads).
constexpr int kStreamUnits = 4;        // unit descriptor ring depth
constexpr int kStreamMergeMax = 4096;  // (query head, split) weights held in shared memory

template <typename T, int HPC, int NST>
__global__ void __launch_bounds__((HPC + 1) * 32, 1)
paged_decode_stream_kernel(const __grid_constant__ CUtensorMap kmap,
                           const __grid_constant__ CUtensorMap vmap, const DecodeParams p,
                           int num_entries) {
  using Shape = DecodeShape<HPC, NST>;
  constexpr int kCons = HPC * 32;  // consumer threads
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[NST];
  __shared__ __align__(8) uint64_t empty_bar[NST];
  __shared__ __align__(8) uint64_t unit_full[kStreamUnits];
  __shared__ __align__(8) uint64_t unit_empty[kStreamUnits];
  __shared__ int4 unit_ring[kStreamUnits];  // b, split, ctx, head group (b < 0: no more work)
  __shared__ float s_w[kStreamMergeMax];
  __shared__ int s_last;
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.G, groups = p.num_groups;
  const int spp = p.stages_per_split;
  const int cap = p.max_blocks * p.bs;
  const int total = num_entries * groups;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < NST; ++s) {
      lk::mbar_init(&full_bar[s], 1);
      lk::mbar_init(&empty_bar[s], HPC);
    }
#pragma unroll
    for (int s = 0; s < kStreamUnits; ++s) {
      lk::mbar_init(&unit_full[s], 1);
      lk::mbar_init(&unit_empty[s], HPC);
    }
    lk::fence_barrier_init();
  }
  __syncthreads();

  // Stages of a unit: [st0, st1) of the sequence's ceil(ctx / 16) stages.
  auto stage_range = [&](int ctx, int sp, int& st0, int& st1) {
    int c = ctx > cap ? cap : (ctx < 0 ? 0 : ctx);
    const int nst = (c + kTok - 1) / kTok;
    st0 = sp * spp;
    st1 = min(nst, st0 + spp);
  };

  if (warp == HPC) {
    // ------------------------------------------------------- producer ---
    if (lane == 0) {
      lk::prefetch_tensormap(&kmap);
      lk::prefetch_tensormap(&vmap);
    }
    const int64_t num_slots = p.num_blocks * p.bs;
    const int oob = static_cast<int>(num_slots < 0x7fffffffLL ? num_slots : 0x7fffffffLL);
    bool ok = true;
    int it = 0;
    for (int n = 0; ok; ++n) {
      int idx = 0;
      if (lane == 0) idx = atomicAdd(p.work, 1);
      idx = __shfl_sync(0xffffffffu, idx, 0);
      int4 u = make_int4(-1, 0, 0, 0);
      if (idx < total) {
        const int2 e = p.order[idx / groups];
        if (e.x >= 0) u = make_int4(e.x / p.num_splits, e.x % p.num_splits, e.y, idx % groups);
      }
      if (lane == 0) {
        const int s = n % kStreamUnits;
        if (lk::mbar_wait(&unit_empty[s], ((n / kStreamUnits) & 1) ^ 1)) {
          unit_ring[s] = u;
          lk::mbar_arrive(&unit_full[s]);
        } else {
          atomicOr(p.status, LK_STATUS_WAIT_TIMEOUT);
          ok = false;
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok || u.x < 0) break;
      int st0, st1;
      stage_range(u.z, u.y, st0, st1);
      const int32_t* bt = p.block_tables + static_cast<int64_t>(u.x) * p.bt_stride;
      const int h0 = u.w * HPC;
      auto lookup = [&](int st) -> int {
        if (st >= st1) return -1;
        const int pos = st * kTok;
        const int blk = __ldg(bt + pos / p.bs);
        if (blk < 0 || blk >= p.num_blocks) {
          atomicOr(p.status, LK_STATUS_BLOCK_OOB);
          return oob;  // past the end: TMA reads zeros
        }
        return blk * p.bs + (pos % p.bs);
      };
      int nxt = lookup(st0 + lane);
      for (int base = st0; base < st1 && ok; base += 32) {
        const int cur = nxt;
        nxt = lookup(base + 32 + lane);
        const int cnt = min(32, st1 - base);
        for (int i = 0; i < cnt; ++i, ++it) {
          const int slot = __shfl_sync(0xffffffffu, cur, i);
          if (lane == 0) {
            const int s = it % NST;
            if (!lk::mbar_wait(&empty_bar[s], ((it / NST) & 1) ^ 1)) {
              atomicOr(p.status, LK_STATUS_WAIT_TIMEOUT);
              ok = false;
            } else {
              lk::mbar_arrive_expect_tx(&full_bar[s], Shape::kStageBytes);
              uint8_t* dst = smem + s * Shape::kStageBytes;
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
    }
    return;
  }

  // ----------------------------------------------------------- consumers ---
  const int g = lane >> 2, c = lane & 3;
  const float sl2 = p.scale_log2;
  bool ok = true;
  int it = 0;
  for (int n = 0;; ++n) {
    int4 u = make_int4(-1, 0, 0, 0);
    {
      const int s = n % kStreamUnits;
      if (ok && lk::mbar_wait(&unit_full[s], (n / kStreamUnits) & 1)) {
        u = unit_ring[s];
      } else {
        ok = false;
      }
      __syncwarp();
      if (lane == 0) lk::mbar_arrive(&unit_empty[s]);
    }
    // All consumer warps leave together (a warp that left alone would strand
    // the others at the merge's named barriers).
    ok = lk::named_sync_and(1, kCons, ok);
    if (!ok || u.x < 0) break;
    const int b = u.x, sp = u.y, hg = u.w;
    if (u.z > cap && sp == 0 && threadIdx.x == 0) atomicOr(p.status, LK_STATUS_CTX_OOB);
    int st0, st1;
    stage_range(u.z, sp, st0, st1);
    const int nst = (min(max(u.z, 0), cap) + kTok - 1) / kTok;
    const int nsp = nst == 0 ? 1 : (nst + spp - 1) / spp;
    T* out = static_cast<T*>(p.out) + static_cast<int64_t>(b) * p.out_stride;
    const int kvh = hg * HPC + warp;
    const int qh0 = kvh * G;
    if (nst == 0) {
      // softmax over an all -inf row is NaN in the reference; reproduce it.
      for (int i = lane; i < G * kD; i += 32)
        store_out<T>(out + qh0 * kD + i, __int_as_float(0x7fc00000));
      continue;
    }
    uint32_t qb[8][2];
    {
      const T* qrow = static_cast<const T*>(p.q) + static_cast<int64_t>(b) * p.q_stride +
                      static_cast<int64_t>(qh0 + g) * kD;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        qb[ks][0] = g < G ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 2 * c) : 0u;
        qb[ks][1] = g < G ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 8 + 2 * c) : 0u;
      }
    }
    DecodeState st;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) st.o[mt][0] = st.o[mt][1] = st.o[mt][2] = st.o[mt][3] = 0.f;
    st.m0 = st.m1 = -INFINITY;
    st.l0 = st.l1 = 0.f;
    const uint32_t wbase = lk::smem_u32(smem) + warp * (kTok * 128);
    for (int t = st0; t < st1; ++t, ++it) {
      const int s = it % NST;
      if (ok && !lk::mbar_wait(&full_bar[s], (it / NST) & 1)) {
        if (lane == 0) atomicOr(p.status, LK_STATUS_WAIT_TIMEOUT);
        ok = false;
      }
      if (ok) {
        const uint32_t kb = wbase + s * Shape::kStageBytes;
        decode_stage<T, Shape::kBoxBytes>(st, qb, kb, kb + 2 * Shape::kBoxBytes, t * kTok, u.z,
                                          sl2, lane);
      }
      __syncwarp();
      if (lane == 0) lk::mbar_arrive(&empty_bar[s]);
    }
    float l0 = st.l0, l1 = st.l1;
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
          store_out<T>(out + (qh0 + n0) * kD + d, st.o[mt][0] * r0);
          store_out<T>(out + (qh0 + n0) * kD + d + 8, st.o[mt][2] * r0);
        }
        if (n1 < G) {
          store_out<T>(out + (qh0 + n1) * kD + d, st.o[mt][1] * r1);
          store_out<T>(out + (qh0 + n1) * kD + d + 8, st.o[mt][3] * r1);
        }
      }
      continue;
    }
    const int64_t prow = (static_cast<int64_t>(b) * p.num_splits + sp) * p.H;
    float* po = p.part_o + prow * kD;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      const int d = mt * 16 + g;
      if (n0 < G) {
        po[(qh0 + n0) * kD + d] = st.o[mt][0];
        po[(qh0 + n0) * kD + d + 8] = st.o[mt][2];
      }
      if (n1 < G) {
        po[(qh0 + n1) * kD + d] = st.o[mt][1];
        po[(qh0 + n1) * kD + d + 8] = st.o[mt][3];
      }
    }
    if (g == 0) {
      float* pml = p.part_ml + prow * 2;
      if (n0 < G) {
        pml[(qh0 + n0) * 2] = st.m0;
        pml[(qh0 + n0) * 2 + 1] = l0;
      }
      if (n1 < G) {
        pml[(qh0 + n1) * 2] = st.m1;
        pml[(qh0 + n1) * 2 + 1] = l1;
      }
    }
    // Last unit of this (sequence, head group) to finish merges the splits.
    __threadfence();
    lk::named_sync(1, kCons);
    if (threadIdx.x == 0) {
      const int prev = atomicAdd(p.counters + b * groups + hg, 1);
      s_last = (prev == nsp - 1);
    }
    lk::named_sync(1, kCons);
    if (!s_last) continue;
    __threadfence();
    const int nq = HPC * G, qbase = hg * nq;
    const int64_t rowb = static_cast<int64_t>(b) * p.num_splits;
    if (nq * nsp <= kStreamMergeMax) {
      for (int q = threadIdx.x; q < nq; q += kCons) {
        const float* ml = p.part_ml + (rowb * p.H + qbase + q) * 2;
        float M = -INFINITY;
        for (int s2 = 0; s2 < nsp; ++s2) M = fmaxf(M, __ldcg(ml + s2 * p.H * 2));
        float L = 0.f;
        for (int s2 = 0; s2 < nsp; ++s2) {
          const float e = exp2f(__ldcg(ml + s2 * p.H * 2) - M);
          s_w[q * nsp + s2] = e;
          L += __ldcg(ml + s2 * p.H * 2 + 1) * e;
        }
        const float inv = 1.f / L;
        for (int s2 = 0; s2 < nsp; ++s2) s_w[q * nsp + s2] *= inv;
      }
      lk::named_sync(1, kCons);
      constexpr int kU = 4;
      const int n4 = nq * kD / 4;
      const float4* po4 = reinterpret_cast<const float4*>(p.part_o + (rowb * p.H + qbase) * kD);
      const int64_t sstride4 = static_cast<int64_t>(p.H) * kD / 4;
      for (int i0 = threadIdx.x; i0 < n4; i0 += kU * kCons) {
        float4 acc[kU];
#pragma unroll
        for (int k = 0; k < kU; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
        for (int s2 = 0; s2 < nsp; ++s2) {
          float4 v[kU];
#pragma unroll
          for (int k = 0; k < kU; ++k) {
            const int i = i0 + k * kCons;
            v[k] = i < n4 ? __ldcg(po4 + s2 * sstride4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
          }
#pragma unroll
          for (int k = 0; k < kU; ++k) {
            const int i = i0 + k * kCons;
            const float wt = i < n4 ? s_w[(i * 4 / kD) * nsp + s2] : 0.f;
            acc[k].x += v[k].x * wt;
            acc[k].y += v[k].y * wt;
            acc[k].z += v[k].z * wt;
            acc[k].w += v[k].w * wt;
          }
        }
#pragma unroll
        for (int k = 0; k < kU; ++k) {
          const int i = i0 + k * kCons;
          if (i < n4) {
            T* o = out + qbase * kD + i * 4;
            store_out<T>(o, acc[k].x);
            store_out<T>(o + 1, acc[k].y);
            store_out<T>(o + 2, acc[k].z);
            store_out<T>(o + 3, acc[k].w);
          }
        }
      }
      lk::named_sync(1, kCons);  // s_w is rewritten by the next merge
    } else {
      for (int i = threadIdx.x; i < nq * kD; i += kCons) {
        const int qh = qbase + i / kD, d = i % kD;
        float M = -INFINITY;
        for (int s2 = 0; s2 < nsp; ++s2)
          M = fmaxf(M, __ldcg(p.part_ml + ((rowb + s2) * p.H + qh) * 2));
        float L = 0.f, acc = 0.f;
        for (int s2 = 0; s2 < nsp; ++s2) {
          const float* ml = p.part_ml + ((rowb + s2) * p.H + qh) * 2;
          const float wt = exp2f(__ldcg(ml) - M);
          L += __ldcg(ml + 1) * wt;
          acc += __ldcg(p.part_o + ((rowb + s2) * p.H + qh) * kD + d) * wt;
        }
        store_out<T>(out + qh * kD + d, acc / L);
      }
    }
    if (threadIdx.x == 0) p.counters[b * groups + hg] = 0;
  }
}

// Streaming persistent split kernel instead of one CTA per unit
// (LITEKERN_DECODE_STREAM, read once; 1 = on).
bool stream_units() {
  static int v = [] {
    const char* e = getenv("LITEKERN_DECODE_STREAM");
    return e && atoi(e) == 1 ? 1 : 0;
  }();
  return v != 0;
}

// KV heads per CTA: the largest of 8, 4, 2, 1 that divides H_kv, capped by the
// LITEKERN_DECODE_HEADS_PER_CTA environment variable (read once; a tuning knob).
int heads_cap() {
  static int cap = [] {
    const char* e = getenv("LITEKERN_DECODE_HEADS_PER_CTA");
    const int v = e ? atoi(e) : 8;
    return (v == 1 || v == 2 || v == 4 || v == 8) ? v : 8;
  }();
  return cap;
}

int heads_per_cta(int H_kv) {
  const int cap = heads_cap();
  if (cap < 8) {
    for (int h = cap; h >= 1; h >>= 1)
      if (H_kv % h == 0) return h;
  }
  if (H_kv % 8 == 0) return 8;
  if (H_kv % 4 == 0) return 4;
  if (H_kv % 2 == 0) return 2;
  return 1;
}

template <typename T, int HPC, int NST>
int launch_decode(const CUtensorMap& km, const CUtensorMap& vm, const DecodeParams& p, int B,
                  cudaStream_t s, bool order_done = false) {
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
  if (p.order != nullptr && !order_done) {
    // Both launches may start before the kernel ahead of them in the stream
    // ends (its launch latency and the split kernel's prologue overlap the KV
    // store and the ordering); each waits for its predecessor before reading.
    if (lk::launch_after_previous(decode_order_kernel, dim3(1), dim3(1024), 0, s, p.context_lens,
                                  B, p.max_blocks * p.bs, p.stages_per_split, p.num_splits,
                                  const_cast<int2*>(p.order), p.work, p.first_stage,
                                  static_cast<int*>(nullptr)) != cudaSuccess)
      return LK_ERR_CUDA;
  }
  if (p.order != nullptr && stream_units() && p.part_offset == 0) {
    static int configured_s[64] = {0};
    if (dev >= 0 && dev < 64 && !configured_s[dev]) {
      if (cudaFuncSetAttribute(paged_decode_stream_kernel<T, HPC, NST>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               Shape::kSmem) != cudaSuccess)
        return LK_ERR_CUDA;
      configured_s[dev] = 1;
    }
    const int64_t units = static_cast<int64_t>(B) * p.num_splits * p.num_groups;
    const int grid = static_cast<int>(units < lk::num_sms() ? units : lk::num_sms());
    paged_decode_stream_kernel<T, HPC, NST>
        <<<grid, Shape::kThreads, Shape::kSmem, s>>>(km, vm, p, B * p.num_splits);
    return lk::check_launch();
  }
  dim3 grid(B * p.num_splits, p.num_groups);
  if (lk::launch_after_previous(paged_decode_kernel<T, HPC, NST>, grid, dim3(Shape::kThreads),
                                Shape::kSmem, s, km, vm, p) != cudaSuccess)
    return LK_ERR_CUDA;
  return lk::check_launch();
}

template <typename T>
int dispatch_decode(int hpc, const CUtensorMap& km, const CUtensorMap& vm, const DecodeParams& p,
                    int B, cudaStream_t s, bool order_done = false) {
  switch (hpc) {
    case 8: return launch_decode<T, 8, 3>(km, vm, p, B, s, order_done);
    case 4: return launch_decode<T, 4, 6>(km, vm, p, B, s, order_done);
    case 2: return launch_decode<T, 2, 8>(km, vm, p, B, s, order_done);
    default: return launch_decode<T, 1, 8>(km, vm, p, B, s, order_done);
  }
}

template <typename T, int HPC, int NST>
int launch_persistent(const CUtensorMap& km, const CUtensorMap& vm, const DecodeParams& p,
                      int num_units, int grid, cudaStream_t s) {
  using Shape = DecodeShape<HPC, NST>;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(paged_decode_persistent_kernel<T, HPC, NST>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Shape::kSmem) != cudaSuccess)
      return LK_ERR_CUDA;
    configured[dev] = 1;
  }
  paged_decode_persistent_kernel<T, HPC, NST>
      <<<grid, Shape::kThreads, Shape::kSmem, s>>>(km, vm, p, num_units);
  return lk::check_launch();
}

template <typename T>
int dispatch_persistent(int hpc, const CUtensorMap& km, const CUtensorMap& vm,
                        const DecodeParams& p, int num_units, int grid, cudaStream_t s) {
  switch (hpc) {
    case 8: return launch_persistent<T, 8, 3>(km, vm, p, num_units, grid, s);
    case 4: return launch_persistent<T, 4, 6>(km, vm, p, num_units, grid, s);
    case 2: return launch_persistent<T, 2, 12>(km, vm, p, num_units, grid, s);
    default: return launch_persistent<T, 1, 24>(km, vm, p, num_units, grid, s);
  }
}

// Stages the producers prefetch into L2 ahead of the shared-memory ring;
// LITEKERN_DECODE_PREFETCH (read once, 0..31) overrides the default.
int prefetch_distance() {
  static int d = [] {
    const char* e = getenv("LITEKERN_DECODE_PREFETCH");
    int v = e ? atoi(e) : 0;
    return v < 0 ? 0 : (v > 31 ? 31 : v);
  }();
  return d;
}

// Longest-first launch order for the split kernel (LITEKERN_DECODE_ORDER=0
// launches units in sequence order without the ordering kernel; read once).
bool order_units() {
  static int v = [] {
    const char* e = getenv("LITEKERN_DECODE_ORDER");
    return e && atoi(e) == 0 ? 0 : 1;
  }();
  return v != 0;
}

// CTAs of the persistent kernel: one per SM (its shared-memory ring takes the SM).
// LITEKERN_DECODE_GRID (read once) overrides it, for tuning.
int persistent_grid() {
  static int override_grid = [] {
    const char* e = getenv("LITEKERN_DECODE_GRID");
    return e ? atoi(e) : 0;
  }();
  return override_grid > 0 ? override_grid : lk::num_sms();
}

}  // namespace

extern "C" int lk_paged_decode_num_splits(int32_t B, int32_t H_kv, int32_t max_blocks_per_seq,
                                          int32_t block_size) {
  if (B <= 0 || H_kv <= 0 || max_blocks_per_seq <= 0 || block_size <= 0) return 1;
  const int groups = H_kv / heads_per_cta(H_kv);
  const int64_t max_stages = (static_cast<int64_t>(max_blocks_per_seq) * block_size + 15) / 16;
  const int64_t units = static_cast<int64_t>(B) * groups;
  // Measured on B200 (config 2: B=256, contexts <= 4096; config 5: B=8..64,
  // contexts 32K-128K), with units launched longest first: fewer, longer
  // CTAs stream faster than many short ones. A split holds at least 128
  // stages (2048 tokens) and long contexts are cut into about 24 splits.
  (void)units;
  const int64_t spp = std::max<int64_t>(128, (max_stages + 23) / 24);
  int64_t splits = (max_stages + spp - 1) / spp;
  splits = std::max<int64_t>(1, std::min<int64_t>(splits, max_stages));
  return static_cast<int>(std::min<int64_t>(splits, 65535));
}

extern "C" size_t lk_paged_decode_workspace_bytes(int32_t B, int32_t H, int32_t H_kv, int32_t D,
                                                  int32_t num_splits) {
  if (B <= 0 || H <= 0 || H_kv <= 0 || D <= 0) return 0;
  const int groups = H_kv / heads_per_cta(H_kv);
  (void)groups;
  size_t bytes = kHeadBytes;
  if (num_splits < 0) {  // persistent kernel: two partial slots per CTA
    const size_t slots = 2 * static_cast<size_t>(persistent_grid());
    bytes += align256(slots * H * 2 * 4);
    bytes += align256(slots * H * D * 4);
  } else {
    if (num_splits > 1) {
      bytes += align256(static_cast<size_t>(B) * num_splits * H * 2 * 4);
      bytes += align256(static_cast<size_t>(B) * num_splits * H * D * 4);
    }
    bytes += align256(static_cast<size_t>(B) * std::max(num_splits, 1) * sizeof(int2));
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
  if (B > 65535 || max_blocks_per_seq == 0) return LK_ERR_INVALID_ARG;
  if ((dtype != LK_DTYPE_BF16 && dtype != LK_DTYPE_F16) || D != kD || block_size % kTok != 0 ||
      H / H_kv > 8) {
    // Shapes the split kernel does not take (fp32 caches, other head dims or
    // block sizes, G > 8) run the generic CUDA-core kernel; its status bits
    // go to the workspace's status word like the split kernel's, and the rest
    // of the workspace holds its split-KV partials when there is room.
    return lk::generic_decode(out, out_token_stride, q, q_token_stride, k_cache, v_cache,
                              num_blocks, block_tables, block_table_stride, context_lens, B, H,
                              H_kv, D, block_size, max_blocks_per_seq, scale, dtype, workspace,
                              workspace_bytes, stream);
  }
  if (static_cast<int64_t>(B) * H_kv > kMaxCounters) return LK_ERR_UNSUPPORTED;
  if (num_blocks * block_size > 0x7fffffffLL) return LK_ERR_UNSUPPORTED;
  if (((reinterpret_cast<uintptr_t>(q) & 3u) != 0) || (q_token_stride & 1) != 0)
    return LK_ERR_ALIGNMENT;
  if (num_splits == 0)
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
  p.prefetch = prefetch_distance();
  p.first_stage = 0;
  p.part_offset = 0;
  const bool persistent = num_splits < 0;
  p.num_splits = persistent ? 1 : num_splits;
  p.stages_per_split = static_cast<int>((max_stages + p.num_splits - 1) / p.num_splits);
  p.num_groups = H_kv / hpc;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const size_t cnt_bytes = kHeadBytes;
  p.status = reinterpret_cast<int32_t*>(ws);
  p.counters = reinterpret_cast<int32_t*>(ws + 256);
  p.part_ml = reinterpret_cast<float*>(ws + cnt_bytes);
  const size_t ml_rows = persistent ? 2 * static_cast<size_t>(persistent_grid())
                                    : static_cast<size_t>(B) * num_splits;
  p.part_o = reinterpret_cast<float*>(ws + cnt_bytes + align256(ml_rows * H * 2 * 4));
  const size_t part_bytes = (persistent || num_splits > 1)
                                ? align256(ml_rows * H * 2 * 4) + align256(ml_rows * H * kD * 4)
                                : 0;
  p.order = reinterpret_cast<const int2*>(ws + cnt_bytes + part_bytes);
  p.work = reinterpret_cast<int*>(ws + 64);  // in the 256-byte status header
  if (!order_units()) p.order = nullptr;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (persistent) {
    const int units = B * p.num_groups;
    if (dtype == LK_DTYPE_BF16)
      return dispatch_persistent<__nv_bfloat16>(hpc, km, vm, p, units, persistent_grid(), s);
    return dispatch_persistent<__half>(hpc, km, vm, p, units, persistent_grid(), s);
  }
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

// --------------------------------------------------------- shared prefix ---
namespace {

// Plan of a shared-prefix decode: key ranges of the prefix for the tensor-core
// pass, and splits of the suffix for the decode kernel.
struct PrefixPlan {
  int prefix_split, ranges;  // prefix keys per range, number of ranges
  int spp, suffix_splits;    // suffix stages per split, splits per row
  int part_splits;           // partial slots per row: ranges + suffix splits
};

PrefixPlan prefix_plan(int B, int H_kv, int max_blocks, int block_size, int prefix_tokens, int G) {
  PrefixPlan pl;
  const int sms = lk::num_sms();
  const int rows_per_item = 256 / G;  // query rows of one prefix work item
  const int items_per_range = ((B + rows_per_item - 1) / rows_per_item) * H_kv;
  const int tiles = (prefix_tokens + 127) / 128;
  // About half the SMs: the suffix decode runs beside the prefix kernel on the
  // rest (measured on config 4, decode step: 8 ranges on 128 SMs 54.8 us, 4
  // on 64 SMs 50.7, 2 on 32 SMs 61.6).
  int ranges = sms / (2 * (items_per_range > 0 ? items_per_range : 1));
  static const int ranges_env = [] {
    const char* e = getenv("LITEKERN_PREFIX_RANGES");
    return e ? atoi(e) : 0;
  }();
  if (ranges_env > 0) ranges = ranges_env;
  ranges = ranges < 1 ? 1 : (ranges > tiles ? tiles : ranges);
  pl.prefix_split = ((tiles + ranges - 1) / ranges) * 128;
  pl.ranges = (prefix_tokens + pl.prefix_split - 1) / pl.prefix_split;
  const int64_t max_stages = (static_cast<int64_t>(max_blocks) * block_size + 15) / 16;
  const int64_t suffix = max_stages - prefix_tokens / 16;
  // About one wave of suffix units over the batch (measured on config 4: one
  // 17-stage split per row beats 3 splits of <= 8 stages, whose ramps and
  // extra partials cost more than the parallelism gains).
  int want = sms / B;
  if (want < 1) want = 1;
  int64_t spp = suffix > 0 ? (suffix + want - 1) / want : 1;
  if (spp < 8) spp = 8;
  static const int spp_env = [] {
    const char* e = getenv("LITEKERN_PREFIX_SPP");
    return e ? atoi(e) : 0;
  }();
  if (spp_env > 0) spp = spp_env;
  pl.spp = static_cast<int>(spp);
  pl.suffix_splits = suffix > 0 ? static_cast<int>((suffix + spp - 1) / spp) : 1;
  pl.part_splits = pl.ranges + pl.suffix_splits;
  return pl;
}

}  // namespace

extern "C" size_t lk_paged_decode_shared_prefix_workspace_bytes(
    int32_t B, int32_t H, int32_t H_kv, int32_t D, int32_t max_blocks_per_seq,
    int32_t block_size, int32_t prefix_tokens) {
  if (B <= 0 || H <= 0 || H_kv <= 0 || D <= 0 || H % H_kv != 0 || block_size <= 0 ||
      prefix_tokens <= 0 || max_blocks_per_seq <= 0)
    return 0;
  const PrefixPlan pl =
      prefix_plan(B, H_kv, max_blocks_per_seq, block_size, prefix_tokens, H / H_kv);
  const size_t rows = static_cast<size_t>(B) * pl.part_splits;
  return kHeadBytes + align256(rows * H * 2 * 4) + align256(rows * H * D * 4) +
         align256(rows * sizeof(int2));
}

extern "C" int lk_paged_decode_shared_prefix(
    void* out, int64_t out_token_stride, const void* q, int64_t q_token_stride,
    const void* k_cache, const void* v_cache, int64_t num_blocks, const int32_t* block_tables,
    int64_t block_table_stride, const int32_t* context_lens, int32_t B, int32_t H, int32_t H_kv,
    int32_t D, int32_t block_size, int32_t max_blocks_per_seq, float scale,
    int32_t prefix_tokens, void* workspace, size_t workspace_bytes, int32_t dtype, void* stream) {
  if (B < 0 || H <= 0 || H_kv <= 0 || H % H_kv != 0 || num_blocks <= 0 || block_size <= 0 ||
      max_blocks_per_seq <= 0)
    return LK_ERR_INVALID_ARG;
  if (B == 0) return LK_OK;
  if (!out || !q || !k_cache || !v_cache || !block_tables || !context_lens)
    return LK_ERR_INVALID_ARG;
  if (dtype != LK_DTYPE_BF16 && dtype != LK_DTYPE_F16) return LK_ERR_UNSUPPORTED;
  if (D != kD || block_size % kTok != 0 || H / H_kv > 8) return LK_ERR_UNSUPPORTED;
  if (prefix_tokens <= 0 || prefix_tokens % block_size != 0 ||
      prefix_tokens > static_cast<int64_t>(max_blocks_per_seq) * block_size)
    return LK_ERR_INVALID_ARG;
  if (B > 65535 || static_cast<int64_t>(B) * H_kv > kMaxCounters) return LK_ERR_UNSUPPORTED;
  if (num_blocks * block_size > 0x7fffffffLL) return LK_ERR_UNSUPPORTED;
  if (((reinterpret_cast<uintptr_t>(q) & 3u) != 0) || (q_token_stride & 1) != 0)
    return LK_ERR_ALIGNMENT;
  const size_t need = lk_paged_decode_shared_prefix_workspace_bytes(
      B, H, H_kv, D, max_blocks_per_seq, block_size, prefix_tokens);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return LK_ERR_WORKSPACE;
  const PrefixPlan pl =
      prefix_plan(B, H_kv, max_blocks_per_seq, block_size, prefix_tokens, H / H_kv);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const size_t rows = static_cast<size_t>(B) * pl.part_splits;
  float* part_ml = reinterpret_cast<float*>(ws + kHeadBytes);
  float* part_o = reinterpret_cast<float*>(ws + kHeadBytes + align256(rows * H * 2 * 4));
  int2* order = reinterpret_cast<int2*>(ws + kHeadBytes + align256(rows * H * 2 * 4) +
                                        align256(rows * H * D * 4));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t* status = reinterpret_cast<int32_t*>(ws);

  // 1. the suffix units' launch order (also zeroes both kernels' work counters)
  int* prefix_counter = reinterpret_cast<int*>(ws + 128);  // in the status header
  decode_order_kernel<<<1, 1024, 0, s>>>(context_lens, B, max_blocks_per_seq * block_size,
                                         pl.spp, pl.part_splits, order,
                                         reinterpret_cast<int*>(ws + 64), prefix_tokens / kTok,
                                         prefix_counter);
  int rc = lk::check_launch();
  if (rc != LK_OK) return rc;
  // 2. the prefix, once for all rows, on the tensor cores: partial slots [0, ranges)
  rc = lk::prefix_attention(q, q_token_stride, k_cache, v_cache, num_blocks, block_tables, B, H,
                            H_kv, block_size, prefix_tokens, pl.prefix_split, pl.ranges, scale,
                            part_ml, part_o, pl.part_splits, dtype, status, prefix_counter, s);
  if (rc != LK_OK) return rc;

  // 3. each row's own suffix on the split decode kernel, merged with the prefix
  const int hpc = heads_per_cta(H_kv);
  const int64_t num_slots = num_blocks * block_size;
  CUtensorMap km, vm;
  rc = lk::get_kv_tensor_map(&km, k_cache, num_slots, H_kv, D, dtype, kTok, hpc);
  if (rc != LK_OK) return rc;
  rc = lk::get_kv_tensor_map(&vm, v_cache, num_slots, H_kv, D, dtype, kTok, hpc);
  if (rc != LK_OK) return rc;
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
  p.prefetch = 0;
  p.stages_per_split = pl.spp;
  p.num_splits = pl.part_splits;  // partial slots per row (and the unit encoding)
  p.num_groups = H_kv / hpc;
  p.status = status;
  p.counters = reinterpret_cast<int32_t*>(ws + 256);
  p.part_ml = part_ml;
  p.part_o = part_o;
  p.order = order;
  p.work = reinterpret_cast<int*>(ws + 64);
  p.first_stage = prefix_tokens / kTok;
  p.part_offset = pl.ranges;
  if (dtype == LK_DTYPE_BF16) return dispatch_decode<__nv_bfloat16>(hpc, km, vm, p, B, s, true);
  return dispatch_decode<__half>(hpc, km, vm, p, B, s, true);
}
