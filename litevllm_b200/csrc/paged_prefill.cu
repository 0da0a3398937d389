// Chunked-prefill attention over prior paged context.
//
// The reference only has Attention._prefill (litevllm/layers/attention.py:141-151):
// causal SDPA over the new tokens of one sequence, with query head h reading
// KV head h / G (repeat_interleave, :147-149) and the default 1/sqrt(D) scale.
// This kernel generalises it to a chunk that sits on top of `prior` tokens
// already in the paged cache: query i (absolute position prior + i) attends
// keys j <= prior + i, gathered through the block table exactly as
// _decode_fast gathers them (attention.py:105-119). With prior = 0 and
// contiguous keys it is _prefill.
//
// B200 design (flash-attention style, tensor cores for QK^T and PV):
//  * CTA = (128-row query tile, KV head, sequence). The 128 rows are
//    BQ = 128 / G positions x the G query heads of the KV head, so each K/V
//    tile read from HBM serves all G heads. 8 consumer warps own 16 rows each
//    (warp w: query head w % G, positions (w / G) * 16 ..); a 9th warp issues
//    TMA loads of 64-token K and V tiles (four 16-token boxes each, gathered
//    through the block table) into a 3-stage shared-memory ring.
//  * Per tile each warp runs S = Q K^T (16 x 64) and O += P V (16 x 128) with
//    mma.sync m16n8k16, fp32 accumulation, and an online softmax in registers;
//    the S accumulators are re-packed as the A operand of PV without shuffles.
#include "lk_common.cuh"
#include "lk_host.h"

#include <stdlib.h>

#include <mutex>
#include <string>
#include <vector>
#include <type_traits>

namespace {

constexpr int kD = 128;
constexpr int kRows = 128;        // query rows (position x head) per CTA
constexpr int kKT = 64;           // keys per tile
constexpr int kNST = 3;           // pipeline stages
constexpr int kCW = 8;            // consumer warps
constexpr int kThreads = (kCW + 1) * 32;
constexpr int kBoxBytes = 16 * 128;                  // 16 slots x 64 values (one head)
constexpr int kHalfBytes = kKT * 128;                // 64 tokens x 64 values
constexpr int kTileBytes = 2 * kHalfBytes;           // one of K or V, both d halves
constexpr int kStageBytes = 2 * kTileBytes;          // K and V
constexpr int kSmem = kNST * kStageBytes + 1024;

struct PrefillParams {
  void* out;
  const void* q;
  int64_t q_stride;     // elements between tokens of q (out is [T, H, D] contiguous)
  const int32_t* block_tables;  // NULL: contiguous keys, slot = cu_seqlens_q[b] + pos
  int64_t bt_stride;
  const int32_t* cu_seqlens_q;
  const int32_t* context_lens;  // may be NULL in contiguous mode (prior = 0)
  int64_t num_slots;
  int64_t num_blocks;
  int H, G, bs, BQ;
  float scale_log2;
  int32_t* status;
  int num_seqs, H_kv, nqt;  // persistent ping-pong kernel: work-item grid
  int* sched;               // its work-item counter (zeroed per launch)
  // Work units of the ping-pong kernel, most key tiles first (NULL: tile-major
  // order over nqt x num_seqs pairs). Unit = pair | piece << 14 | split << 16,
  // pair = sequence * nqt + query tile; piece 0 = all key tiles, 1 / 2 = the
  // first / second half of them (a key-split pair, merged through split_*).
  const int* order;
  const int* units_count;  // number of units in order
  int* split_cnt;          // [split items][softmax warp][arrivals, ready]
  float* split_ml;         // [split items][piece][256 rows][2] (m, l)
  float* split_o;          // [split items][piece][256 rows][D] unnormalised o
  // Shared-prefix mode (decode rows against a prefix every row shares): the
  // B query rows are one "chunk" (q_len = prefix_rows), keys [0, prefix_len)
  // through block-table row 0 in key ranges of prefix_split tokens (num_seqs
  // ranges), no causal mask; (m, l, o) partials go to part_ml / part_o at
  // split slot = range index, in rows of part_splits slots.
  int prefix_rows, prefix_len, prefix_split, part_splits;
  float* part_ml;  // [rows][part_splits][H][2]
  float* part_o;   // [rows][part_splits][H][D]
};

template <typename T>
LK_DEVINL void store2(T* p, float a, float b) {
  *reinterpret_cast<uint32_t*>(p) = lk::pack2<T>(a, b);
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
paged_prefill_kernel(const __grid_constant__ CUtensorMap kmap,
                     const __grid_constant__ CUtensorMap vmap, const PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kNST];
  __shared__ __align__(8) uint64_t empty_bar[kNST];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

  const int qt = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.G, BQ = p.BQ;
  const int q_start = p.cu_seqlens_q[b];
  const int q_len = p.cu_seqlens_q[b + 1] - q_start;
  const int pos0 = qt * BQ;
  if (pos0 >= q_len) return;
  int prior = 0;
  if (p.block_tables != nullptr && p.context_lens != nullptr) {
    prior = p.context_lens[b] - q_len;
    if (prior < 0) {
      if (threadIdx.x == 0 && p.status) atomicOr(p.status, LK_STATUS_CTX_OOB);
      prior = 0;
    }
  }
  const int kv_end = prior + min(q_len, pos0 + BQ);  // keys [0, kv_end) feed this tile
  const int ntiles = (kv_end + kKT - 1) / kKT;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < kNST; ++s) {
      lk::mbar_init(&full_bar[s], 1);
      lk::mbar_init(&empty_bar[s], kCW);
    }
    lk::fence_barrier_init();
  }
  __syncthreads();

  if (warp == kCW) {
    // ------------------------------------------------------- producer ---
    if (lane == 0) {
      lk::prefetch_tensormap(&kmap);
      lk::prefetch_tensormap(&vmap);
      const int32_t* bt =
          p.block_tables ? p.block_tables + static_cast<int64_t>(b) * p.bt_stride : nullptr;
      const int oob = static_cast<int>(p.num_slots < 0x7fffffffLL ? p.num_slots : 0x7fffffffLL);
      for (int kt = 0; kt < ntiles; ++kt) {
        const int s = kt % kNST;
        if (!lk::mbar_wait(&empty_bar[s], ((kt / kNST) & 1) ^ 1)) {
          if (p.status) atomicOr(p.status, LK_STATUS_WAIT_TIMEOUT);
          break;
        }
        lk::mbar_arrive_expect_tx(&full_bar[s], kStageBytes);
        uint8_t* dst = smem + s * kStageBytes;
#pragma unroll
        for (int tb = 0; tb < 4; ++tb) {
          const int tok = kt * kKT + tb * 16;
          int slot = oob;  // boxes past the needed keys read zeros
          if (tok < kv_end) {
            if (bt) {
              const int blk = bt[tok / p.bs];
              if (blk < 0 || blk >= p.num_blocks) {
                if (p.status) atomicOr(p.status, LK_STATUS_BLOCK_OOB);
              } else {
                slot = blk * p.bs + tok % p.bs;
              }
            } else {
              slot = q_start + tok;
            }
          }
#pragma unroll
          for (int dh = 0; dh < 2; ++dh) {
            lk::tma_load_3d(dst + dh * kHalfBytes + tb * kBoxBytes, &kmap, &full_bar[s], dh * 64,
                            slot, kvh);
            lk::tma_load_3d(dst + kTileBytes + dh * kHalfBytes + tb * kBoxBytes, &vmap,
                            &full_bar[s], dh * 64, slot, kvh);
          }
        }
      }
    }
    return;
  }

  // --------------------------------------------------------- consumers ---
  const int g = lane >> 2, c = lane & 3;
  const int qhead = kvh * G + warp % G;
  const int prow = pos0 + (warp / G) * 16;  // first position of this warp's 16 rows
  const int r0 = prow + g, r1 = prow + g + 8;
  const int H = p.H;

  uint32_t qa[8][4];
  {
    const T* base = static_cast<const T*>(p.q) + static_cast<int64_t>(qhead) * kD;
    const T* q0 = base + static_cast<int64_t>(q_start + r0) * p.q_stride;
    const T* q1 = base + static_cast<int64_t>(q_start + r1) * p.q_stride;
    const bool v0 = r0 < q_len, v1 = r1 < q_len;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int k0 = ks * 16 + 2 * c;
      qa[ks][0] = v0 ? *reinterpret_cast<const uint32_t*>(q0 + k0) : 0u;
      qa[ks][1] = v1 ? *reinterpret_cast<const uint32_t*>(q1 + k0) : 0u;
      qa[ks][2] = v0 ? *reinterpret_cast<const uint32_t*>(q0 + k0 + 8) : 0u;
      qa[ks][3] = v1 ? *reinterpret_cast<const uint32_t*>(q1 + k0 + 8) : 0u;
    }
  }
  float o[16][4];
#pragma unroll
  for (int dt = 0; dt < 16; ++dt) o[dt][0] = o[dt][1] = o[dt][2] = o[dt][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const float sl2 = p.scale_log2;
  // Keys this warp can see: up to prior + (its last valid row).
  const int warp_kv_end = prior + min(prow + 15, q_len - 1) + 1;
  const uint32_t sbase = lk::smem_u32(smem);
  const int j = lane >> 3;

  for (int kt = 0; kt < ntiles; ++kt) {
    const int s = kt % kNST;
    if (!lk::mbar_wait(&full_bar[s], (kt / kNST) & 1)) {
      if (lane == 0 && p.status) atomicOr(p.status, LK_STATUS_WAIT_TIMEOUT);
      break;
    }
    if (kt * kKT < warp_kv_end) {
      const uint32_t kb = sbase + s * kStageBytes;
      const uint32_t vb = kb + kTileBytes;
      float sc[8][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
        for (int nt = 0; nt < 8; nt += 2) {
          const uint32_t tok = (nt + (j >> 1)) * 8 + (lane & 7);
          const uint32_t chunk = ((ks & 3) << 1) + (j & 1);
          uint32_t r[4];
          lk::ldsm_x4(kb + (ks >> 2) * kHalfBytes + lk::swz128(tok, chunk), r[0], r[1], r[2],
                      r[3]);
          lk::mma16816<T>(sc[nt], qa[ks], r[0], r[1]);
          lk::mma16816<T>(sc[nt + 1], qa[ks], r[2], r[3]);
        }
      }
      // causal mask: key j visible to row i iff j <= prior + i
      const bool need_mask = kt * kKT + kKT - 1 > prior + prow;
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = kt * kKT + nt * 8 + 2 * c + e;
          float x0 = sc[nt][e] * sl2, x1 = sc[nt][2 + e] * sl2;
          if (need_mask) {
            if (key > prior + r0) x0 = -INFINITY;
            if (key > prior + r1) x1 = -INFINITY;
          }
          sc[nt][e] = x0;
          sc[nt][2 + e] = x1;
          mx0 = fmaxf(mx0, x0);
          mx1 = fmaxf(mx1, x1);
        }
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float ms0 = mn0 == -INFINITY ? 0.f : mn0, ms1 = mn1 == -INFINITY ? 0.f : mn1;
      const float al0 = exp2f(m0 - ms0), al1 = exp2f(m1 - ms1);
      m0 = mn0;
      m1 = mn1;
      float ps0 = 0.f, ps1 = 0.f;
      uint32_t pa[4][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const float e0 = exp2f(sc[nt][0] - ms0), e1 = exp2f(sc[nt][1] - ms0);
        const float e2 = exp2f(sc[nt][2] - ms1), e3 = exp2f(sc[nt][3] - ms1);
        ps0 += e0 + e1;
        ps1 += e2 + e3;
        pa[nt >> 1][(nt & 1) * 2 + 0] = lk::pack2<T>(e0, e1);
        pa[nt >> 1][(nt & 1) * 2 + 1] = lk::pack2<T>(e2, e3);
      }
      l0 = l0 * al0 + ps0;
      l1 = l1 * al1 + ps1;
#pragma unroll
      for (int dt = 0; dt < 16; ++dt) {
        o[dt][0] *= al0;
        o[dt][1] *= al0;
        o[dt][2] *= al1;
        o[dt][3] *= al1;
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
        for (int dt = 0; dt < 16; dt += 2) {
          const uint32_t tok = kk * 16 + (j & 1) * 8 + (lane & 7);
          const uint32_t dchunk = dt + (j >> 1);
          uint32_t r[4];
          lk::ldsm_x4_t(vb + (dchunk >> 3) * kHalfBytes + lk::swz128(tok, dchunk & 7), r[0],
                        r[1], r[2], r[3]);
          lk::mma16816<T>(o[dt], pa[kk], r[0], r[1]);
          lk::mma16816<T>(o[dt + 1], pa[kk], r[2], r[3]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) lk::mbar_arrive(&empty_bar[s]);
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float i0 = 1.f / l0, i1 = 1.f / l1;
  T* out = static_cast<T*>(p.out) + static_cast<int64_t>(qhead) * kD + 2 * c;
  const int64_t ostride = static_cast<int64_t>(H) * kD;
  if (r0 < q_len) {
    T* o0 = out + static_cast<int64_t>(q_start + r0) * ostride;
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) store2<T>(o0 + dt * 8, o[dt][0] * i0, o[dt][1] * i0);
  }
  if (r1 < q_len) {
    T* o1 = out + static_cast<int64_t>(q_start + r1) * ostride;
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) store2<T>(o1 + dt * 8, o[dt][2] * i1, o[dt][3] * i1);
  }
}

template <typename T>
int launch_prefill(const CUtensorMap& km, const CUtensorMap& vm, const PrefillParams& p,
                   int num_seqs, int max_q_len, int H_kv, cudaStream_t s) {
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(paged_prefill_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSmem) != cudaSuccess)
      return LK_ERR_CUDA;
    configured[dev] = 1;
  }
  dim3 grid((max_q_len + p.BQ - 1) / p.BQ, H_kv, num_seqs);
  paged_prefill_kernel<T><<<grid, kThreads, kSmem, s>>>(km, vm, p);
  return lk::check_launch();
}


// ---------------------------------------------------------------------------
// tcgen05 (fifth-generation tensor core) version.
//
// A CTA holds NSUB query sub-tiles of 128 rows (rows = positions x the G heads
// of one KV head), all reading the same K/V tiles. Per sub-tile u:
//   warps 8u .. 8u+7: softmax and epilogue; warps w and w+4 share TMEM lanes
//     32 (w % 4) .. +31, thread (half, r) handles half of row r's 64 scores
//     and half of its 128 outputs, the halves agree on the row max through
//     shared memory and a 64-thread named barrier;
//   TMEM columns [256u, 256u+128): S double buffer (64 keys each, P written in
//     place over the S it came from); [256u+128, 256u+256): O accumulator.
// Warp 8 NSUB: TMA producer (64-token K and V tiles through the block table,
// separate K and V rings of NKV stages); warp 8 NSUB + 1: MMA issuer:
//   S_u = Q_u K^T   (kind::f16, M=128, N=64, K=128, A and B from shared memory)
//   O_u += P_u V    (M=128, N=128, K=64, A = P from TMEM, B = V MN-major)
// issued as S(j+1) for every sub-tile, then PV(j) for every sub-tile, so the
// tensor core works on tile j+1 while the softmax works on tile j. The
// running max is applied lazily: O is rescaled only when a row's max grows
// by more than 2^8.
constexpr int kTcKT = 64;                 // keys per tile
constexpr int kTcQHalf = 128 * 128;       // Q: 128 rows x 128 B (64 values of D)
constexpr int kTcKHalf = kTcKT * 128;     // K or V: 64 rows x 128 B
constexpr int kTcStage = 4 * kTcKHalf;    // K (two halves) + V (two halves) = 32 KB
constexpr float kLazyRescale = 8.f;       // log2 units

template <int NSUB, int NKV> struct TcShape {
  static constexpr int kThreads = NSUB * 256 + 64;
  static constexpr int kProducer = NSUB * 8, kMma = NSUB * 8 + 1;
  static constexpr int kSmem = NSUB * 2 * kTcQHalf + NKV * kTcStage + 1024;
  static constexpr int kTmemCols = NSUB * 256;
  static constexpr int kRows = NSUB * 128;
};

template <typename T, int NSUB, int NKV>
__global__ void __launch_bounds__(TcShape<NSUB, NKV>::kThreads, NSUB == 1 ? 2 : 1)
paged_prefill_tc_kernel(const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap, const PrefillParams p) {
  using Sh = TcShape<NSUB, NKV>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t k_full[NKV];
  __shared__ __align__(8) uint64_t k_empty[NKV];
  __shared__ __align__(8) uint64_t v_full[NKV];
  __shared__ __align__(8) uint64_t v_empty[NKV];
  __shared__ __align__(8) uint64_t s_full[NSUB][2];
  __shared__ __align__(8) uint64_t p_full[NSUB][2];
  __shared__ __align__(8) uint64_t o_done[NSUB][2];  // PV(j) completes o_done[u][j & 1]
  __shared__ __align__(8) uint64_t o_final;
  __shared__ uint32_t tmem_slot;
  __shared__ float s_red[NSUB][2][2][128];  // [sub][tile parity][half][row] partial row max
  __shared__ float s_sum[NSUB][2][128];     // [sub][half][row] partial row sum
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;                          // sub u at u * 2 * kTcQHalf
  uint8_t* sKV = smem + NSUB * 2 * kTcQHalf;

  const int qt = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.G, BQ = p.BQ;
  const int q_start = p.cu_seqlens_q[b];
  const int q_len = p.cu_seqlens_q[b + 1] - q_start;
  const int pos0 = qt * BQ;
  if (pos0 >= q_len) return;
  int prior = 0;
  if (p.block_tables != nullptr && p.context_lens != nullptr) {
    prior = p.context_lens[b] - q_len;
    if (prior < 0) {
      if (threadIdx.x == 0 && p.status) atomicOr(p.status, LK_STATUS_CTX_OOB);
      prior = 0;
    }
  }
  const int kv_end = prior + min(q_len, pos0 + BQ);
  const int ntiles = (kv_end + kTcKT - 1) / kTcKT;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NKV; ++i) {
      lk::mbar_init(&k_full[i], 1);
      lk::mbar_init(&k_empty[i], 1);
      lk::mbar_init(&v_full[i], 1);
      lk::mbar_init(&v_empty[i], 1);
    }
    for (int u = 0; u < NSUB; ++u) {
      lk::mbar_init(&s_full[u][0], 1);
      lk::mbar_init(&s_full[u][1], 1);
      lk::mbar_init(&p_full[u][0], 8);
      lk::mbar_init(&p_full[u][1], 8);
      lk::mbar_init(&o_done[u][0], 1);
      lk::mbar_init(&o_done[u][1], 1);
    }
    lk::mbar_init(&o_final, 1);
    lk::fence_barrier_init();
  }
  if (warp == Sh::kMma) lk::tc::alloc(&tmem_slot, Sh::kTmemCols);
  if (warp < NSUB * 8) {
    // Q -> shared memory, K-major with 128-byte swizzle: sub-tile u, half h of
    // the head dimension of row r.
    const int u = warp >> 3, t = threadIdx.x & 255;
    const int r = t & 127, h = t >> 7;
    const int R = u * 128 + r;
    const int pos = pos0 + R / G, g = R % G;
    const T* qrow = static_cast<const T*>(p.q) + static_cast<int64_t>(q_start + pos) * p.q_stride +
                    static_cast<int64_t>(kvh * G + g) * kD + h * 64;
    uint8_t* dq = sQ + u * 2 * kTcQHalf + h * kTcQHalf;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (pos < q_len) v = *reinterpret_cast<const uint4*>(qrow + c * 8);
      *reinterpret_cast<uint4*>(dq + lk::swz128(r, c)) = v;
    }
    lk::fence_proxy_async();
  }
  lk::tc::fence_before();
  __syncthreads();
  lk::tc::fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == Sh::kProducer) {
    // ------------------------------------------------------------ producer
    // The whole warp resolves block-table entries, 32 boxes (8 tiles) per
    // batch, one batch ahead, so the table reads never sit between two TMA
    // issues; lane 0 waits on the rings and issues the copies.
    if (lane == 0) {
      lk::prefetch_tensormap(&kmap);
      lk::prefetch_tensormap(&vmap);
    }
    const int32_t* bt =
        p.block_tables ? p.block_tables + static_cast<int64_t>(b) * p.bt_stride : nullptr;
    const int oob = static_cast<int>(p.num_slots < 0x7fffffffLL ? p.num_slots : 0x7fffffffLL);
    auto slot_of = [&](int tok) -> int {
      if (tok >= kv_end) return oob;
      if (!bt) return q_start + tok;
      const int blk = __ldg(bt + tok / p.bs);
      if (blk < 0 || blk >= p.num_blocks) {
        if (p.status) atomicOr(p.status, LK_STATUS_BLOCK_OOB);
        return oob;
      }
      return blk * p.bs + tok % p.bs;
    };
    constexpr int kBoxes = kTcKT / 16;      // boxes per tile
    constexpr int kTilesPer = 32 / kBoxes;  // tiles per 32-box batch
    int nxt = slot_of(lane * 16);
    bool ok = true;
    for (int j0 = 0; j0 < ntiles && ok; j0 += kTilesPer) {
      const int cur = nxt;
      nxt = slot_of((j0 + kTilesPer) * kTcKT + lane * 16);
      const int jn = min(ntiles, j0 + kTilesPer);
      for (int j = j0; j < jn; ++j) {
        int slots[kBoxes];
#pragma unroll
        for (int tb = 0; tb < kBoxes; ++tb)
          slots[tb] = __shfl_sync(0xffffffffu, cur, (j - j0) * kBoxes + tb);
        if (lane == 0) {
          const int st = j % NKV;
          const uint32_t ph = ((j / NKV) & 1) ^ 1;
          uint8_t* dk = sKV + st * kTcStage;
          if (!lk::mbar_wait(&k_empty[st], ph)) {
            ok = false;
          } else {
            lk::mbar_arrive_expect_tx(&k_full[st], 2 * kTcKHalf);
#pragma unroll
            for (int tb = 0; tb < kBoxes; ++tb)
#pragma unroll
              for (int dh = 0; dh < 2; ++dh)
                lk::tma_load_3d(dk + dh * kTcKHalf + tb * 2048, &kmap, &k_full[st], dh * 64,
                                slots[tb], kvh);
          }
          if (ok && !lk::mbar_wait(&v_empty[st], ph)) ok = false;
          if (ok) {
            lk::mbar_arrive_expect_tx(&v_full[st], 2 * kTcKHalf);
#pragma unroll
            for (int tb = 0; tb < kBoxes; ++tb)
#pragma unroll
              for (int dh = 0; dh < 2; ++dh)
                lk::tma_load_3d(dk + 2 * kTcKHalf + dh * kTcKHalf + tb * 2048, &vmap,
                                &v_full[st], dh * 64, slots[tb], kvh);
          }
          if (!ok && p.status) atomicOr(p.status, LK_STATUS_WAIT_TIMEOUT);
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
      }
    }
  } else if (warp == Sh::kMma) {
    // ----------------------------------------------------------- MMA issue
    if (lane == 0) {
      constexpr int fmt = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
      constexpr uint32_t idS = lk::tc::idesc_f16(fmt, 0, 0, 128, kTcKT);
      constexpr uint32_t idO = lk::tc::idesc_f16(fmt, 0, 1, 128, 128);
      const uint32_t q_addr = lk::smem_u32(sQ);
      bool ok = true;
      auto issue_s = [&](int j) -> bool {
        const int st = j % NKV;
        if (!lk::mbar_wait(&k_full[st], (j / NKV) & 1)) return false;
        lk::tc::fence_after();
        const uint32_t k_addr = lk::smem_u32(sKV + st * kTcStage);
#pragma unroll
        for (int u = 0; u < NSUB; ++u) {
          const uint32_t qa = q_addr + u * 2 * kTcQHalf;
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            lk::tc::mma_f16(
                tmem + 256 * u + 64 * (j & 1),
                lk::tc::smem_desc_sw128(qa + (ks >> 2) * kTcQHalf + (ks & 3) * 32, 16, 1024),
                lk::tc::smem_desc_sw128(k_addr + (ks >> 2) * kTcKHalf + (ks & 3) * 32, 16, 1024),
                idS, ks > 0 ? 1u : 0u);
          lk::tc::commit(&s_full[u][j & 1]);
        }
        lk::tc::commit(&k_empty[st]);
        return true;
      };
      ok = issue_s(0);
      for (int j = 0; j < ntiles && ok; ++j) {
        const int sb = j & 1, st = j % NKV;
        if (j + 1 < ntiles && !issue_s(j + 1)) {
          ok = false;
          break;
        }
        if (!lk::mbar_wait(&v_full[st], (j / NKV) & 1)) {
          ok = false;
          break;
        }
        const uint32_t v_addr = lk::smem_u32(sKV + st * kTcStage) + 2 * kTcKHalf;
#pragma unroll
        for (int u = 0; u < NSUB; ++u) {
          if (!lk::mbar_wait(&p_full[u][sb], (j >> 1) & 1)) {
            ok = false;
            break;
          }
          lk::tc::fence_after();
#pragma unroll
          for (int kk = 0; kk < kTcKT / 16; ++kk) {
            const uint64_t bd = lk::tc::smem_desc_sw128(v_addr + kk * 2048, kTcKHalf, 1024);
            lk::tc::mma_f16_ts(tmem + 256 * u + 128, tmem + 256 * u + 64 * sb + kk * 8, bd, idO,
                               (j > 0 || kk > 0) ? 1u : 0u);
          }
          lk::tc::commit(&o_done[u][sb]);
        }
        if (!ok) break;
        lk::tc::commit(&v_empty[st]);
      }
      if (!ok && p.status) atomicOr(p.status, LK_STATUS_WAIT_TIMEOUT);
      lk::tc::commit(&o_final);
    }
  } else {
    // ------------------------------------------------- softmax / epilogue
    const int u = warp >> 3, wg = (warp >> 2) & 1, r = threadIdx.x & 127;
    const int R = u * 128 + r;
    const int pos = pos0 + R / G, g = R % G;
    const int limit = prior + pos;  // last visible key of this row
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tSub = tmem + 256 * u, tO = tSub + 128;
    const int pair_bar = 1 + (warp & 3) + 4 * u;
    const float sl2 = p.scale_log2;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int sb = j & 1;
      const uint32_t tS = tSub + 64 * sb;
      // On a (never expected) wait timeout the warp carries on with garbage
      // instead of leaving: its partner warp must still meet it at every
      // named barrier below.
      if (ok && !lk::mbar_wait(&s_full[u][sb], (j >> 1) & 1)) ok = false;
      ok = __all_sync(0xffffffffu, ok);
      lk::tc::fence_after();
      uint32_t sv[32];
      lk::tc::ld32(tS + lane_base + 32 * wg, sv);
      lk::tc::wait_ld();
      const int kb = j * kTcKT + 32 * wg;
      if (kb + 31 > limit) {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (kb + i > limit) sv[i] = __float_as_uint(-INFINITY);
      }
      float ma = -INFINITY, mb = -INFINITY;
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        ma = lk::fmax3(ma, __uint_as_float(sv[i]), __uint_as_float(sv[i + 1]));
        mb = lk::fmax3(mb, __uint_as_float(sv[i + 2]), __uint_as_float(sv[i + 3]));
      }
      s_red[u][sb][wg][r] = fmaxf(ma, mb);
      lk::named_sync(pair_bar, 64);
      // both halves have read their scores (wait::ld above) before either
      // writes P over the buffer below
      const float mraw = fmaxf(s_red[u][sb][0][r], s_red[u][sb][1][r]);
      const float mx = mraw * sl2;  // sl2 > 0: max commutes with the scaling
      float new_m = m_used;
      if (mx > m_used + kLazyRescale) new_m = mx;
      const float alpha = (new_m == m_used) ? 1.f : exp2f(m_used - new_m);
      const float ms = new_m == -INFINITY ? 0.f : new_m;
      // two scores per packed fp32x2 instruction, one MUFU ex2 per score
      float sum0 = 0.f, sum1 = 0.f;
      uint32_t pw[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        float x0, x1;
        lk::ffma2(x0, x1, __uint_as_float(sv[2 * c]), __uint_as_float(sv[2 * c + 1]), sl2, sl2,
                  -ms, -ms);
        const float e0 = lk::ex2_mufu(x0);
        const float e1 = lk::ex2_mufu(x1);
        lk::fadd2(sum0, sum1, sum0, sum1, e0, e1);
        pw[c] = lk::pack2<T>(e0, e1);
      }
      lk::tc::st16(tS + lane_base + 16 * wg, pw);  // P over the S buffer it came from
      l = l * alpha + (sum0 + sum1);
      // tcgen05.ld / st are warp-collective: the warp rescales together if
      // any of its rows needs it (alpha is 1 for the others). O may only be
      // touched once PV(j-1) has completed: PV(i) completes o_done[i & 1]
      // for the (i >> 1)-th time, and PV(j+1) cannot complete before this
      // warp releases P(j), so a parity wait is exact even though most tiles
      // skip it.
      if (j > 0 && __any_sync(0xffffffffu, new_m != m_used)) {
        if (ok && !lk::mbar_wait(&o_done[u][(j - 1) & 1], ((j - 1) >> 1) & 1)) ok = false;
        ok = __all_sync(0xffffffffu, ok);
        lk::tc::fence_after();
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {
          uint32_t ov[32];
          const uint32_t ta = tO + lane_base + 64 * wg + 32 * c2;
          lk::tc::ld32(ta, ov);
          lk::tc::wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
          lk::tc::st32(ta, ov);
        }
      }
      lk::tc::wait_st();
      m_used = new_m;
      lk::tc::fence_before();
      __syncwarp();
      if (lane == 0) lk::mbar_arrive(&p_full[u][sb]);
    }
    // row sum = the two halves' partial sums (same running max in both)
    s_sum[u][wg][r] = l;
    lk::named_sync(pair_bar, 64);
    l = s_sum[u][0][r] + s_sum[u][1][r];
    if (ok && lk::mbar_wait(&o_final, 0)) {
      lk::tc::fence_after();
      const float inv = 1.f / l;
      T* orow = static_cast<T*>(p.out) + static_cast<int64_t>(q_start + pos) * p.H * kD +
                static_cast<int64_t>(kvh * G + g) * kD + 64 * wg;
#pragma unroll
      for (int c2 = 0; c2 < 2; ++c2) {
        uint32_t ov[32];
        lk::tc::ld32(tO + lane_base + 64 * wg + 32 * c2, ov);  // whole warp, every row
        lk::tc::wait_ld();
        if (pos < q_len) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
              w[e] = lk::pack2<T>(__uint_as_float(ov[c * 8 + 2 * e]) * inv,
                                  __uint_as_float(ov[c * 8 + 2 * e + 1]) * inv);
            *reinterpret_cast<uint4*>(orow + c2 * 32 + c * 8) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
    } else if (p.status && lane == 0) {
      atomicOr(p.status, LK_STATUS_WAIT_TIMEOUT);
    }
  }
  lk::tc::fence_before();
  __syncthreads();
  lk::tc::fence_after();
  if (warp == Sh::kMma) lk::tc::dealloc(tmem, Sh::kTmemCols);
}

template <typename T, int NSUB, int NKV>
int launch_prefill_tc_n(const CUtensorMap& km, const CUtensorMap& vm, PrefillParams p,
                        int num_seqs, int max_q_len, int H_kv, cudaStream_t s) {
  using Sh = TcShape<NSUB, NKV>;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(paged_prefill_tc_kernel<T, NSUB, NKV>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Sh::kSmem) != cudaSuccess)
      return LK_ERR_CUDA;
    configured[dev] = 1;
  }
  p.BQ = Sh::kRows / p.G;
  dim3 grid((max_q_len + p.BQ - 1) / p.BQ, H_kv, num_seqs);
  paged_prefill_tc_kernel<T, NSUB, NKV><<<grid, Sh::kThreads, Sh::kSmem, s>>>(km, vm, p);
  return lk::check_launch();
}

// Query sub-tiles per CTA: 1 (128-row CTAs, two per SM; measured fastest on
// B200) by default; LITEKERN_PREFILL_SUBTILES=2 selects one CTA per SM with
// two 128-row sub-tiles sharing each K/V tile (read once).
int prefill_subtiles() {
  static int v = [] {
    const char* e = getenv("LITEKERN_PREFILL_SUBTILES");
    return (e && atoi(e) == 2) ? 2 : 1;
  }();
  return v;
}

template <typename T>
int launch_prefill_tc(const CUtensorMap& km, const CUtensorMap& vm, const PrefillParams& p,
                      int num_seqs, int max_q_len, int H_kv, cudaStream_t s) {
  if (prefill_subtiles() == 1)
    return launch_prefill_tc_n<T, 1, 2>(km, vm, p, num_seqs, max_q_len, H_kv, s);
  return launch_prefill_tc_n<T, 2, 4>(km, vm, p, num_seqs, max_q_len, H_kv, s);
}

// ---------------------------------------------------------------------------
// Ping-pong kernel (the default): persistent, one CTA per SM; each work item
// is two 128-row query sub-tiles A and B (256 rows: BQ = 256 / G positions x
// G heads) sharing 128-token K/V tiles. TMEM (512 columns): S_A [0,128),
// S_B [128,256), O_A [256,384), O_B [384,512); each sub-tile's P (16-bit
// pairs) is written over the first 64 columns of its own S, in two 64-key
// halves released separately so PV on keys 0-63 overlaps the exponentials of
// keys 64-127. The MMA thread issues PV_A(j), S_A(j+1), PV_B(j), S_B(j+1), ...
// so the tensor core works on one sub-tile while the other's softmax runs.
// Warps 0-3: softmax of A, 4-7: softmax of B (one row per thread); warp 8:
// TMA producer and work scheduler; warp 9: MMA issue. Work items come from a
// global counter (the hardware's dynamic CTA dispatch, kept inside one
// persistent CTA), so barriers and TMEM are set up once per SM and the next
// item's K/V and Q loads overlap the current item's last tiles and output.
constexpr int kPpKT = 128;                 // keys per tile
constexpr int kPpKHalf = kPpKT * 128;      // K or V d-half: 128 rows x 128 B = 16 KB
constexpr int kPpKStage = 2 * kPpKHalf;    // one K (or V) tile: 32 KB
constexpr int kPpThreads = 320;
constexpr int kPpSmem = 2 * 2 * kTcQHalf + 4 * kPpKStage + 1024;  // Q_A, Q_B, 2 K + 2 V stages

template <typename T, bool PREFIX>
__global__ void __launch_bounds__(kPpThreads, 1)
paged_prefill_pp_kernel(const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap, const PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t k_full[2];
  __shared__ __align__(8) uint64_t k_empty[2];
  __shared__ __align__(8) uint64_t v_full[2];
  __shared__ __align__(8) uint64_t v_empty[2];
  __shared__ __align__(8) uint64_t q_full[2];     // [sub-tile]
  __shared__ __align__(8) uint64_t s_full[2];     // [sub-tile]
  __shared__ __align__(8) uint64_t p_full[2][2];  // [sub-tile][key half]
  __shared__ __align__(8) uint64_t o_final[2];   // [sub-tile]: its last PV completed
  __shared__ __align__(8) uint64_t item_full[2];   // work-item ring, depth 2
  __shared__ __align__(8) uint64_t item_empty[2];
  __shared__ int item_ring[2];
  __shared__ uint32_t tmem_slot;
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;                           // sub-tile u at u * 2 * kTcQHalf
  uint8_t* sK = smem + 4 * kTcQHalf;            // stage st at st * kPpKStage
  uint8_t* sV = sK + 2 * kPpKStage;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.G, BQ = p.BQ;
  const int per_q = p.H_kv * p.num_seqs;
  const int num_items =
      (!PREFIX && p.order != nullptr) ? __ldg(p.units_count) * p.H_kv : p.nqt * per_q;

  // Work item w: all items of query tile nqt - 1 first, then nqt - 2, ...
  // (later tiles see more keys under the causal mask). The producer warp
  // takes items from a global counter as it runs out of work and passes
  // them to the MMA thread and the softmax warps through item_ring.
  struct Item {
    int q_start, q_len, pos0, prior, kv_begin, kv_end, ntiles, kvh, b;
  };
  auto item = [&](int w) {
    Item it;
    int qt, piece = 0;
    if (!PREFIX && p.order != nullptr) {
      const int un = __ldg(p.order + w / p.H_kv);
      const int pr = un & 0x3fff;
      piece = (un >> 14) & 3;
      it.kvh = w % p.H_kv;
      it.b = pr / p.nqt;
      qt = pr % p.nqt;
    } else {
      qt = p.nqt - 1 - w / per_q;
      const int rem = w % per_q;
      it.kvh = rem % p.H_kv;
      it.b = rem / p.H_kv;
    }
    if constexpr (PREFIX) {  // b = key range; every row sees the whole range
      it.q_start = 0;
      it.q_len = p.prefix_rows;
      it.pos0 = qt * BQ;
      it.prior = 0;
      it.kv_begin = it.b * p.prefix_split;
      it.kv_end = min(p.prefix_len, it.kv_begin + p.prefix_split);
      it.ntiles = it.pos0 < it.q_len && it.kv_end > it.kv_begin
                      ? (it.kv_end - it.kv_begin + kPpKT - 1) / kPpKT
                      : 0;
      return it;
    }
    it.kv_begin = 0;
    it.q_start = p.cu_seqlens_q[it.b];
    it.q_len = p.cu_seqlens_q[it.b + 1] - it.q_start;
    it.pos0 = qt * BQ;
    it.prior = 0;
    if (p.block_tables != nullptr && p.context_lens != nullptr) {
      it.prior = p.context_lens[it.b] - it.q_len;
      if (it.prior < 0) {
        if (threadIdx.x == 0 && p.status) atomicOr(p.status, LK_STATUS_CTX_OOB);
        it.prior = 0;
      }
    }
    it.kv_end = it.prior + min(it.q_len, it.pos0 + BQ);
    it.ntiles = it.pos0 < it.q_len ? (it.kv_end + kPpKT - 1) / kPpKT : 0;
    if (piece != 0) {  // key-split pair: first or second half of the key tiles
      const int a = (it.ntiles + 1) / 2;
      if (piece == 1) {
        it.ntiles = a;
      } else {
        it.kv_begin = a * kPpKT;
        it.ntiles -= a;
      }
    }
    return it;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      lk::mbar_init(&k_full[i], 1);
      lk::mbar_init(&k_empty[i], 1);
      lk::mbar_init(&v_full[i], 1);
      lk::mbar_init(&v_empty[i], 1);
      lk::mbar_init(&q_full[i], 4);
      lk::mbar_init(&s_full[i], 1);
      lk::mbar_init(&p_full[i][0], 4);
      lk::mbar_init(&p_full[i][1], 4);
    }
    lk::mbar_init(&o_final[0], 1);
    lk::mbar_init(&o_final[1], 1);
    for (int i = 0; i < 2; ++i) {
      lk::mbar_init(&item_full[i], 1);
      lk::mbar_init(&item_empty[i], 9);  // the MMA thread + 8 softmax warps
    }
    lk::fence_barrier_init();
  }
  if (warp == 9) lk::tc::alloc(&tmem_slot, 512);
  lk::tc::fence_before();
  __syncthreads();
  lk::tc::fence_after();
  const uint32_t tmem = tmem_slot;
  if constexpr (PREFIX) {
    // Launched to overlap the ordering kernel ahead of it (the set-up above
    // touches no global memory): wait for it, and through it for the step's
    // KV store. Then the split decode kernel launched after this one may
    // start on the SMs this grid leaves free: everything it reads first is
    // complete by now, and it waits for this grid before merging in the
    // prefix partials.
    lk::pdl_wait();
    lk::pdl_launch_dependents();
  }
  // Consumers: the n-th item this CTA processes (num_items = no more work).
  // Lane 0 waits, reads and releases the slot; the result goes to all lanes.
  auto next_item = [&](int n, bool& ok) -> int {
    int w = num_items;
    if (lane == 0) {
      if (ok && lk::mbar_wait(&item_full[n & 1], (n >> 1) & 1)) {
        w = item_ring[n & 1];
        lk::mbar_arrive(&item_empty[n & 1]);
      } else {
        ok = false;
      }
    }
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    return __shfl_sync(0xffffffffu, w, 0);
  };

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      lk::prefetch_tensormap(&kmap);
      lk::prefetch_tensormap(&vmap);
    }
    const int oob = static_cast<int>(p.num_slots < 0x7fffffffLL ? p.num_slots : 0x7fffffffLL);
    constexpr int kBoxes = kPpKT / 16;      // 8 boxes per tile
    constexpr int kTilesPer = 32 / kBoxes;  // 4 tiles per block-table batch
    bool ok = true;
    int g = 0;  // K/V tiles loaded so far by this CTA
    for (int n = 0; ok; ++n) {
      int w = num_items;
      if (lane == 0) {
        do {
          w = atomicAdd(p.sched, 1);
        } while (w < num_items && item(w).ntiles == 0);
        if (w > num_items) w = num_items;
        if (lk::mbar_wait(&item_empty[n & 1], ((n >> 1) & 1) ^ 1)) {
          item_ring[n & 1] = w;
          lk::mbar_arrive(&item_full[n & 1]);
        } else {
          ok = false;
          if (p.status) atomicOr(p.status, LK_STATUS_WAIT_TIMEOUT);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      w = __shfl_sync(0xffffffffu, w, 0);
      if (!ok || w >= num_items) break;
      const Item it = item(w);
      const int32_t* bt = p.block_tables ? p.block_tables + (PREFIX ? 0 : static_cast<int64_t>(it.b) * p.bt_stride)
                                         : nullptr;
      auto slot_of = [&](int tok) -> int {  // tok counts from the item's first key
        tok += it.kv_begin;
        if (tok >= it.kv_end) return oob;
        if (!bt) return it.q_start + tok;
        const int blk = __ldg(bt + tok / p.bs);
        if (blk < 0 || blk >= p.num_blocks) {
          if (p.status) atomicOr(p.status, LK_STATUS_BLOCK_OOB);
          return oob;
        }
        return blk * p.bs + tok % p.bs;
      };
      int nxt = it.ntiles > 0 ? slot_of(lane * 16) : oob;
      for (int j0 = 0; j0 < it.ntiles && ok; j0 += kTilesPer) {
        const int cur = nxt;
        nxt = slot_of((j0 + kTilesPer) * kPpKT + lane * 16);
        const int jn = min(it.ntiles, j0 + kTilesPer);
        for (int j = j0; j < jn; ++j, ++g) {
          int slots[kBoxes];
#pragma unroll
          for (int tb = 0; tb < kBoxes; ++tb)
            slots[tb] = __shfl_sync(0xffffffffu, cur, (j - j0) * kBoxes + tb);
          if (lane == 0) {
            const int st = g & 1;
            const uint32_t ph = ((g >> 1) & 1) ^ 1;
            if (!lk::mbar_wait(&k_empty[st], ph)) {
              ok = false;
            } else {
              lk::mbar_arrive_expect_tx(&k_full[st], kPpKStage);
#pragma unroll
              for (int tb = 0; tb < kBoxes; ++tb)
#pragma unroll
                for (int dh = 0; dh < 2; ++dh)
                  lk::tma_load_3d(sK + st * kPpKStage + dh * kPpKHalf + tb * 2048, &kmap,
                                  &k_full[st], dh * 64, slots[tb], it.kvh);
            }
            if (ok && !lk::mbar_wait(&v_empty[st], ph)) ok = false;
            if (ok) {
              lk::mbar_arrive_expect_tx(&v_full[st], kPpKStage);
#pragma unroll
              for (int tb = 0; tb < kBoxes; ++tb)
#pragma unroll
                for (int dh = 0; dh < 2; ++dh)
                  lk::tma_load_3d(sV + st * kPpKStage + dh * kPpKHalf + tb * 2048, &vmap,
                                  &v_full[st], dh * 64, slots[tb], it.kvh);
            }
            if (!ok && p.status) atomicOr(p.status, LK_STATUS_WAIT_TIMEOUT);
          }
          ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
          if (!ok) break;
        }
      }
    }
  } else if (warp == 9) {
    // ----------------------------------------------------------- MMA issue
    if (lane == 0) {
      constexpr int fmt = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
      constexpr uint32_t idS = lk::tc::idesc_f16(fmt, 0, 0, 128, kPpKT);
      constexpr uint32_t idO = lk::tc::idesc_f16(fmt, 0, 1, 128, 128);
      const uint32_t q_addr = lk::smem_u32(sQ), k_addr0 = lk::smem_u32(sK),
                     v_addr0 = lk::smem_u32(sV);
      auto issue_s = [&](int u, int g) {
        const uint32_t qa = q_addr + u * 2 * kTcQHalf;
        const uint32_t ka = k_addr0 + (g & 1) * kPpKStage;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          lk::tc::mma_f16(
              tmem + 128 * u,
              lk::tc::smem_desc_sw128(qa + (ks >> 2) * kTcQHalf + (ks & 3) * 32, 16, 1024),
              lk::tc::smem_desc_sw128(ka + (ks >> 2) * kPpKHalf + (ks & 3) * 32, 16, 1024), idS,
              ks > 0 ? 1u : 0u);
        lk::tc::commit(&s_full[u]);
      };
      auto issue_pv = [&](int u, int g, bool first, int h) {  // keys 64h .. 64h + 63
        const uint32_t va = v_addr0 + (g & 1) * kPpKStage;
#pragma unroll
        for (int kk = 4 * h; kk < 4 * h + 4; ++kk) {
          const uint64_t bd = lk::tc::smem_desc_sw128(va + kk * 2048, kPpKHalf, 1024);
          lk::tc::mma_f16_ts(tmem + 256 + 128 * u, tmem + 128 * u + kk * 8, bd, idO,
                             (!first || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = true;
      int g = 0, n_items = 0;
      for (;;) {
        int w = num_items;
        if (lk::mbar_wait(&item_full[n_items & 1], (n_items >> 1) & 1)) {
          w = item_ring[n_items & 1];
          lk::mbar_arrive(&item_empty[n_items & 1]);
        } else {
          ok = false;
        }
        if (!ok || w >= num_items) break;
        const Item it = item(w);
        // first tile's S for both sub-tiles, each once its Q is in shared memory
        ok = lk::mbar_wait(&k_full[g & 1], (g >> 1) & 1);
#pragma unroll
        for (int u = 0; u < 2 && ok; ++u) {
          ok = lk::mbar_wait(&q_full[u], n_items & 1);
          lk::tc::fence_after();
          if (ok) issue_s(u, g);
        }
        if (!ok) break;
        lk::tc::commit(&k_empty[g & 1]);
        for (int j = 0; j < it.ntiles && ok; ++j, ++g) {
          const int st = g & 1;
          const bool more = j + 1 < it.ntiles;
          if (!lk::mbar_wait(&v_full[st], (g >> 1) & 1)) { ok = false; break; }
          if (more && !lk::mbar_wait(&k_full[st ^ 1], ((g + 1) >> 1) & 1)) { ok = false; break; }
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            if (!lk::mbar_wait(&p_full[u][0], g & 1)) { ok = false; break; }
            lk::tc::fence_after();
            issue_pv(u, g, j == 0, 0);
            if (!lk::mbar_wait(&p_full[u][1], g & 1)) { ok = false; break; }
            lk::tc::fence_after();
            issue_pv(u, g, j == 0, 1);
            if (u == 1) lk::tc::commit(&v_empty[st]);
            if (more) issue_s(u, g + 1);  // S_u(j+1) after PV_u(j): P_u(j) is read first
            else lk::tc::commit(&o_final[u]);  // O_u complete: its epilogue need not wait for the other sub-tile
          }
          if (!ok) break;
          if (more) lk::tc::commit(&k_empty[st ^ 1]);
        }
        ++n_items;
      }
      if (!ok && p.status) atomicOr(p.status, LK_STATUS_WAIT_TIMEOUT);
    }
  } else {
    // ------------------------------------------------- softmax / epilogue
    const int u = warp >> 2, t = threadIdx.x, r = t & 127;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + 128 * u, tO = tmem + 256 + 128 * u;
    uint8_t* dq = sQ + u * 2 * kTcQHalf;
    const float sl2 = p.scale_log2;
    // Row t of an item's 256-row tile: position pos0 + t / G, head g = t % G,
    // copied straight into the (128-byte swizzled) Q buffer with cp.async.
    auto load_q = [&](const Item& it) {
      const int pos = it.pos0 + t / G, gq = t % G;
      const bool valid = pos < it.q_len;
      const T* qrow = static_cast<const T*>(p.q) +
                      static_cast<int64_t>(it.q_start + (valid ? pos : 0)) * p.q_stride +
                      static_cast<int64_t>(it.kvh * G + gq) * kD;
#pragma unroll
      for (int c = 0; c < 16; ++c)
        lk::cp_async16(dq + (c >> 3) * kTcQHalf + lk::swz128(r, c & 7), qrow + c * 8, valid);
    };
    auto publish_q = [&]() {
      lk::cp_async_wait_all();
      lk::fence_proxy_async();
      __syncwarp();
      if (lane == 0) lk::mbar_arrive(&q_full[u]);
    };
    bool ok = true;
    int g = 0, n_items = 0;
    int w = next_item(0, ok);
    if (w < num_items) {
      load_q(item(w));
      publish_q();
    }
    while (w < num_items && ok) {
      const Item it = item(w);
      const int pos = it.pos0 + t / G, gh = t % G;
      const int limit = PREFIX ? it.kv_end - 1 : it.prior + pos;  // last visible key of this row
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < it.ntiles; ++j, ++g) {
        if (ok && !lk::mbar_wait(&s_full[u], g & 1)) ok = false;
        ok = __all_sync(0xffffffffu, ok);
        lk::tc::fence_after();
        // Pass 1: row maximum over the 128 scores, 64 columns per TMEM load.
        const int kb = it.kv_begin + j * kPpKT;
        const bool diag = kb + kPpKT - 1 > limit;  // tile crosses the causal edge
        auto load_half = [&](int h, uint32_t (&sv)[2][32]) {
          lk::tc::ld32(tS + lane_base + 64 * h, sv[0]);
          lk::tc::ld32(tS + lane_base + 64 * h + 32, sv[1]);
          lk::tc::wait_ld();
          if (diag) {
#pragma unroll
            for (int c2 = 0; c2 < 2; ++c2)
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (kb + 64 * h + 32 * c2 + i > limit) sv[c2][i] = __float_as_uint(-INFINITY);
          }
        };
        float mc[4];  // four independent max chains
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t sv[2][32];
          load_half(h, sv);
#pragma unroll
          for (int c2 = 0; c2 < 2; ++c2) {
            float m = lk::fmax3(__uint_as_float(sv[c2][0]), __uint_as_float(sv[c2][1]),
                                __uint_as_float(sv[c2][2]));
#pragma unroll
            for (int i = 3; i < 31; i += 2)
              m = lk::fmax3(m, __uint_as_float(sv[c2][i]), __uint_as_float(sv[c2][i + 1]));
            mc[2 * h + c2] = fmaxf(m, __uint_as_float(sv[c2][31]));
          }
        }
        const float mx = fmaxf(fmaxf(mc[0], mc[1]), fmaxf(mc[2], mc[3])) * sl2;
        float new_m = m_used;
        if (mx > m_used + kLazyRescale) new_m = mx;
        const float alpha = (new_m == m_used) ? 1.f : lk::ex2_mufu(m_used - new_m);
        const float ms = new_m == -INFINITY ? 0.f : new_m;
        // Rescale O_u before any of P(j) is released (PV(j) accumulates onto
        // it). O_u is stable here: S_u(j) was issued after PV_u(j-1), and
        // s_full of tile j was committed after S_u(j). The warp rescales
        // together if any of its rows needs it (tcgen05.ld / st are
        // warp-collective); the first half's wait_st orders these stores
        // before the release.
        if (j > 0 && __any_sync(0xffffffffu, new_m != m_used)) {
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) {
            uint32_t ov[32];
            lk::tc::ld32(tO + lane_base + 32 * c4, ov);
            lk::tc::wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
            lk::tc::st32(tO + lane_base + 32 * c4, ov);
          }
        }
        // Pass 2: exponentials per 64-key half, P written over the half's
        // first 32 columns and released half by half.
        float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t sv[2][32];
          load_half(h, sv);
          uint32_t pw[32];
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            float x0, x1;
            lk::ffma2(x0, x1, __uint_as_float(sv[c >> 4][(2 * c) & 31]),
                      __uint_as_float(sv[c >> 4][(2 * c + 1) & 31]), sl2, sl2, -ms, -ms);
            const float e0 = lk::ex2_mufu(x0);
            const float e1 = lk::ex2_mufu(x1);
            lk::fadd2(sum0, sum1, sum0, sum1, e0, e1);
            pw[c] = lk::pack2<T>(e0, e1);
          }
          lk::tc::st32(tS + lane_base + 32 * h, pw);  // keys 64h.. -> P columns 32h..
          lk::tc::wait_st();
          lk::tc::fence_before();
          __syncwarp();
          if (lane == 0) lk::mbar_arrive(&p_full[u][h]);
        }
        l = l * alpha + (sum0 + sum1);
        m_used = new_m;
      }
      // The next item's query rows go to the Q buffer (its only reader, S of
      // this item's last tile, has completed) while the last PV MMAs run.
      // They are published before this item's output leaves TMEM: the next
      // S MMAs only touch the S / P columns, so they overlap the epilogue,
      // and PV of the next item (which overwrites O) waits for P from these
      // threads, i.e. for the end of the epilogue.
      const int wn = next_item(n_items + 1, ok);
      if (wn < num_items) load_q(item(wn));
      if (ok && lk::mbar_wait(&o_final[u], n_items & 1)) {
        if (wn < num_items) publish_q();
        lk::tc::fence_after();
        if constexpr (PREFIX) {
          // partial (m, l, unnormalised o) of row (sequence pos, head) for this key range
          const int64_t prow =
              (static_cast<int64_t>(pos) * p.part_splits + it.b) * p.H + it.kvh * G + gh;
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) {
            uint32_t ov[32];
            lk::tc::ld32(tO + lane_base + 32 * c4, ov);  // whole warp, every row
            lk::tc::wait_ld();
            if (pos < it.q_len) {
              float4* po = reinterpret_cast<float4*>(p.part_o + prow * kD + c4 * 32);
#pragma unroll
              for (int c = 0; c < 8; ++c)
                po[c] = make_float4(__uint_as_float(ov[4 * c]), __uint_as_float(ov[4 * c + 1]),
                                    __uint_as_float(ov[4 * c + 2]), __uint_as_float(ov[4 * c + 3]));
            }
          }
          if (pos < it.q_len) {
            p.part_ml[prow * 2] = m_used;
            p.part_ml[prow * 2 + 1] = l;
          }
        } else if (p.order != nullptr && (__ldg(p.order + w / p.H_kv) >> 14) != 0) {
          // Key-split pair, per warp (32 rows): the piece that arrives first
          // writes its (m, l, unnormalised o) to the workspace and raises a
          // ready flag; the one that arrives second waits for the flag (the
          // first is resident and past all its waits: only stores remain;
          // the wait is bounded all the same), reads that partial and merges
          // it with its own O from TMEM. The merge puts piece 1's term first
          // whichever piece runs it, so the bits do not depend on the order.
          // Partials are [piece][16-byte d chunk][256 rows]: a warp's store
          // or load of one chunk covers 512 contiguous bytes.
          const int un = __ldg(p.order + w / p.H_kv);
          const int64_t slot = static_cast<int64_t>(un >> 16) * p.H_kv + it.kvh;
          const int piece = (un >> 14) & 3;
          int* cnt = p.split_cnt + (slot * 8 + warp) * 2;  // [arrivals, ready]
          int arrival = 0;
          if (lane == 0) arrival = atomicAdd(cnt, 1);
          arrival = __shfl_sync(0xffffffffu, arrival, 0);
          if (arrival == 0) {
            float4* po = reinterpret_cast<float4*>(p.split_o) + (slot * 2 + (piece - 1)) * 32 * 256 + t;
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4) {
              uint32_t ov[32];
              lk::tc::ld32(tO + lane_base + 32 * c4, ov);  // whole warp, every row
              lk::tc::wait_ld();
#pragma unroll
              for (int c = 0; c < 8; ++c)
                __stcg(po + (c4 * 8 + c) * 256,
                       make_float4(__uint_as_float(ov[4 * c]), __uint_as_float(ov[4 * c + 1]),
                                   __uint_as_float(ov[4 * c + 2]), __uint_as_float(ov[4 * c + 3])));
            }
            __stcg(reinterpret_cast<float2*>(p.split_ml) + (slot * 2 + (piece - 1)) * 256 + t,
                   make_float2(m_used, l));
            __threadfence();
            __syncwarp();
            if (lane == 0) atomicExch(cnt + 1, 1);
          } else {
            bool ready = true;
            if (lane == 0) {
              const uint64_t t0 = lk::globaltimer_ns();
              while (atomicAdd(cnt + 1, 0) == 0) {
                if (lk::globaltimer_ns() - t0 > lk::kWaitTimeoutNs) {
                  ready = false;
                  if (p.status) atomicOr(p.status, LK_STATUS_WAIT_TIMEOUT);
                  break;
                }
                __nanosleep(64);
              }
              cnt[0] = 0;  // both pieces have arrived: leave the counters zero
              cnt[1] = 0;
            }
            ready = __shfl_sync(0xffffffffu, ready ? 1 : 0, 0) != 0;
            __threadfence();
            const float2 mo = __ldcg(reinterpret_cast<const float2*>(p.split_ml) +
                                     (slot * 2 + (2 - piece)) * 256 + t);
            const float2 ml1 = piece == 1 ? make_float2(m_used, l) : mo;
            const float2 ml2 = piece == 1 ? mo : make_float2(m_used, l);
            const float mm = fmaxf(ml1.x, ml2.x);  // finite: piece 1 always sees key 0
            const float a1 = exp2f(ml1.x - mm), a2 = exp2f(ml2.x - mm);
            const float inv = 1.f / (ml1.y * a1 + ml2.y * a2);
            const float w1 = a1 * inv, w2 = a2 * inv;
            const float4* oo = reinterpret_cast<const float4*>(p.split_o) +
                               (slot * 2 + (2 - piece)) * 32 * 256 + t;
            T* orow = static_cast<T*>(p.out) + static_cast<int64_t>(it.q_start + pos) * p.H * kD +
                      static_cast<int64_t>(it.kvh * G + gh) * kD;
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4) {
              uint32_t ov[32];
              lk::tc::ld32(tO + lane_base + 32 * c4, ov);  // whole warp, every row
              lk::tc::wait_ld();
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                const float4 y0 = __ldcg(oo + (c4 * 8 + 2 * c) * 256);
                const float4 y1 = __ldcg(oo + (c4 * 8 + 2 * c + 1) * 256);
                const float yv[8] = {y0.x, y0.y, y0.z, y0.w, y1.x, y1.y, y1.z, y1.w};
                uint32_t o4[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float s0 = __uint_as_float(ov[c * 8 + 2 * e]);
                  const float s1 = __uint_as_float(ov[c * 8 + 2 * e + 1]);
                  const float p0 = piece == 1 ? s0 : yv[2 * e], q0 = piece == 1 ? yv[2 * e] : s0;
                  const float p1 = piece == 1 ? s1 : yv[2 * e + 1], q1 = piece == 1 ? yv[2 * e + 1] : s1;
                  o4[e] = lk::pack2<T>(p0 * w1 + q0 * w2, p1 * w1 + q1 * w2);
                }
                if (ready && pos < it.q_len)
                  *reinterpret_cast<uint4*>(orow + c4 * 32 + c * 8) =
                      make_uint4(o4[0], o4[1], o4[2], o4[3]);
              }
            }
          }
        } else {
        const float inv = 1.f / l;
        T* orow = static_cast<T*>(p.out) + static_cast<int64_t>(it.q_start + pos) * p.H * kD +
                  static_cast<int64_t>(it.kvh * G + gh) * kD;
        // two 32-column TMEM loads in flight per wait (the loop's registers are free here)
#pragma unroll
        for (int c8 = 0; c8 < 2; ++c8) {
          uint32_t ov[2][32];
          lk::tc::ld32(tO + lane_base + 64 * c8, ov[0]);  // whole warp, every row
          lk::tc::ld32(tO + lane_base + 64 * c8 + 32, ov[1]);
          lk::tc::wait_ld();
          if (pos < it.q_len) {
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              uint32_t o4[4];
#pragma unroll
              for (int e = 0; e < 4; ++e)
                o4[e] = lk::pack2<T>(__uint_as_float(ov[c >> 2][(c & 3) * 8 + 2 * e]) * inv,
                                     __uint_as_float(ov[c >> 2][(c & 3) * 8 + 2 * e + 1]) * inv);
              *reinterpret_cast<uint4*>(orow + c8 * 64 + c * 8) =
                  make_uint4(o4[0], o4[1], o4[2], o4[3]);
            }
          }
        }
        }
      } else {
        ok = false;
        if (p.status && lane == 0) atomicOr(p.status, LK_STATUS_WAIT_TIMEOUT);
      }
      ok = __all_sync(0xffffffffu, ok);
      ++n_items;
      w = wn;
      lk::tc::fence_before();  // O reads done before P of the next item is released
    }
    lk::cp_async_wait_all();  // nothing left in flight after a failed wait
  }
  lk::tc::fence_before();
  __syncthreads();
  lk::tc::fence_after();
  if (warp == 9) lk::tc::dealloc(tmem, 512);
}

// Work plan of the ping-pong kernel, made on the device by one CTA before
// each launch (it also zeroes the work-item counter, so it replaces the
// counter's memset).
//  * Longest first. Items of one (sequence, query tile) pair have the same
//    number of key tiles for every KV head, and that number grows with the
//    sequence's prior context, not only with the query tile: a tile-major
//    order leaves SMs that drew a long item early to draw a second long one
//    at the end. Pairs are counted into key-tile buckets, scanned from the
//    longest bucket down and scattered.
//  * Key split of the tail. When the launch has at most four waves of items,
//    pairs whose items start after the first wave and have at least half the
//    key tiles of the longest pair (and >= 4) are
//    cut into two pieces of half the tiles each (merged through the
//    workspace by whichever piece ends second), and the pieces are ordered
//    with the rest by length: the last wave is then made of shorter items.
//    At most cap_split pairs are cut (the workspace's room), the earliest in
//    the longest-first order.
// Within a bucket the order is arbitrary: items are independent, only the
// timing depends on it.
constexpr int kOrderCap = 16384;     // pairs the plan can order (pair ids fit 14 bits)
constexpr int kOrderBuckets = 1024;  // key-tile counts >= 1023 share the last bucket
constexpr int kPlanHeaderBytes = 256;
constexpr size_t kPlanBytes = kPlanHeaderBytes + sizeof(int) * 3 * kOrderCap;  // + pairs + units
constexpr size_t kSplitItemBytes = 16 * sizeof(int) + 2 * 256 * 2 * sizeof(float) +
                                   2 * 256 * kD * sizeof(float);

// Exclusive scan over the 1024 threads of the block; *total gets the sum.
LK_DEVINL int block_exclusive_scan(int v, int* warp_tot, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tot[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int t = warp_tot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    warp_tot[lane] = t;  // inclusive
  }
  __syncthreads();
  const int r = x - v + (warp > 0 ? warp_tot[warp - 1] : 0);
  *total = warp_tot[31];
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(1024)
prefill_plan_kernel(const int32_t* __restrict__ cu_seqlens_q,
                    const int32_t* __restrict__ context_lens, int num_seqs, int nqt, int BQ,
                    int H_kv, int num_sms, int cap_split, int* __restrict__ header,
                    int* __restrict__ pairs, int* __restrict__ units,
                    int* __restrict__ split_cnt) {
  __shared__ int hist[kOrderBuckets];
  __shared__ int bstart[kOrderBuckets];  // first position of each bucket
  __shared__ int bcut[kOrderBuckets];    // 1: every pair of the bucket is cut
  __shared__ int warp_tot[32];
  __shared__ int n_valid;
  const int tid = threadIdx.x;
  const int n = num_seqs * nqt;
  hist[tid] = 0;
  if (tid == 0) {
    header[0] = 0;  // work-item counter of the launch that follows
    n_valid = 0;
  }
  for (int i = tid; i < 16 * cap_split * H_kv; i += 1024) split_cnt[i] = 0;
  __syncthreads();
  auto ntiles = [&](int pr) {
    const int b = pr / nqt, qt = pr % nqt;
    const int q_start = __ldg(cu_seqlens_q + b), q_len = __ldg(cu_seqlens_q + b + 1) - q_start;
    const int pos0 = qt * BQ;
    if (pos0 >= q_len) return 0;
    const int prior = context_lens ? max(__ldg(context_lens + b) - q_len, 0) : 0;
    return (prior + min(q_len, pos0 + BQ) + 127) / 128;
  };
  auto bucket = [](int nt) { return kOrderBuckets - 1 - min(nt, kOrderBuckets - 1); };
  int total;
  // 1. pairs, longest first
  for (int pr = tid; pr < n; pr += 1024) {
    const int nt = ntiles(pr);
    if (nt > 0) atomicAdd(&n_valid, 1);
    atomicAdd(&hist[bucket(nt)], 1);
  }
  __syncthreads();
  const int count = hist[tid];  // pairs in bucket tid
  hist[tid] = block_exclusive_scan(hist[tid], warp_tot, &total);
  bstart[tid] = hist[tid];
  __syncthreads();
  for (int pr = tid; pr < n; pr += 1024) pairs[atomicAdd(&hist[bucket(ntiles(pr))], 1)] = pr;
  __syncthreads();
  // 2. which pairs to cut. The order inside a bucket comes from atomics and
  // differs between launches, and a cut pair's result differs from the uncut
  // one in the last bits; so the decision is made per bucket: a bucket is cut
  // whole when it starts after the first wave of items, its pairs have at
  // least min_cut key tiles, and all its pairs fit in the workspace's room
  // (cap_split) after the longer buckets' cuts. Same inputs, same bits.
  const bool enable = cap_split > 0 && static_cast<int64_t>(n_valid) * H_kv <= 4LL * num_sms;
  const int min_cut = n > 0 ? max(4, (ntiles(pairs[0] & 0x3fff) + 1) / 2) : 4;
  {
    const int nt_b = kOrderBuckets - 1 - tid;  // key tiles of bucket tid (last: >= that)
    const bool cuttable = enable && count > 0 && nt_b >= min_cut &&
                          static_cast<int64_t>(bstart[tid] + 1) * H_kv > num_sms;
    const int want = cuttable ? count : 0;
    const int before = block_exclusive_scan(want, warp_tot, &total);
    bcut[tid] = cuttable && before + count <= cap_split ? 1 : 0;
  }
  __syncthreads();
  // split ids: contiguous positions per thread, a scan over the cut ones
  const int seg = (n + 1023) / 1024, k0 = min(n, tid * seg), k1 = min(n, k0 + seg);
  auto cut = [&](int nt) { return bcut[bucket(nt)] != 0; };
  int cnt = 0;
  for (int k = k0; k < k1; ++k) cnt += cut(ntiles(pairs[k])) ? 1 : 0;
  int sid = block_exclusive_scan(cnt, warp_tot, &total);
  const int nsplit = total;  // <= cap_split by construction
  for (int k = k0; k < k1; ++k) {
    const int pr = pairs[k];
    if (cut(ntiles(pr))) {
      pairs[k] = pr | ((sid + 1) << 14);
      ++sid;
    }
  }
  hist[tid] = 0;
  __syncthreads();
  // 3. units (whole pairs and pieces), longest first
  for (int k = tid; k < n; k += 1024) {
    const int e = pairs[k], nt = ntiles(e & 0x3fff);
    if (e >> 14) {
      atomicAdd(&hist[bucket((nt + 1) / 2)], 1);
      atomicAdd(&hist[bucket(nt / 2)], 1);
    } else {
      atomicAdd(&hist[bucket(nt)], 1);
    }
  }
  __syncthreads();
  hist[tid] = block_exclusive_scan(hist[tid], warp_tot, &total);
  __syncthreads();
  for (int k = tid; k < n; k += 1024) {
    const int e = pairs[k], pr = e & 0x3fff, nt = ntiles(pr), s1 = e >> 14;
    if (s1) {
      const int id = (s1 - 1) << 16;
      units[atomicAdd(&hist[bucket((nt + 1) / 2)], 1)] = pr | (1 << 14) | id;
      units[atomicAdd(&hist[bucket(nt / 2)], 1)] = pr | (2 << 14) | id;
    } else {
      units[atomicAdd(&hist[bucket(nt)], 1)] = pr;
    }
  }
  if (tid == 0) header[1] = n + nsplit;
}

// Longest-first plan on (LITEKERN_PREFILL_ORDER=0 turns it off) and key
// splits of the tail on (LITEKERN_PREFILL_SPLIT=0 turns them off); read once.
bool env_on(const char* name) {
  const char* e = getenv(name);
  return !(e && atoi(e) == 0);
}
bool use_prefill_order() {
  static int v = env_on("LITEKERN_PREFILL_ORDER") ? 1 : 0;
  return v != 0;
}
bool use_prefill_split() {
  static int v = env_on("LITEKERN_PREFILL_SPLIT") ? 1 : 0;
  return v != 0;
}

// Where the plan and the key-split partials live: the caller's workspace, or
// (no workspace: no splits) a buffer kept per (device, stream) so that
// launches on different streams never share one.
struct PrefillWs {
  int* header;  // [0] work-item counter, [1] number of units
  int* pairs;
  int* units;
  int* split_cnt;
  float* split_ml;
  float* split_o;
  int cap_split_items;
};

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

size_t prefill_ws_bytes(int cap) {
  return kPlanBytes + align256(sizeof(int) * 16 * cap) + align256(sizeof(float) * 2 * 256 * 2 * cap) +
         sizeof(float) * 2 * 256 * kD * cap;
}

PrefillWs prefill_ws_layout(void* ws, size_t bytes) {
  PrefillWs w{};
  uint8_t* b = static_cast<uint8_t*>(ws);
  w.header = reinterpret_cast<int*>(b);
  w.pairs = w.header + kPlanHeaderBytes / sizeof(int);
  w.units = w.pairs + kOrderCap;
  int cap = bytes > kPlanBytes ? static_cast<int>((bytes - kPlanBytes) / kSplitItemBytes) : 0;
  cap = min(cap, lk::num_sms());
  while (cap > 0 && prefill_ws_bytes(cap) > bytes) --cap;
  w.cap_split_items = cap;
  uint8_t* c = b + kPlanBytes;
  w.split_cnt = reinterpret_cast<int*>(c);
  c += align256(sizeof(int) * 16 * cap);
  w.split_ml = reinterpret_cast<float*>(c);
  c += align256(sizeof(float) * 2 * 256 * 2 * cap);
  w.split_o = reinterpret_cast<float*>(c);
  return w;
}

int* sched_counter(cudaStream_t s) {
  struct Entry {
    int dev;
    cudaStream_t stream;
    int* ptr;
  };
  static std::mutex mu;
  static std::vector<Entry> table;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  for (const Entry& e : table)
    if (e.dev == dev && e.stream == s) return e.ptr;
  int* ptr = nullptr;
  if (cudaMalloc(&ptr, kPlanBytes) != cudaSuccess) return nullptr;
  table.push_back({dev, s, ptr});
  return ptr;
}

template <typename T>
int launch_prefill_pp(const CUtensorMap& km, const CUtensorMap& vm, PrefillParams p,
                      int num_seqs, int max_q_len, int H_kv, void* workspace,
                      size_t workspace_bytes, cudaStream_t s) {
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(paged_prefill_pp_kernel<T, false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kPpSmem) != cudaSuccess)
      return LK_ERR_CUDA;
    configured[dev] = 1;
  }
  p.BQ = 256 / p.G;
  p.nqt = (max_q_len + p.BQ - 1) / p.BQ;
  p.num_seqs = num_seqs;
  p.H_kv = H_kv;
  const int64_t items = static_cast<int64_t>(p.nqt) * H_kv * num_seqs;
  if (items > 0x7fffffffLL) return LK_ERR_TOO_LARGE;
  PrefillWs w{};
  if (workspace != nullptr) {
    w = prefill_ws_layout(workspace, workspace_bytes);
  } else {
    w.header = sched_counter(s);
    if (w.header == nullptr) return LK_ERR_CUDA;
    w.pairs = w.header + kPlanHeaderBytes / sizeof(int);
    w.units = w.pairs + kOrderCap;
  }
  p.sched = w.header;
  p.order = nullptr;
  p.units_count = nullptr;
  p.split_cnt = w.split_cnt;
  p.split_ml = w.split_ml;
  p.split_o = w.split_o;
  const int64_t pairs = static_cast<int64_t>(p.nqt) * num_seqs;
  if (pairs <= kOrderCap && use_prefill_order()) {
    const int cap_split = use_prefill_split() ? w.cap_split_items / H_kv : 0;
    prefill_plan_kernel<<<1, 1024, 0, s>>>(
        p.cu_seqlens_q, (p.block_tables && p.context_lens) ? p.context_lens : nullptr,
        num_seqs, p.nqt, p.BQ, H_kv, lk::num_sms(), cap_split, w.header, w.pairs, w.units,
        w.split_cnt);
    p.order = w.units;
    p.units_count = w.header + 1;
  } else if (cudaMemsetAsync(p.sched, 0, sizeof(int), s) != cudaSuccess) {
    return LK_ERR_CUDA;
  }
  // A split turns one pair into two units: at most twice the pairs' items.
  const int64_t max_items = p.order ? 2 * items : items;
  if (max_items > 0x7fffffffLL) return LK_ERR_TOO_LARGE;
  const int grid = static_cast<int>(max_items < lk::num_sms() ? max_items : lk::num_sms());
  paged_prefill_pp_kernel<T, false><<<grid, kPpThreads, kPpSmem, s>>>(km, vm, p);
  return lk::check_launch();
}

// Shared-prefix mode of the ping-pong kernel: B decode rows (q [B, H, D]) of
// every KV head against prefix keys [0, prefix_len) in ranges of prefix_split
// tokens; writes (m, l, o) partials.
template <typename T>
int launch_prefix_pp(const CUtensorMap& km, const CUtensorMap& vm, PrefillParams p, int B,
                     int H_kv, int* zeroed_counter, cudaStream_t s) {
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(paged_prefill_pp_kernel<T, true>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kPpSmem) != cudaSuccess)
      return LK_ERR_CUDA;
    configured[dev] = 1;
  }
  p.BQ = 256 / p.G;
  p.nqt = (B + p.BQ - 1) / p.BQ;
  p.H_kv = H_kv;
  p.order = nullptr;
  p.units_count = nullptr;
  p.split_cnt = nullptr;
  p.split_ml = nullptr;
  p.split_o = nullptr;
  const int64_t items = static_cast<int64_t>(p.nqt) * H_kv * p.num_seqs;
  if (items > 0x7fffffffLL) return LK_ERR_TOO_LARGE;
  if (zeroed_counter != nullptr) {  // zeroed earlier on this stream by the caller
    p.sched = zeroed_counter;
  } else {
    p.sched = sched_counter(s);
    if (p.sched == nullptr) return LK_ERR_CUDA;
    if (cudaMemsetAsync(p.sched, 0, sizeof(int), s) != cudaSuccess) return LK_ERR_CUDA;
  }
  const int grid = static_cast<int>(items < lk::num_sms() ? items : lk::num_sms());
  const cudaError_t e = lk::launch_after_previous(paged_prefill_pp_kernel<T, true>, dim3(grid),
                                                  dim3(kPpThreads), kPpSmem, s, km, vm, p);
  return e == cudaSuccess ? LK_OK : LK_ERR_CUDA;
}

// Prefill kernel choice: the two-sub-tile ping-pong kernel by default;
// LITEKERN_PREFILL_KERNEL=single selects the one-sub-tile kernel (read once).
bool use_pingpong() {
  static int v = [] {
    const char* e = getenv("LITEKERN_PREFILL_KERNEL");
    return (e && std::string(e) == "single") ? 0 : 1;
  }();
  return v != 0;
}

// mma.sync kernel instead of tcgen05 (LITEKERN_PREFILL_MMA_SYNC=1, read once).
bool use_mma_sync() {
  static int v = [] {
    const char* e = getenv("LITEKERN_PREFILL_MMA_SYNC");
    return (e && atoi(e) != 0) ? 1 : 0;
  }();
  return v != 0;
}

}  // namespace

extern "C" size_t lk_paged_prefill_workspace_bytes(void) {
  return prefill_ws_bytes(lk::num_sms());
}

extern "C" int lk_paged_prefill_ws(void* out, const void* q, int64_t q_token_stride,
                                   const void* k_cache, const void* v_cache, int64_t num_blocks,
                                   const int32_t* block_tables, int64_t block_table_stride,
                                   const int32_t* cu_seqlens_q, const int32_t* context_lens,
                                   int32_t num_seqs, int32_t max_q_len, int32_t H, int32_t H_kv,
                                   int32_t D, int32_t block_size, float scale, int32_t dtype,
                                   void* workspace, size_t workspace_bytes, int32_t* status,
                                   void* stream) {
  if (workspace != nullptr &&
      ((reinterpret_cast<uintptr_t>(workspace) & 255u) || workspace_bytes < kPlanBytes))
    return workspace_bytes < kPlanBytes ? LK_ERR_INVALID_ARG : LK_ERR_ALIGNMENT;
  if (num_seqs < 0 || max_q_len < 0 || H <= 0 || H_kv <= 0 || H % H_kv != 0 || num_blocks <= 0)
    return LK_ERR_INVALID_ARG;
  if (num_seqs == 0 || max_q_len == 0) return LK_OK;
  if (!out || !q || !k_cache || !v_cache || !cu_seqlens_q) return LK_ERR_INVALID_ARG;
  if (num_seqs > 65535 || H_kv > 65535) return LK_ERR_INVALID_ARG;
  const int G = H / H_kv;
  if ((dtype != LK_DTYPE_BF16 && dtype != LK_DTYPE_F16) || D != kD ||
      (G != 1 && G != 2 && G != 4 && G != 8) || (block_tables && block_size % 16 != 0)) {
    // Shapes the tensor-core kernel does not take (fp32, other head dims, G,
    // or block sizes) run the generic CUDA-core kernel (no workspace needed).
    return lk_paged_attention_generic(out, static_cast<int64_t>(H) * D, q, q_token_stride,
                                      k_cache, v_cache, num_blocks, block_tables,
                                      block_table_stride, cu_seqlens_q, context_lens, num_seqs,
                                      max_q_len, H, H_kv, D, block_size, 0, scale, dtype, status,
                                      stream);
  }
  // Paged mode: num_blocks blocks of block_size slots. Contiguous mode: the
  // key tensor holds num_blocks tokens (block_size is ignored).
  int64_t num_slots;
  if (block_tables) {
    if (block_size <= 0 || block_size % 16 != 0) return LK_ERR_UNSUPPORTED;
    num_slots = num_blocks * block_size;
  } else {
    num_slots = num_blocks;
  }
  if (num_slots > 0x7fffffffLL) return LK_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(q) & 3u) || (q_token_stride & 1) ||
      (reinterpret_cast<uintptr_t>(out) & 3u))
    return LK_ERR_ALIGNMENT;
  CUtensorMap km, vm;
  int rc = lk::get_kv_tensor_map(&km, k_cache, num_slots, H_kv, D, dtype, 16, 1);
  if (rc != LK_OK) return rc;
  rc = lk::get_kv_tensor_map(&vm, v_cache, num_slots, H_kv, D, dtype, 16, 1);
  if (rc != LK_OK) return rc;
  PrefillParams p{};
  p.out = out;
  p.q = q;
  p.q_stride = q_token_stride;
  p.block_tables = block_tables;
  p.bt_stride = block_table_stride;
  p.cu_seqlens_q = cu_seqlens_q;
  p.context_lens = context_lens;
  p.num_slots = num_slots;
  p.num_blocks = block_tables ? num_blocks : 1;
  p.H = H;
  p.G = G;
  p.bs = block_tables ? block_size : 16;
  p.BQ = kRows / G;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.status = status;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!use_mma_sync() && use_pingpong()) {
    if (dtype == LK_DTYPE_BF16)
      return launch_prefill_pp<__nv_bfloat16>(km, vm, p, num_seqs, max_q_len, H_kv, workspace,
                                              workspace_bytes, s);
    return launch_prefill_pp<__half>(km, vm, p, num_seqs, max_q_len, H_kv, workspace,
                                     workspace_bytes, s);
  }
  if (!use_mma_sync()) {
    if (dtype == LK_DTYPE_BF16)
      return launch_prefill_tc<__nv_bfloat16>(km, vm, p, num_seqs, max_q_len, H_kv, s);
    return launch_prefill_tc<__half>(km, vm, p, num_seqs, max_q_len, H_kv, s);
  }
  if (dtype == LK_DTYPE_BF16)
    return launch_prefill<__nv_bfloat16>(km, vm, p, num_seqs, max_q_len, H_kv, s);
  return launch_prefill<__half>(km, vm, p, num_seqs, max_q_len, H_kv, s);
}

extern "C" int lk_paged_prefill(void* out, const void* q, int64_t q_token_stride,
                                const void* k_cache, const void* v_cache, int64_t num_blocks,
                                const int32_t* block_tables, int64_t block_table_stride,
                                const int32_t* cu_seqlens_q, const int32_t* context_lens,
                                int32_t num_seqs, int32_t max_q_len, int32_t H, int32_t H_kv,
                                int32_t D, int32_t block_size, float scale, int32_t dtype,
                                int32_t* status, void* stream) {
  return lk_paged_prefill_ws(out, q, q_token_stride, k_cache, v_cache, num_blocks, block_tables,
                             block_table_stride, cu_seqlens_q, context_lens, num_seqs, max_q_len,
                             H, H_kv, D, block_size, scale, dtype, nullptr, 0, status, stream);
}

namespace lk {

// Library-internal (no C export): the shared-prefix attention of
// lk_paged_decode_shared_prefix, on the ping-pong tensor-core kernel.
int prefix_attention(const void* q, int64_t q_stride, const void* k_cache, const void* v_cache,
                     int64_t num_blocks, const int32_t* block_table_row, int B, int H, int H_kv,
                     int block_size, int prefix_len, int prefix_split, int num_ranges,
                     float scale, float* part_ml, float* part_o, int part_splits, int dtype,
                     int32_t* status, int* zeroed_counter, cudaStream_t s) {
  const int G = H / H_kv;
  if (G != 1 && G != 2 && G != 4 && G != 8) return LK_ERR_UNSUPPORTED;
  const int64_t num_slots = num_blocks * block_size;
  CUtensorMap km, vm;
  int rc = lk::get_kv_tensor_map(&km, k_cache, num_slots, H_kv, kD, dtype, 16, 1);
  if (rc != LK_OK) return rc;
  rc = lk::get_kv_tensor_map(&vm, v_cache, num_slots, H_kv, kD, dtype, 16, 1);
  if (rc != LK_OK) return rc;
  PrefillParams p{};
  p.q = q;
  p.q_stride = q_stride;
  p.block_tables = block_table_row;
  p.bt_stride = 0;
  p.num_slots = num_slots;
  p.num_blocks = num_blocks;
  p.H = H;
  p.G = G;
  p.bs = block_size;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.status = status;
  p.num_seqs = num_ranges;
  p.prefix_rows = B;
  p.prefix_len = prefix_len;
  p.prefix_split = prefix_split;
  p.part_splits = part_splits;
  p.part_ml = part_ml;
  p.part_o = part_o;
  if (dtype == LK_DTYPE_BF16)
    return launch_prefix_pp<__nv_bfloat16>(km, vm, p, B, H_kv, zeroed_counter, s);
  return launch_prefix_pp<__half>(km, vm, p, B, H_kv, zeroed_counter, s);
}

}  // namespace lk
