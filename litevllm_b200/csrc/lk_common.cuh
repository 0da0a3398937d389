// Shared device helpers for liblitekern: status codes, dtype traits and thin
// inline-PTX wrappers for the sm_100a features the kernels use (mbarrier,
// bulk-tensor (TMA) loads, ldmatrix / movmatrix, mma.sync).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/litekern.h"

#define LK_DEVINL __device__ __forceinline__

namespace lk {

// ---------------------------------------------------------------- dtypes ---
template <typename T> struct Elem;
template <> struct Elem<float> {
  static constexpr int code = LK_DTYPE_F32;
  LK_DEVINL static float to_f(float x) { return x; }
};
template <> struct Elem<__half> {
  static constexpr int code = LK_DTYPE_F16;
  LK_DEVINL static float to_f(__half x) { return __half2float(x); }
};
template <> struct Elem<__nv_bfloat16> {
  static constexpr int code = LK_DTYPE_BF16;
  LK_DEVINL static float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
};

// Pack two fp32 values into one 32-bit register of 16-bit elements
// (lo -> bits 0..15), round to nearest even.
template <typename T> LK_DEVINL uint32_t pack2(float lo, float hi);
template <> LK_DEVINL uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <> LK_DEVINL uint32_t pack2<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// ------------------------------------------- programmatic dependent launch ---
// A kernel launched with lk::launch_after_previous may start while the kernel
// before it in the stream still runs. pdl_wait() blocks until that kernel has
// completed and its memory is visible (a no-op for an ordinary launch);
// pdl_launch_dependents() lets the next such kernel start launching now.
LK_DEVINL void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
LK_DEVINL void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------------ timeouts ---
// Every spin-wait in these kernels is bounded by wall time read from the
// global nanosecond timer; on expiry the waiter reports failure instead of
// hanging the SM.
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;  // 2 s

LK_DEVINL uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// -------------------------------------------------------------- mbarrier ---
LK_DEVINL uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

LK_DEVINL void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

LK_DEVINL void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

LK_DEVINL void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

LK_DEVINL void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

LK_DEVINL void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

LK_DEVINL bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete. Returns false when the
// wait exceeded kWaitTimeoutNs (the caller then flags an error and unwinds).
LK_DEVINL bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t timeout_ns = kWaitTimeoutNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t it = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++it & 255u) == 0 && globaltimer_ns() - t0 > timeout_ns) return false;
  }
  return true;
}

// 16-byte asynchronous global -> shared copy (cp.async, L2 only); with
// valid = false the destination is zero-filled and nothing is read.
LK_DEVINL void cp_async16(void* smem_dst, const void* gsrc, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)),
               "l"(gsrc), "r"(valid ? 16 : 0)
               : "memory");
}
LK_DEVINL void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// ------------------------------------------------------------------- TMA ---
// 3-D tiled bulk-tensor load global -> shared, completion signalled on an
// mbarrier via complete_tx. No multicast.
LK_DEVINL void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0,
                           int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// 1-D bulk copy global -> shared (both 16-byte aligned, size a multiple of
// 16), completion signalled on an mbarrier via complete_tx. No multicast.
LK_DEVINL void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Bulk-tensor prefetch of one box into L2 (no shared memory, no completion
// signal): used to put more bytes in flight than the shared-memory ring holds.
LK_DEVINL void tma_prefetch_3d(const CUtensorMap* map, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

LK_DEVINL void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// --------------------------------------------------------- warp matrices ---
LK_DEVINL void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
LK_DEVINL void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                         uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// Transpose an 8x8 matrix of 16-bit elements held one row-pair per lane.
LK_DEVINL uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// D += A(16x16) * B(16x8), fp32 accumulate.
template <typename T> LK_DEVINL void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                              uint32_t b1);
template <> LK_DEVINL void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4],
                                                   uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <> LK_DEVINL void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                            uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Byte offset of 16-byte chunk `chunk` (0..7) in row `row` of a tile written
// by TMA with CU_TENSOR_MAP_SWIZZLE_128B (128-byte rows, tile base 1024-byte
// aligned): the chunk index is XORed with the row index modulo 8.
LK_DEVINL uint32_t swz128(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

// 2^x on the special-function unit (single MUFU instruction, flush to zero).
LK_DEVINL float ex2_mufu(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32x2 arithmetic (sm_100): two lanes per instruction.
LK_DEVINL void ffma2(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0,
                     float c1) {
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}
LK_DEVINL void fadd2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// 2^x on the FMA / ALU pipes: x = n + f with n = round(x), f in [-1/2, 1/2];
// 2^f by a cubic least-squares fit on Chebyshev nodes (coefficients fitted
// for this library; max relative error 2.5e-4, below the rounding of the
// 16-bit attention probabilities it feeds); 2^n added to the exponent.
// Returns 0 for x < -126 (masked scores are -inf).
LK_DEVINL float exp2_fma(float x) {
  const float xc = fmaxf(x, -126.f);
  const float y = xc + 12582912.f;  // 1.5 * 2^23: integer part lands in the low bits
  const int n = __float_as_int(y) - 0x4B400000;
  const float f = xc - (y - 12582912.f);
  const float pf = fmaf(fmaf(fmaf(0.05746771767735481f, f, 0.24254462122917175f), f,
                             0.6928921341896057f),
                        f, 0.9999291300773621f);
  const float r = __int_as_float(__float_as_int(pf) + (n << 23));
  return x < -126.f ? 0.f : r;
}



// Three-input fp32 max (sm_100).
LK_DEVINL float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Named barrier over `count` threads (id 1..15; 0 is __syncthreads).
LK_DEVINL void named_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Named barrier that also ANDs a predicate over the participating threads.
LK_DEVINL bool named_sync_and(int id, int count, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %3, 0;\n\t"
      "barrier.cta.red.and.pred p, %1, %2, q;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(id), "r"(count), "r"(static_cast<uint32_t>(v))
      : "memory");
  return r != 0;
}


LK_DEVINL float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}


// ------------------------------------------------------------- tcgen05 ---
// Fifth-generation tensor core (UMMA) helpers: TMEM allocation, MMA issue
// with shared-memory matrix descriptors, completion through mbarriers, and
// TMEM <-> register moves. cta_group::1 throughout (no CTA pairs, no
// multicast).
namespace tc {

// Shared-memory matrix descriptor (sm_100): start address, leading- and
// stride-dimension byte offsets (all >> 4), descriptor version 1, 128-byte
// swizzle layout. The swizzle atoms (8 rows x 128 B) must be 1024-byte aligned.
LK_DEVINL uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) |
         (static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// Shared-memory matrix descriptor with a 32-byte swizzle, K-major: a K = 16
// (32-byte) slice of R rows is one contiguous R x 32-byte block, 8-row groups
// sbo_bytes apart (256 when packed); the leading offset is unused.
LK_DEVINL uint64_t smem_desc_sw32(uint32_t saddr, uint32_t sbo_bytes) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (1ull << 16) |
         (static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (6ull << 61);
}

// Instruction descriptor for kind::f16 with fp32 accumulation.
// fmt: 0 = f16, 1 = bf16 (A and B the same type); major: 0 = K-major, 1 = MN-major.
LK_DEVINL constexpr uint32_t idesc_f16(int fmt, int a_major, int b_major, int M, int N) {
  return (1u << 4) | (static_cast<uint32_t>(fmt) << 7) | (static_cast<uint32_t>(fmt) << 10) |
         (static_cast<uint32_t>(a_major) << 15) | (static_cast<uint32_t>(b_major) << 16) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

LK_DEVINL void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Same with the A operand in TMEM (a_tmem: lane = row, each 32-bit column
// holds two consecutive 16-bit K values, the lower index in the low half).
LK_DEVINL void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on the mbarrier when all previously issued tcgen05 ops of
// this thread have completed.
LK_DEVINL void commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

LK_DEVINL void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
LK_DEVINL void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Whole-warp TMEM allocation; the base address is written to *slot (smem).
LK_DEVINL void alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
LK_DEVINL void dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// 32 lanes x 32 columns of 32-bit values: lane i of the warp gets TMEM lane
// (taddr lane + i), columns col..col+31.
LK_DEVINL void ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
LK_DEVINL void st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
LK_DEVINL void st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}
LK_DEVINL void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
LK_DEVINL void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

}  // namespace tc
}  // namespace lk
