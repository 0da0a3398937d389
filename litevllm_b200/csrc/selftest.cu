// Self-test of the failure path every bounded wait in this library takes:
// one CTA waits on an mbarrier that nothing ever arrives on, with the given
// time limit, and reports LK_STATUS_WAIT_TIMEOUT in *status instead of
// hanging. The kernel then returns normally and the context stays usable.
#include "lk_common.cuh"
#include "lk_host.h"

namespace {

__global__ void wait_timeout_kernel(int32_t* status, uint64_t timeout_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    lk::mbar_init(&bar, 1);
    lk::fence_barrier_init();
  }
  __syncthreads();
  // parity 0 of a fresh barrier completes only after one arrival: none comes
  if (!lk::mbar_wait(&bar, 0, timeout_ns)) {
    if (threadIdx.x == 0) atomicOr(status, LK_STATUS_WAIT_TIMEOUT);
  }
}

}  // namespace

extern "C" int lk_selftest_wait_timeout(int32_t* status, uint64_t timeout_ns, void* stream) {
  if (!status || timeout_ns == 0 || timeout_ns > 100000000ull) return LK_ERR_INVALID_ARG;
  wait_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status, timeout_ns);
  return lk::check_launch();
}

// Issue rate of the fifth-generation tensor core, the figure the prefill
// kernel's tile shapes are chosen by: one CTA per SM, one thread issues
// n_mma back-to-back tcgen05.mma (kind::f16, bf16 operands, fp32 accumulator
// in TMEM, M = 128) of one shape, then commits and waits on an mbarrier
// (bounded); cycles[cta] receives the SM clock cycles from the first issue to
// the completion. Shapes: 0 = A and B from shared memory, N = 128; 1 = the
// same with N = 256; 2 = A from TMEM, N = 128; 3 = A from TMEM, B N-major
// (d contiguous, as the V tile of P.V), N = 128; 4 = A from shared memory and
// B N-major, N = 128. The operands are whatever the
// shared memory and TMEM hold: only the rate is measured.
namespace {

constexpr int kMmaSmem = 16384 + 32768 + 1024;  // A 128 x 64, B 256 x 64 bf16 (SW128), align

__global__ void __launch_bounds__(128) mma_rate_kernel(int n_mma, int shape, int64_t* cycles,
                                                      int32_t* status) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t done;
  __shared__ uint32_t tmem_slot;
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t a_addr = lk::smem_u32(base), b_addr = a_addr + 16384;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    lk::mbar_init(&done, 1);
    lk::fence_barrier_init();
  }
  if (warp == 0) lk::tc::alloc(&tmem_slot, 512);
  lk::tc::fence_before();
  __syncthreads();
  lk::tc::fence_after();
  const uint32_t tmem = tmem_slot;
  // shapes 8-15: shapes 0-7 with consecutive MMAs rotating over independent
  // accumulators (4 for N = 128 from shared memory, 2 otherwise), so no MMA
  // waits for the previous one's result
  const bool rotate = shape >= 8;
  shape &= 7;
  const int N = (shape == 1 || shape == 7) ? 256 : 128;
  const bool a_tmem = shape == 2 || shape == 3;
  const int nacc = !rotate ? 1 : (N == 128 && !a_tmem) ? 4 : 2;
  if (threadIdx.x == 0) {
    const uint32_t idesc = lk::tc::idesc_f16(1, 0, 0, 128, N);
    const long long t0 = clock64();
    for (int i = 0; i < n_mma; ++i) {
      const int ks = i & 3;  // the four K = 16 steps of one 64-wide swizzle atom
      const uint32_t d = tmem + static_cast<uint32_t>((i % nacc) * N);
      const uint64_t bd = lk::tc::smem_desc_sw128(b_addr + ks * 32, 16, 1024);
      if (shape == 5)  // B K-major with a 32-byte swizzle: each K step one 4 KiB block
        lk::tc::mma_f16(d, lk::tc::smem_desc_sw128(a_addr + ks * 32, 16, 1024),
                        lk::tc::smem_desc_sw32(b_addr + ks * 4096, 256), idesc, 1u);
      else if (shape == 6)  // A and B K-major with a 32-byte swizzle
        lk::tc::mma_f16(d, lk::tc::smem_desc_sw32(a_addr + ks * 4096, 256),
                        lk::tc::smem_desc_sw32(b_addr + ks * 4096, 256), idesc, 1u);
      else if (shape == 7)  // N = 256, B with a 32-byte swizzle (8 KiB per K step)
        lk::tc::mma_f16(d, lk::tc::smem_desc_sw128(a_addr + ks * 32, 16, 1024),
                        lk::tc::smem_desc_sw32(b_addr + ks * 8192, 256), idesc, 1u);
      else if (shape == 4)  // A from shared memory, B N-major
        lk::tc::mma_f16(d, lk::tc::smem_desc_sw128(a_addr + ks * 32, 16, 1024),
                        lk::tc::smem_desc_sw128(b_addr + ks * 2048, 16384, 1024),
                        lk::tc::idesc_f16(1, 0, 1, 128, 128), 1u);
      else if (shape == 3)  // the P.V form: B holds 16 keys x 128 d, d contiguous (MN-major)
        lk::tc::mma_f16_ts(d, tmem + 256 + ks * 8,
                           lk::tc::smem_desc_sw128(b_addr + ks * 2048, 16384, 1024),
                           lk::tc::idesc_f16(1, 0, 1, 128, 128), 1u);
      else if (shape == 2)
        lk::tc::mma_f16_ts(d, tmem + 256 + ks * 8, bd, idesc, 1u);
      else
        lk::tc::mma_f16(d, lk::tc::smem_desc_sw128(a_addr + ks * 32, 16, 1024), bd, idesc, 1u);
    }
    lk::tc::commit(&done);
    const bool ok = lk::mbar_wait(&done, 0, 100000000ull);  // 100 ms
    const long long t1 = clock64();
    cycles[blockIdx.x] = ok ? static_cast<int64_t>(t1 - t0) : -1;
    if (!ok && status) atomicOr(status, LK_STATUS_WAIT_TIMEOUT);
  }
  lk::tc::fence_before();
  __syncthreads();
  lk::tc::fence_after();
  if (warp == 0) lk::tc::dealloc(tmem, 512);
}

}  // namespace

extern "C" int lk_selftest_mma_rate(int32_t n_mma, int32_t shape, int64_t* cycles,
                                    int32_t* status, void* stream) {
  if (!cycles || n_mma <= 0 || n_mma > (1 << 20) || shape < 0 || shape > 15)
    return LK_ERR_INVALID_ARG;
  static bool configured[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return LK_ERR_CUDA;
  if (!configured[dev]) {
    if (cudaFuncSetAttribute(mma_rate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kMmaSmem) != cudaSuccess)
      return LK_ERR_CUDA;
    configured[dev] = true;
  }
  mma_rate_kernel<<<lk::num_sms(), 128, kMmaSmem, static_cast<cudaStream_t>(stream)>>>(
      n_mma, shape, cycles, status);
  return lk::check_launch();
}
