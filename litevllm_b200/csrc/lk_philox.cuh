// In-kernel Gumbel noise shared by the sampler kernels.
//
// Bits: Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel Random Numbers:
// As Easy as 1, 2, 3", SC'11), keyed by the 64-bit seed, counter
// (v / 4, row, offset_lo, offset_hi); word v % 4 of the block feeds element v.
// The ten round keys depend on the seed alone, so the host computes them once
// per launch (PhiloxKey) and they reach the kernel in its parameter space,
// where every round's xor reads its key as a constant operand: a round is two
// 32x32->64-bit multiplies and two three-input xors.
//
// Uniform: u = ((r >> 9) + 0.5) * 2^-23, u in (0, 1), built from the bit
// pattern 1 + k * 2^-23 minus (1 - 2^-24) (both steps exact; no int->float
// conversion).
//
// Gumbel: g = -ln(-ln u), evaluated with the hardware base-2 logarithm
// (lg2.approx, absolute error about 2^-22) in two regimes so that g keeps an
// absolute error below 1e-6 everywhere:
//   u <= 3/4:  E = -ln u (|log2 u| >= 0.41, so E has relative error < 1e-6)
//              and g = -ln E;
//   u >  3/4:  t = 1 - u (exact) and g = -ln t - phi(t), where
//              phi(t) = ln(-ln(1 - t) / t) = t/2 + 5t^2/24 + ... is a degree-6
//              polynomial t * p5(t) fitted (Chebyshev, then monomial form) on
//              [0, 1/4] to 3e-8 (in fp32 Horner form). Computing -ln(1 - t) through ln u would lose
//              the small E = -ln u that the largest g come from.
// Both regimes are computed and one is selected, so a warp never diverges.
// Emulated in fp32 over all 2^23 uniforms with lg2 errors of +-2^-22, g is
// within 5e-7 relative (1.6e-6 absolute at g = 16, one fp32 ulp there) of
// the double-precision -ln(-ln u). Callers who need the exact bits read them
// back through the kernels' noise dump.
#pragma once

#include <stdint.h>

#include "lk_common.cuh"

namespace lk {

struct PhiloxKey {
  uint32_t k0[10], k1[10];
};

inline PhiloxKey philox_key(uint64_t seed) {
  PhiloxKey k;
  uint32_t a = static_cast<uint32_t>(seed), b = static_cast<uint32_t>(seed >> 32);
  for (int r = 0; r < 10; ++r) {
    k.k0[r] = a;
    k.k1[r] = b;
    a += 0x9E3779B9u;
    b += 0xBB67AE85u;
  }
  return k;
}

struct U4 {
  uint32_t x, y, z, w;
};

LK_DEVINL U4 philox4x32_10(U4 c, const PhiloxKey& k) {
  constexpr uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    // one 32 x 32 -> 64-bit product gives both halves
    const uint64_t p0 = static_cast<uint64_t>(M0) * c.x, p1 = static_cast<uint64_t>(M1) * c.z;
    const uint32_t hi0 = static_cast<uint32_t>(p0 >> 32), lo0 = static_cast<uint32_t>(p0);
    const uint32_t hi1 = static_cast<uint32_t>(p1 >> 32), lo1 = static_cast<uint32_t>(p1);
    c = U4{hi1 ^ c.y ^ k.k0[r], lo1, hi0 ^ c.w ^ k.k1[r], lo0};
  }
  return c;
}

LK_DEVINL float lg2_approx(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

LK_DEVINL float gumbel_from_bits(uint32_t r) {
  constexpr float kLn2 = 0.693147180559945309f;
  // 1 + k * 2^-23 in [1, 2), k = r >> 9
  const float one_k = __uint_as_float(0x3f800000u | (r >> 9));
  const float u = __fsub_rn(one_k, 0.99999994039535522f);  // - (1 - 2^-24): (k + 1/2) 2^-23
  const float t = __fsub_rn(1.f, u);                        // 1 - u, exact for u >= 1/2
  const float e = -kLn2 * lg2_approx(u);                    // -ln u
  // phi(t) / t on [0, 1/4], Horner
  float q = 0.10394973307847977f;
  q = fmaf(q, t, 0.049355968832969666f);
  q = fmaf(q, t, 0.08950251340866089f);
  q = fmaf(q, t, 0.1248493492603302f);
  q = fmaf(q, t, 0.20833708345890045f);
  q = fmaf(q, t, 0.4999999701976776f);
  const bool low = u <= 0.75f;
  const float z = low ? e : t;
  const float c = low ? 0.f : q * t;
  return fmaf(-kLn2, lg2_approx(z), -c);
}

}  // namespace lk
