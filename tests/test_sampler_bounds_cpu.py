"""The in-kernel-noise sampler's skip bounds, checked exhaustively on the CPU.

gumbel_segment (litevllm_b200/csrc/sampler.cu) skips a vector of 8 logits
when fl(qu + fl(h(u_max) + 1e-3)) is below a key already reached, where
  qu = fma(|q0|, 2^-22, q0), q0 = fl(x_max * RN(1/T))   (not the IEEE quotient)
  h(u) = -ln(1 - u)                                       (not the Gumbel map g)
and every key is fl(fl(x / T) + g(u)) with IEEE division. fl(a + b) is
monotone in a and b, so the skip drops no vector that could win or tie as
long as qu >= fl(x_max / T) and h(u) + 1e-3 >= g(u) beyond the two maps'
computed errors (a few 1e-6). These tests replay the kernel's fp32 steps in
numpy for every 16-bit logit value (bf16 and fp16) at a spread of
temperatures, and for all 2^23 uniforms the kernel can draw.
"""

import numpy as np
import pytest

from oracle import sampler as osamp

_TEMPS = np.concatenate([
    np.geomspace(1e-3, 1e3, 61),
    [0.05, 0.1, 0.3, 0.5, 0.7, 0.9, 1.0, 1.1, 1.5, 2.0, 30.0, 0.3333333, 1.0 / 7.0],
]).astype(np.float32)


def _all_16bit(kind: str) -> np.ndarray:
    bits = np.arange(1 << 16, dtype=np.uint32)
    if kind == "bf16":
        x = (bits << np.uint32(16)).view(np.float32)
    else:
        x = bits.astype(np.uint16).view(np.float16).astype(np.float32)
    return x[np.isfinite(x)]


def _quotient_bound(x: np.ndarray, t: np.float32) -> np.ndarray:
    """The kernel's qu in fp32: q0 = RN(x * RN(1/T)); fma(|q0|, 2^-22, q0)."""
    y = np.float32(1.0) / t
    q0 = (x * y).astype(np.float32)
    # q0 and q0 * 2^-22 fit a float64 sum exactly (46 significant bits), so
    # one rounding to fp32 is the fused multiply-add's
    return (q0.astype(np.float64) + np.abs(q0).astype(np.float64) * 2.0**-22).astype(np.float32)


@pytest.mark.parametrize("kind", ["bf16", "fp16"])
def test_quotient_bound_covers_ieee_division(kind):
    x = _all_16bit(kind)
    with np.errstate(over="ignore", invalid="ignore"):
        for t in _TEMPS:
            q = (x / t).astype(np.float32)   # IEEE fp32 division, as the keys use
            qu = _quotient_bound(x, t)
            # a product that overflows to -inf gives fma(inf, 2^-22, -inf) = NaN:
            # a NaN bound never compares below the threshold, so the vector is
            # always computed (safe). A subnormal quotient can come out a few
            # subnormal steps (~1e-45) short: the bound's 1e-3 margin on the
            # noise side covers any shortfall that far below it; normal
            # results must be covered outright.
            normal = np.abs(q) >= np.float32(2.0**-126)
            ok = (qu >= q) | np.isnan(qu) | (~normal & ((q - qu) < np.float32(1e-30)))
            assert ok.all(), (kind, float(t), x[~ok][:4], q[~ok][:4], qu[~ok][:4])


def _kernel_uniforms():
    """u and t = 1 - u exactly as the kernel forms them from r >> 9 = k."""
    k = np.arange(1 << 23, dtype=np.uint32)
    one_k = (np.uint32(0x3F800000) | k).view(np.float32)          # 1 + k 2^-23
    u = (one_k - np.float32(0.99999994039535522)).astype(np.float32)
    t = (np.float32(1.0) - u).astype(np.float32)
    return k, u, t


def test_uniforms_match_the_oracle():
    k, u, _ = _kernel_uniforms()
    assert np.array_equal(u, osamp.uniform_bits_to_u(k << np.uint32(9)))


def test_one_log_bound_is_above_the_gumbel_map():
    _, u, t = _kernel_uniforms()
    g = -np.log(-np.log(u.astype(np.float64)))   # the map the keys use, exactly
    h = -np.log(t.astype(np.float64))            # the bound, from the kernel's fp32 t
    gap = h - g
    # h >= g everywhere; where u is near 1 the two meet (h - g ~ (1 - u) / 2),
    # and the 1e-3 margin then covers both maps' computed errors (a few 1e-6)
    assert gap.min() >= 0.0, gap.min()
    assert (gap + 1e-3).min() > 1e-4
    # the logits-only test uses the largest noise the map gives: every bit set
    g_cap = float(osamp.gumbel_from_u(osamp.uniform_bits_to_u(np.array([0xFFFFFFFF], np.uint32)))[0])
    assert g_cap >= g.max() - 1e-5 and 16.0 < g_cap < 17.0
