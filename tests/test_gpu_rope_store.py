"""Fused q/k RMSNorm + RoPE + KV store vs the reference (golden) and the oracle.

The reference produces fp32 rotated q / k (16-bit x fp32 cos); the kernel
rounds once to the 16-bit activation dtype, the rounding the store applies to
k anyway. Parity: at least 98 % of the values bit-identical to the rounded
reference and every value within 2^-7 (one bf16 ulp at magnitude 1) plus one
ulp of its own magnitude: rsqrt and the order of the variance sum can move a
normalised input across a rounding boundary, and the rotation can cancel, so
an input ulp may be large relative to a small output."""

import pytest
import torch

from litevllm_b200 import ops
from oracle import rope as orope
from tests import golden_io

pytestmark = pytest.mark.gpu


def _close_16bit(got: torch.Tensor, ref_fp32: torch.Tensor):
    ref = ref_fp32.to(got.dtype).float()
    got = got.float().cpu()
    tol = 2.0 ** -7 + ref.abs() * 2.0 ** -7
    diff = (got - ref).abs()
    assert (diff <= tol).all(), float(diff.max())
    assert (diff == 0).float().mean() >= 0.98


def test_norm_rope_store_matches_reference_golden(cuda):
    d = golden_io.load("rope.npz")
    q, k = golden_io.bf16(d["q"]).to(cuda), golden_io.bf16(d["k"]).to(cuda)
    T, H, D = q.shape
    H_kv = k.shape[1]
    v = torch.randn((T, H_kv, D), device=cuda).bfloat16()
    cos, sin = torch.from_numpy(d["cos"]).to(cuda), torch.from_numpy(d["sin"]).to(cuda)
    pos = torch.arange(T, device=cuda)  # the table holds only the used positions' rows
    kc = torch.zeros((4, 16, H_kv, D), device=cuda, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slots = torch.tensor([5, 0, 63, 17, 33, 2, 40, 41, 9], device=cuda)
    qo = ops.rope_store_kvcache(q, k, v, kc, vc, slots, pos, cos, sin,
                                golden_io.bf16(d["q_w"]).to(cuda), golden_io.bf16(d["k_w"]).to(cuda),
                                float(d["eps"]))
    _close_16bit(qo, torch.from_numpy(d["q_out"]))
    _close_16bit(kc.view(-1, H_kv, D)[slots], torch.from_numpy(d["k_out"]))
    assert torch.equal(vc.view(-1, H_kv, D)[slots], v)


@pytest.mark.parametrize("with_norm", [False, True])
def test_rope_store_random_matches_oracle(cuda, with_norm):
    g = torch.Generator().manual_seed(3)
    T, H, H_kv, D, maxp = 300, 32, 8, 128, 2048
    inv = 1.0 / (500000.0 ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
    freqs = torch.outer(torch.arange(maxp, dtype=torch.float32), inv)
    cos, sin = freqs.cos(), freqs.sin()
    pos = torch.randint(0, maxp, (T,), generator=g)
    q = torch.randn((T, H, D), generator=g).bfloat16()
    k = torch.randn((T, H_kv, D), generator=g).bfloat16()
    v = torch.randn((T, H_kv, D), generator=g).bfloat16()
    qw = (1 + 0.1 * torch.randn(D, generator=g)).bfloat16() if with_norm else None
    kw = (1 + 0.1 * torch.randn(D, generator=g)).bfloat16() if with_norm else None
    qref = orope.norm_rope(q, cos[pos], sin[pos], qw, 1e-6)
    kref = orope.norm_rope(k, cos[pos], sin[pos], kw, 1e-6)
    kc = torch.zeros((32, 16, H_kv, D), device=cuda, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slots = torch.randperm(512, generator=g)[:T].to(cuda)
    qo = ops.rope_store_kvcache(q.to(cuda), k.to(cuda), v.to(cuda), kc, vc, slots, pos.to(cuda),
                                cos.to(cuda), sin.to(cuda),
                                None if qw is None else qw.to(cuda),
                                None if kw is None else kw.to(cuda))
    _close_16bit(qo, qref)
    _close_16bit(kc.view(-1, H_kv, D)[slots], kref)
    assert torch.equal(vc.view(-1, H_kv, D)[slots].cpu(), v)
