"""The fused q/k RMSNorm + RoPE + KV store on the drop-in path
(model_hooks.fused_forward, bound by install(fused_rope=True)) against the
reference's own Qwen3Attention and LlamaAttention blocks: a 20-token prefill
that fills a paged cache, then one decode step over it, bf16, outputs and
cache from tests/golden/attn_block.npz (made by tests/golden/make_golden.py
on CPU). The fused kernel rotates in fp32 and rounds once where the
reference rounds each product to bf16, so the block outputs agree to bf16
precision: 2e-2 max-abs and 1e-2 mean-relative, the attention tolerance."""

import types

import pytest
import torch
import torch.nn as nn

from litevllm_b200 import model_hooks
from litevllm_b200.attention import Attention
from tests import golden_io
from tests.tolerance import assert_attn_close

pytestmark = pytest.mark.gpu


def _block(d, tag, cuda):
    hidden, H, H_kv, D, bs, S = (int(x) for x in d["shape"])
    m = types.SimpleNamespace(num_heads=H, num_kv_heads=H_kv, head_dim=D)

    def lin(name, n_in, n_out):
        layer = nn.Linear(n_in, n_out, bias=False, device=cuda, dtype=torch.bfloat16)
        with torch.no_grad():
            layer.weight.copy_(golden_io.bf16(d[f"{tag}.{name}.linear.weight"]))
        return layer

    m.q_proj, m.k_proj = lin("q_proj", hidden, H * D), lin("k_proj", hidden, H_kv * D)
    m.v_proj, m.o_proj = lin("v_proj", hidden, H_kv * D), lin("o_proj", H * D, hidden)
    m.use_qk_norm = f"{tag}.q_norm.weight" in d
    if m.use_qk_norm:
        eps = float(d[f"{tag}.eps"])
        m.q_norm = types.SimpleNamespace(weight=golden_io.bf16(d[f"{tag}.q_norm.weight"]).to(cuda),
                                         eps=eps)
        m.k_norm = types.SimpleNamespace(weight=golden_io.bf16(d[f"{tag}.k_norm.weight"]).to(cuda),
                                         eps=eps)
    m.rotary_emb = types.SimpleNamespace(cos_cached=golden_io.bf16(d[f"{tag}.cos"]).to(cuda),
                                         sin_cached=golden_io.bf16(d[f"{tag}.sin"]).to(cuda))
    m.attn = Attention(H, D, H_kv)
    return m, (hidden, H, H_kv, D, bs, S)


@pytest.mark.parametrize("tag", ["qwen3", "llama"])
def test_fused_block_matches_reference_prefill_then_decode(cuda, tag):
    d = golden_io.load("attn_block.npz")
    m, (hidden, H, H_kv, D, bs, S) = _block(d, tag, cuda)
    blocks = [int(b) for b in d["blocks"]]
    kc = torch.zeros((8, bs, H_kv, D), dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros_like(kc)
    x = golden_io.bf16(d[f"{tag}.x"]).to(cuda)
    x2 = golden_io.bf16(d[f"{tag}.x2"]).to(cuda)
    pos = torch.arange(S, device=cuda)
    slots = torch.tensor([blocks[p // bs] * bs + p % bs for p in range(S)], device=cuda)
    fwd = model_hooks.fused_forward
    with torch.no_grad():
        y = fwd(m, x, pos, (kc, vc), slots, None, None, True)
        y2 = fwd(m, x2, torch.tensor([S], device=cuda), (kc, vc),
                 torch.tensor([blocks[S // bs] * bs + S % bs], device=cuda),
                 torch.tensor([blocks], dtype=torch.int32, device=cuda),
                 torch.tensor([S + 1], dtype=torch.int32, device=cuda), False)
    assert y.dtype == torch.bfloat16 and y.shape == (S, hidden)
    assert_attn_close(y, torch.from_numpy(d[f"{tag}.y"]))
    assert_attn_close(y2, torch.from_numpy(d[f"{tag}.y2"]))
    # the cache the prefill and decode stored: the reference's, to bf16 rounding
    for name, got in (("k_cache", kc), ("v_cache", vc)):
        want = golden_io.bf16(d[f"{tag}.{name}"]).float()
        diff = (got.float().cpu() - want).abs()
        assert (diff <= 2.0 ** -7 + want.abs() * 2.0 ** -7).all(), (name, float(diff.max()))
