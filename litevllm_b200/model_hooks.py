"""Fused q/k RMSNorm + RoPE + KV store on the drop-in path.

Qwen3Attention.forward (litevllm/models/qwen3.py:63-93) and
LlamaAttention.forward (litevllm/models/llama.py:68-97) run, between the
q/k/v projections and attention, the q/k RMSNorm (Qwen3 only), the rotary
embedding of q and k, and the KV-cache store as separate torch ops. The
replacement forward below does those three steps in one launch
(lk_rope_store_kv) and then calls the (already replaced) Attention without
a second store. Shapes the fused kernel does not take (head_dim != 128,
non-16-bit activations) run the module's original forward unchanged.

The fused kernel rotates in fp32 from the module's cos / sin tables (a bf16
model holds them in bf16; they are widened once per module, exactly) and
rounds once, where the reference rounds each product to the activation dtype:
the results agree to the activations' precision (tested against the
reference's own blocks).
"""

from __future__ import annotations

import importlib

import torch

from . import ops

_ORIGINAL: dict = {}


def _tables(rot) -> tuple:
    """fp32 copies of a RotaryEmbedding's cos / sin tables, cached on the
    module and rebuilt if the buffers move or change dtype."""
    key = (rot.cos_cached.data_ptr(), rot.cos_cached.dtype, rot.cos_cached.device)
    cached = getattr(rot, "_litekern_tables", None)
    if cached is None or cached[0] != key:
        cached = (key, rot.cos_cached.float().contiguous(), rot.sin_cached.float().contiguous())
        rot._litekern_tables = cached
    return cached[1], cached[2]


def fused_forward(self, hidden_states, positions, kv_cache=None, slot_mapping=None,
                  block_table=None, context_lens=None, is_prefill=True):
    """Qwen3Attention / LlamaAttention forward with the norm, rotation and
    store fused (same signature and result as the reference forward)."""
    if (self.head_dim != 128 or hidden_states.dtype not in (torch.bfloat16, torch.float16)
            or not hidden_states.is_cuda):
        return _ORIGINAL[type(self)](self, hidden_states, positions, kv_cache, slot_mapping,
                                     block_table, context_lens, is_prefill)
    T = hidden_states.shape[0]
    q = self.q_proj(hidden_states).view(T, self.num_heads, self.head_dim)
    k = self.k_proj(hidden_states).view(T, self.num_kv_heads, self.head_dim)
    v = self.v_proj(hidden_states).view(T, self.num_kv_heads, self.head_dim)
    qw = kw = None
    eps = 1e-6
    if getattr(self, "use_qk_norm", False):
        qw, kw, eps = self.q_norm.weight, self.k_norm.weight, float(self.q_norm.eps)
    cos, sin = _tables(self.rotary_emb)
    key_cache, value_cache = kv_cache if kv_cache is not None else (None, None)
    store = slot_mapping is not None and key_cache is not None
    # attention over the new tokens alone reads the rotated k itself
    contiguous = block_table is None
    ops.rope_store_kvcache(q, k, v, key_cache if store else None,
                           value_cache if store else None, slot_mapping if store else None,
                           positions, cos, sin, qw, kw, eps, key_out=k if contiguous else None)
    attn_output = self.attn(q, k, v, key_cache=key_cache, value_cache=value_cache,
                            block_table=block_table, slot_mapping=None,
                            context_lens=context_lens, is_prefill=is_prefill)
    return self.o_proj(attn_output.reshape(T, -1))


_SITES = (("litevllm.models.qwen3", "Qwen3Attention"), ("litevllm.models.llama", "LlamaAttention"))


def install() -> list[str]:
    """Rebind the forward of the reference attention blocks that import."""
    patched = []
    for mod_name, cls_name in _SITES:
        try:
            cls = getattr(importlib.import_module(mod_name), cls_name)
        except Exception:
            continue
        if cls.forward is not fused_forward:
            _ORIGINAL[cls] = cls.forward
            cls.forward = fused_forward
        patched.append(f"{mod_name}.{cls_name}.forward")
    return patched
