"""RMSNorm + rotary embedding oracle (torch, CPU). Test infrastructure only.

Restates, with the same dtype promotions and rounding points:
  LlamaRMSNorm.forward          litevllm/models/llama.py:18-27
      variance = x.float().pow(2).mean(-1); x * rsqrt(variance + eps)
      -> .to(weight.dtype) -> weight * x
  apply_rotary_emb              litevllm/layers/rotary_emb.py:104-117
      x1, x2 = halves; cat(x1 * cos - x2 * sin, x2 * cos + x1 * sin)
      (16-bit x times fp32 cos / sin: the result is fp32)
as applied in Qwen3Attention.forward (litevllm/models/qwen3.py:79-84).
"""

from __future__ import annotations

from typing import Optional

import torch


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    variance = x.float().pow(2).mean(-1, keepdim=True)
    y = x * torch.rsqrt(variance + eps)
    return weight * y.to(weight.dtype)


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [T, heads, D]; cos / sin [T, D/2] fp32 -> fp32 [T, heads, D]."""
    c, s = cos.unsqueeze(1), sin.unsqueeze(1)
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def norm_rope(x, cos, sin, weight: Optional[torch.Tensor] = None, eps: float = 1e-6):
    if weight is not None:
        x = rms_norm(x, weight, eps)
    return rope(x, cos, sin)
