"""Drop-in replacement for litevllm.layers.sampler.Sampler.

`Sampler.sample(logits, sampling_params, past_token_ids=None)` keeps the
reference signature (litevllm/layers/sampler.py:147-187):

* repetition penalty -> liblitekern fused kernel on a clone of the logits, the
  reference's arithmetic and dedupe (:190-201);
* temperature 0 -> liblitekern greedy argmax (replaces _argmax_kernel);
* top-k / top-p -> fused liblitekern filter + Gumbel-max draw (same kept set
  and distribution as :204-225; fp32, f16 and bf16 logits), no probability
  tensor, no sort;
* otherwise -> liblitekern Gumbel-max with in-kernel Philox noise: one pass,
  no probability tensor. The seed is drawn from torch's CPU generator, so
  torch.manual_seed makes it reproducible; sampling_params.seed, when set,
  is used instead.

`Sampler.sample_batch` is the batched, per-row-temperature entry the engine
calls once per step.
"""

from __future__ import annotations

import threading
from typing import Optional

import torch

from . import ops


class Sampler:
    """Stateless (apart from an RNG call counter) sampler."""

    _offset = 0
    _lock = threading.Lock()

    @classmethod
    def _next_offset(cls) -> int:
        with cls._lock:
            cls._offset += 1
            return cls._offset

    @staticmethod
    def _seed(sampling_params=None) -> int:
        s = getattr(sampling_params, "seed", None)
        if s is not None:
            return int(s)
        return int(torch.randint(0, 2**62, (1,)).item())

    @staticmethod
    def sample(logits: torch.Tensor, sampling_params, past_token_ids: Optional[torch.Tensor] = None):
        if logits.dim() == 1:
            logits = logits.unsqueeze(0)
        if past_token_ids is not None and sampling_params.repetition_penalty != 1.0:
            logits = ops.repetition_penalty_(
                logits.clone(memory_format=torch.contiguous_format), past_token_ids,
                sampling_params.repetition_penalty,
            )
        B = logits.shape[0]
        T = float(sampling_params.temperature)
        if T == 0.0:
            return ops.sample(logits)
        temps = torch.full((B,), T, dtype=torch.float32, device=logits.device)
        if sampling_params.top_k > 0 or sampling_params.top_p < 1.0:
            # fused: filter + Gumbel-max in one launch, no probability tensor
            ks = torch.full((B,), int(sampling_params.top_k), dtype=torch.int32,
                            device=logits.device)
            ps = torch.full((B,), float(sampling_params.top_p), dtype=torch.float32,
                            device=logits.device)
            return ops.sample_filtered(logits, temps, ks, ps,
                                       seed=Sampler._seed(sampling_params),
                                       offset=Sampler._next_offset())
        return ops.sample(
            logits, temps, seed=Sampler._seed(sampling_params), offset=Sampler._next_offset()
        )

    # north-star alias
    forward = sample

    @staticmethod
    def sample_batch(
        logits: torch.Tensor,
        temperatures: Optional[torch.Tensor] = None,
        noise: Optional[torch.Tensor] = None,
        seed: Optional[int] = None,
        offset: Optional[int] = None,
        noise_dump: Optional[torch.Tensor] = None,
        out: Optional[torch.Tensor] = None,
        top_k: Optional[torch.Tensor] = None,
        top_p: Optional[torch.Tensor] = None,
    ) -> torch.Tensor:
        """One sampler launch for a whole step: rows with temperature 0 are
        greedy, the others Gumbel-max at their own temperature; with per-row
        top_k (int32, <= 0 off) / top_p (fp32, >= 1 off) the fused filtered
        kernel runs instead."""
        if temperatures is not None and temperatures.dtype != torch.float32:
            temperatures = temperatures.float()
        if top_k is not None or top_p is not None:
            if temperatures is None:
                temperatures = torch.zeros(logits.shape[0], dtype=torch.float32,
                                           device=logits.device)
            return ops.sample_filtered(
                logits, temperatures, top_k, top_p, noise=noise,
                seed=Sampler._seed() if seed is None else seed,
                offset=Sampler._next_offset() if offset is None else offset, out=out)
        return ops.sample(
            logits,
            temperatures,
            noise=noise,
            seed=Sampler._seed() if seed is None else seed,
            offset=Sampler._next_offset() if offset is None else offset,
            noise_dump=noise_dump,
            out=out,
        )
