"""Drop-in replacements for litevllm.layers.attention (Attention, PagedAttention).

Same constructor and forward signature as the reference
(litevllm/layers/attention.py:68-89), so Qwen3Attention / LlamaAttention
(models/qwen3.py:87-92, models/llama.py:90-97) call it unchanged. Every path
runs the liblitekern CUDA kernels; there is no PyTorch or CPU fallback.
"""

from __future__ import annotations

import os
from typing import Callable, Optional

import torch
import torch.nn as nn

from . import ops

# Mixed steps run the decode rows on a side stream next to the prefill chunks
# (LITEKERN_MIXED_OVERLAP=0: one after the other on the caller's stream).
MIXED_OVERLAP = os.environ.get("LITEKERN_MIXED_OVERLAP", "1") != "0"
_SIDE_STREAMS: dict = {}


def run_overlapped(first: Callable[[], None], second: Callable[[], None]) -> None:
    """Run first() on the current stream and second() on a per-device side
    stream forked from it, then join: the current stream continues only when
    both are done. first() is launched first, so its grid takes the SMs and
    second()'s blocks fill each SM as first()'s blocks retire (the persistent
    prefill kernel's tail, where items run out unevenly, is then not idle).
    Tensors second() reads or writes need no record_stream: the join orders
    every later use on the current stream after them."""
    main = torch.cuda.current_stream()
    dev = main.device
    side = _SIDE_STREAMS.get(dev)
    if side is None:
        side = _SIDE_STREAMS[dev] = torch.cuda.Stream(device=dev)
    side.wait_stream(main)
    first()
    with torch.cuda.stream(side):
        second()
    main.wait_stream(side)

# Shared-prefix hint for the current decode step, set by the engine hook that
# builds the step's block tables (engine_hooks.prepare_inputs): the tensor it
# applies to and the number of leading tokens every row shares (full blocks).
# Attention.forward uses the shared-prefix decode only for that exact tensor.
_SHARED_PREFIX = {"table": None, "tokens": 0}
# Below these, the per-row decode kernel is as fast.
SHARED_PREFIX_MIN_TOKENS = 256
SHARED_PREFIX_MIN_ROWS = 4


# Mixed-step hint, set by engine_hooks.prepare_inputs_mixed for a step whose
# batch holds prefill chunks (rows [0, num_prefill_tokens) of every layer's
# q / k / v, packed by cu_seqlens_q) followed by one decode token per
# sequence. The model's layers pass the step's block_tables tensor to
# Attention.forward unchanged; a call with that exact tensor runs
# forward_mixed with the hint's layout (the reference's call signature has
# no room for it).
_MIXED_STEP = {"table": None}


def set_mixed_step_hint(block_tables: Optional[torch.Tensor], cu_seqlens_q=None,
                        num_prefill_seqs: int = 0, num_prefill_tokens: int = 0,
                        max_q_len: int = 0) -> None:
    """Declare the mixed layout of the step whose table is `block_tables`
    (None clears the hint)."""
    _MIXED_STEP.clear()
    _MIXED_STEP.update(table=block_tables, cu_seqlens_q=cu_seqlens_q, P=int(num_prefill_seqs),
                       TP=int(num_prefill_tokens), max_q_len=int(max_q_len))


def set_shared_prefix_hint(block_tables: Optional[torch.Tensor], prefix_tokens: int) -> None:
    """Declare that every row of `block_tables` starts with the same
    `prefix_tokens` tokens (whole, filled blocks); None clears the hint."""
    _SHARED_PREFIX["table"] = block_tables
    _SHARED_PREFIX["tokens"] = int(prefix_tokens) if block_tables is not None else 0


class PagedAttention:
    """Static helpers with the reference's names (attention.py:14-65)."""

    @staticmethod
    def write_to_cache(
        key: torch.Tensor,
        value: torch.Tensor,
        key_cache: torch.Tensor,
        value_cache: torch.Tensor,
        slot_mapping: torch.Tensor,
    ) -> None:
        """key_cache[slot // bs, slot % bs] = key (attention.py:18-33)."""
        ops.store_kvcache(key, value, key_cache, value_cache, slot_mapping)

    # north-star alias
    store_kvcache = write_to_cache


def store_kvcache(key, value, key_cache, value_cache, slot_mapping) -> None:
    """Module-level alias of the KV store (north-star name)."""
    ops.store_kvcache(key, value, key_cache, value_cache, slot_mapping)


class Attention(nn.Module):
    """Attention over the paged KV cache (reference: attention.py:68-151)."""

    def __init__(self, num_heads, head_dim, num_kv_heads, scale=None):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.num_kv_heads = num_kv_heads
        self.num_kv_groups = num_heads // num_kv_heads
        self.scale = scale or (1.0 / (head_dim**0.5))

    def forward(
        self,
        query,
        key,
        value,
        key_cache,
        value_cache,
        block_table,
        slot_mapping,
        context_lens,
        is_prefill=True,
        cu_seqlens_q: Optional[torch.Tensor] = None,
        max_q_len: Optional[int] = None,
    ):
        """Store the new K/V, then prefill or decode attention.

        Reference semantics (attention.py:77-89): the store runs when
        slot_mapping is given; prefill with block_table None attends the new
        tokens only, causally (one sequence, _prefill); decode reads the
        paged history (_decode_fast). Extension: prefill with block_table,
        context_lens and cu_seqlens_q attends prior paged context plus the
        chunk, for several sequences at once.
        """
        mixed = _MIXED_STEP
        if block_table is not None and block_table is mixed["table"]:
            # a merged prefill + decode step (engine_hooks.prepare_inputs_mixed)
            return self.forward_mixed(
                query, key, value, key_cache, value_cache, block_table, slot_mapping,
                context_lens, mixed["cu_seqlens_q"], mixed["P"], mixed["TP"], mixed["max_q_len"])

        if slot_mapping is not None and key_cache is not None:
            ops.store_kvcache(key, value, key_cache, value_cache, slot_mapping)

        if is_prefill:
            if block_table is None:
                S = query.shape[0]
                cu = torch.tensor([0, S], dtype=torch.int32, device=query.device)
                # SDPA's default scale 1/sqrt(D), as the reference's _prefill uses.
                return ops.paged_prefill(
                    query, key, value, cu, S, 1.0 / (self.head_dim**0.5)
                )
            if cu_seqlens_q is None:
                # one sequence whose chunk is the whole query
                S = query.shape[0]
                cu_seqlens_q = torch.tensor([0, S], dtype=torch.int32, device=query.device)
                max_q_len = S
            if max_q_len is None:
                # an upper bound, known on the host: reading the longest chunk
                # back from cu_seqlens_q would wait for the device; query tiles
                # past a chunk's end take no work
                max_q_len = query.shape[0]
            return ops.paged_prefill(
                query, key_cache, value_cache, cu_seqlens_q, max_q_len, self.scale,
                block_tables=block_table, context_lens=context_lens,
            )

        pref = _SHARED_PREFIX["tokens"]
        if (
            pref >= SHARED_PREFIX_MIN_TOKENS
            and block_table is _SHARED_PREFIX["table"]
            and query.shape[0] >= SHARED_PREFIX_MIN_ROWS
            and ops.tuned_attention_shape(query.dtype, self.head_dim, key_cache.shape[1],
                                          self.num_kv_groups)
        ):
            # the rows share their first `pref` tokens: compute them once
            return ops.paged_decode_shared_prefix(
                query, key_cache, value_cache, block_table, context_lens, self.scale, pref
            )
        return ops.paged_decode(
            query, key_cache, value_cache, block_table, context_lens, self.scale
        )

    def forward_mixed(
        self,
        query: torch.Tensor,
        key: torch.Tensor,
        value: torch.Tensor,
        key_cache: torch.Tensor,
        value_cache: torch.Tensor,
        block_table: torch.Tensor,
        slot_mapping: torch.Tensor,
        context_lens: torch.Tensor,
        cu_seqlens_q: torch.Tensor,
        num_prefill_seqs: int,
        num_prefill_tokens: int,
        max_q_len: int,
    ) -> torch.Tensor:
        """One mixed chunked-prefill + decode step.

        Rows [0, num_prefill_tokens) of query belong to the first
        num_prefill_seqs sequences (chunks, packed by cu_seqlens_q); the
        remaining rows are one decode token per sequence. All K/V are stored
        first; then the prefill kernel runs on the caller's stream and the
        decode kernel on a side stream next to it (run_overlapped), joined
        before returning.
        """
        if slot_mapping is not None:
            ops.store_kvcache(key, value, key_cache, value_cache, slot_mapping)
        out = torch.empty_like(query)
        P, TP = num_prefill_seqs, num_prefill_tokens

        def prefill():
            ops.paged_prefill(
                query[:TP], key_cache, value_cache, cu_seqlens_q[: P + 1], max_q_len, self.scale,
                block_tables=block_table[:P], context_lens=context_lens[:P], out=out[:TP],
            )

        def decode():
            ops.paged_decode(
                query[TP:], key_cache, value_cache, block_table[P:], context_lens[P:], self.scale,
                out=out[TP:],
            )

        has_p, has_d = P > 0, query.shape[0] > TP
        if has_p and has_d and MIXED_OVERLAP:
            run_overlapped(prefill, decode)
        else:
            if has_p:
                prefill()
            if has_d:
                decode()
        return out
