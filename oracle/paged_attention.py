"""Attention oracles (torch fp32 on CPU). Test infrastructure only.

decode():  restates Attention._decode_fast, litevllm/layers/attention.py:91-139,
           one sequence at a time (the reference's padded gather costs
           B x max_ctx memory; rows do not interact, so per-row evaluation
           gives the same numbers).
prefill(): no reference exists for a chunk on top of prior paged context
           (the reference's _prefill, :141-151, ignores the cache). This
           composes _decode_fast's gather (:105-119) for the prior keys with
           _prefill's causal mask for the chunk: query i sees keys
           j <= prior + i. For prior == 0 it equals _prefill (SDPA causal,
           scale 1/sqrt(D), GQA by repeat_interleave, :147-149).
"""

from __future__ import annotations

import math

import torch


def _gather(cache: torch.Tensor, blocks: torch.Tensor, n: int) -> torch.Tensor:
    """Rows 0..n-1 of one sequence: cache[block_table[p // bs], p % bs] (attention.py:112-119)."""
    bs = cache.shape[1]
    pos = torch.arange(n)
    return cache[blocks.long()[pos // bs], pos % bs]  # [n, H_kv, D]


def decode_one(q: torch.Tensor, key_cache, value_cache, blocks, ctx: int, scale: float,
               round_probs_to=None) -> torch.Tensor:
    """q [H, D] of one sequence -> [H, D] fp32.

    Scores in fp32 (einsum, attention.py:129), * scale, softmax in fp32
    (:135). If round_probs_to is a dtype, the probabilities are rounded to it
    before the PV product, as the reference does with `.to(query.dtype)`.
    """
    H, D = q.shape
    H_kv = key_cache.shape[2]
    G = H // H_kv
    if ctx <= 0:
        return torch.full((H, D), float("nan"))
    k = _gather(key_cache, blocks, ctx).float().permute(1, 0, 2)  # [H_kv, n, D]
    v = _gather(value_cache, blocks, ctx).float().permute(1, 0, 2)
    qg = q.float().view(H_kv, G, D)                               # attention.py:124
    s = torch.einsum("hgd,hsd->hgs", qg, k) * scale               # :129
    p = torch.softmax(s, dim=-1, dtype=torch.float32)             # :135
    if round_probs_to is not None:
        p = p.to(round_probs_to).float()
    return torch.einsum("hgs,hsd->hgd", p, v).reshape(H, D)       # :138-139


def decode(query, key_cache, value_cache, block_tables, context_lens, scale,
           rows=None, round_probs_to=None) -> torch.Tensor:
    """query [B, H, D] -> fp32 [B, H, D] (or [len(rows), H, D] for a subset)."""
    query, key_cache, value_cache = query.cpu(), key_cache.cpu(), value_cache.cpu()
    block_tables, context_lens = block_tables.cpu(), context_lens.cpu()
    rows = range(query.shape[0]) if rows is None else rows
    out = [decode_one(query[b], key_cache, value_cache, block_tables[b], int(context_lens[b]),
                      scale, round_probs_to) for b in rows]
    return torch.stack(out)


def decode_batched_reference(query, key_cache, value_cache, block_table, context_lens, scale):
    """Literal restatement of _decode_fast (attention.py:91-139), padded gather
    and all, in the input dtype; for small cases and the CPU baseline."""
    B, H, D = query.shape
    bs = key_cache.shape[1]
    max_s = block_table.shape[1] * bs
    H_kv = key_cache.shape[2]
    G = H // H_kv
    positions = torch.arange(max_s).unsqueeze(0)
    b_idx = torch.gather(block_table.long(), 1, (positions // bs).expand(B, max_s))
    b_off = (positions % bs).expand(B, max_s)
    k = key_cache[b_idx, b_off].permute(0, 2, 1, 3).contiguous()
    v = value_cache[b_idx, b_off].permute(0, 2, 1, 3).contiguous()
    q = query.view(B, H_kv, G, D)
    attn = torch.einsum("bhgd,bhsd->bhgs", q, k) * scale
    mask = positions < context_lens.unsqueeze(1).to(positions.dtype)
    attn = attn.masked_fill(~mask.view(B, 1, 1, max_s), float("-inf"))
    attn = torch.softmax(attn, dim=-1, dtype=torch.float32).to(query.dtype)
    return torch.einsum("bhgs,bhsd->bhgd", attn, v).reshape(B, H, D)


def prefill_one(q, key_cache, value_cache, blocks, prior: int, scale: float) -> torch.Tensor:
    """q [S, H, D] chunk at positions prior..prior+S-1; keys from the paged cache
    (which already holds the chunk's own K/V). -> fp32 [S, H, D]."""
    S, H, D = q.shape
    H_kv = key_cache.shape[2]
    G = H // H_kv
    n = prior + S
    k = _gather(key_cache, blocks, n).float()  # [n, H_kv, D]
    v = _gather(value_cache, blocks, n).float()
    return _causal(q.float(), k, v, prior, scale, G)


def _causal(q, k, v, prior, scale, G):
    S, H, D = q.shape
    n = k.shape[0]
    k = k.repeat_interleave(G, dim=1).permute(1, 0, 2)  # [H, n, D]   (attention.py:147-149)
    v = v.repeat_interleave(G, dim=1).permute(1, 0, 2)
    s = torch.einsum("shd,hnd->hsn", q, k) * scale
    i = torch.arange(S).unsqueeze(1)
    j = torch.arange(n).unsqueeze(0)
    s = s.masked_fill((j > prior + i).unsqueeze(0), float("-inf"))
    p = torch.softmax(s, dim=-1, dtype=torch.float32)
    return torch.einsum("hsn,hnd->shd", p, v)


def prefill_contiguous(q, k, v, scale=None) -> torch.Tensor:
    """Reference _prefill (attention.py:141-151) in fp32: causal over the chunk."""
    S, H, D = q.shape
    G = H // k.shape[1]
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    return _causal(q.float(), k.float(), v.float(), 0, scale, G)


def prefill(query, key_cache, value_cache, block_tables, context_lens, cu_seqlens_q, scale,
            seqs=None) -> torch.Tensor:
    """Packed chunks -> fp32 [T, H, D] (rows of sequences not in `seqs` are 0)."""
    query, key_cache, value_cache = query.cpu(), key_cache.cpu(), value_cache.cpu()
    bt, cl, cu = block_tables.cpu(), context_lens.cpu(), cu_seqlens_q.cpu()
    out = torch.zeros(query.shape, dtype=torch.float32)
    seqs = range(cu.numel() - 1) if seqs is None else seqs
    for b in seqs:
        s0, s1 = int(cu[b]), int(cu[b + 1])
        prior = int(cl[b]) - (s1 - s0)
        out[s0:s1] = prefill_one(query[s0:s1], key_cache, value_cache, bt[b], prior, scale)
    return out
