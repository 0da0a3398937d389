"""An engine-shaped loop on the GPU through the drop-in API only: sequences
grow token by token across block boundaries, blocks are allocated as a
BlockManager would (a new physical block whenever a sequence fills its last
one), and every step runs Attention.forward (store + decode, the
LlamaAttention / Qwen3Attention call, litevllm/models/qwen3.py:87-92) and
Sampler.sample (litevllm/layers/sampler.py:151-187). Each step is checked
against the oracle: the stored slots bit-exact, attention within the stated
tolerance, greedy ids bit-exact. The next token is the GPU path's own
sample (teacher forcing keeps both sides on the same history)."""

import numpy as np
import pytest
import torch

from litevllm_b200.attention import Attention
from litevllm_b200.sampler import Sampler
from oracle import paged_attention as pa
from oracle import sampler as osamp
from tests.tolerance import assert_attn_close

pytestmark = pytest.mark.gpu


class SP:
    def __init__(self, temperature=0.0):
        self.temperature, self.top_p, self.top_k = temperature, 1.0, -1
        self.repetition_penalty, self.seed = 1.0, None


def test_decode_loop_across_block_boundaries(cuda):
    g = torch.Generator().manual_seed(99)
    H, H_kv, D, bs, V = 32, 8, 128, 16, 97
    prompts = [5, 16, 17, 31, 40, 1]
    steps = 20
    B = len(prompts)
    nblocks = 64
    # token -> q / k / v rows, and the output projection to logits
    emb = {n: (torch.randn((V, H if n == "q" else H_kv, D), generator=g) * 0.5).bfloat16()
           for n in "qkv"}
    w_out = torch.randn((H * D, V), generator=g) * 0.05
    free = torch.randperm(nblocks, generator=g).tolist()
    tables = [[] for _ in range(B)]
    kc = torch.zeros((nblocks, bs, H_kv, D), dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros_like(kc)
    attn = Attention(H, D, H_kv)
    tokens = [torch.randint(0, V, (n,), generator=g).tolist() for n in prompts]

    def slot(b, pos):
        while len(tables[b]) <= pos // bs:  # BlockManager.append_slot: new block when full
            tables[b].append(free.pop())
        return tables[b][pos // bs] * bs + pos % bs

    # prompts: store their K/V (the prefill step's store)
    for b in range(B):
        sl = torch.tensor([slot(b, p) for p in range(prompts[b])], device=cuda)
        ids = torch.tensor(tokens[b])
        attn.forward(emb["q"][ids].to(cuda), emb["k"][ids].to(cuda), emb["v"][ids].to(cuda),
                     kc, vc, None, sl, None, is_prefill=True)
    for step in range(steps):
        last = torch.tensor([t[-1] for t in tokens])
        pos = [len(t) - 1 for t in tokens]
        sl = torch.tensor([slot(b, pos[b]) for b in range(B)], device=cuda)
        ctx = torch.tensor([p + 1 for p in pos], dtype=torch.int32, device=cuda)
        mb = max(len(t) for t in tables)
        bt = torch.zeros((B, mb), dtype=torch.int32)
        for b in range(B):
            bt[b, :len(tables[b])] = torch.tensor(tables[b], dtype=torch.int32)
        bt = bt.to(cuda)
        q, k, v = (emb[n][last].to(cuda) for n in "qkv")
        out = attn.forward(q, k, v, kc, vc, bt, sl, ctx, is_prefill=False)
        # the new token's K/V sit in their slots, bit-exact
        assert torch.equal(kc.view(-1, H_kv, D)[sl], k) and torch.equal(vc.view(-1, H_kv, D)[sl], v)
        ref = pa.decode(q.float(), kc.float(), vc.float(), bt, ctx, attn.scale)
        assert_attn_close(out, ref)
        logits = (out.float().reshape(B, H * D).cpu() @ w_out).to(cuda)
        ids = Sampler.sample(logits, SP(0.0))
        assert np.array_equal(ids.cpu().numpy(), osamp.greedy(logits.cpu().numpy())), step
        for b in range(B):
            tokens[b].append(int(ids[b]))
    assert all(len(t) == n + steps for t, n in zip(tokens, prompts))
    assert max(len(t) for t in tables) >= 4  # crossed several block boundaries
