"""Seeded synthetic inputs for the hot-path configurations.

No public dataset or model checkpoint is involved: the configurations name
only shapes and value distributions, so every tensor is drawn from seeded
generators. Per-sequence quantities (context length) are keyed by
(config id, seed, global sequence index), so any number of GPUs that shard
the sequences by index reproduces the same union of inputs.

Configurations (H = query heads, H_kv = KV heads, D = head_dim, bs = 16):
  1  CPU reference decode, fp32, H=16 H_kv=8, B=8, ctx ~ U[1,512], 512-block pool,
     logits [8,151936] ~ N(0, 2^2); rows 0-3 greedy, rows 4-7 T=0.7.
  2  bf16 decode, H=32 H_kv=8, B=256, ctx = clip(round(lognormal(ln 1024, 0.5)), 16, 4096)
     (sigma is not given by the configuration; 0.5 is this build's choice),
     greedy sampler over [256, 128256] ~ N(0,1).
  3  bf16 mixed step: 4 prefill chunks of 512 on prior ~ U[0,3584] + 252 decode
     sequences with ctx ~ U[64,2048]; pool of 65536 blocks.
  4  bf16 prefix-shared decode: 128 sequences share 128 blocks (2048 tokens) then
     16 private blocks (256 tokens); T=0.7 over V=151936.
  5  bf16 long-context decode: B=64, ctx ~ U[32768,131072], T=1.0, V=151936.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import numpy as np
import torch

SHAPES = {
    1: dict(H=16, H_kv=8, D=128, bs=16, B=8, V=151936),
    2: dict(H=32, H_kv=8, D=128, bs=16, B=256, V=128256),
    3: dict(H=32, H_kv=8, D=128, bs=16, B=256, V=151936),
    4: dict(H=32, H_kv=8, D=128, bs=16, B=128, V=151936),
    5: dict(H=32, H_kv=8, D=128, bs=16, B=64, V=151936),
}


def _rng(cfg: int, seed: int, idx: int) -> np.random.Generator:
    return np.random.default_rng(np.random.SeedSequence([cfg, seed, idx]))


def context_len(cfg: int, seed: int, idx: int) -> int:
    """Context length (including this step's token) of global sequence idx."""
    r = _rng(cfg, seed, idx)
    if cfg == 1:
        return int(r.integers(1, 513))
    if cfg == 2:
        return int(np.clip(np.round(np.exp(r.normal(math.log(1024.0), 0.5))), 16, 4096))
    if cfg == 3:
        return int(r.integers(64, 2049))
    if cfg == 4:
        return 2048 + 256
    if cfg == 5:
        return int(r.integers(32768, 131073))
    raise ValueError(cfg)


def prefill_prior(seed: int, idx: int) -> int:
    """Config 3: prior paged context of prefill sequence idx."""
    return int(_rng(3, seed, 10_000 + idx).integers(0, 3585))


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _randn(shape, dtype, device, seed: int, std: float = 1.0) -> torch.Tensor:
    dev = torch.device(device)
    t = torch.empty(shape, dtype=torch.float32 if dtype == torch.float32 else dtype, device=dev)
    if dev.type == "cuda":
        # generate in chunks to bound the fp32 temporary
        flat = t.view(-1)
        g = _gen(seed, dev)
        step = 1 << 27
        for s in range(0, flat.numel(), step):
            e = min(flat.numel(), s + step)
            flat[s:e] = torch.randn(e - s, generator=g, device=dev, dtype=torch.float32).mul_(std).to(dtype)
        return t
    g = _gen(seed, "cpu")
    return (torch.randn(shape, generator=g, dtype=torch.float32) * std).to(dtype)


@dataclass
class DecodeBatch:
    """One decode step's inputs for B sequences on one device."""

    query: torch.Tensor          # [B, H, D]
    key: torch.Tensor            # [B, H_kv, D]  this step's new K
    value: torch.Tensor          # [B, H_kv, D]
    key_cache: torch.Tensor      # [num_blocks, bs, H_kv, D]
    value_cache: torch.Tensor
    block_tables: torch.Tensor   # int32 [B, max_blocks], zero padded
    context_lens: torch.Tensor   # int32 [B]
    slot_mapping: torch.Tensor   # int64 [B]
    ctx: list = field(default_factory=list)
    scale: float = 1.0 / math.sqrt(128)

    @property
    def B(self) -> int:
        return self.query.shape[0]


def make_decode_batch(
    cfg: int,
    B: int,
    seed: int = 0,
    first_seq: int = 0,
    dtype: torch.dtype = torch.bfloat16,
    device="cpu",
    ctx: Optional[list] = None,
    H: Optional[int] = None,
    H_kv: Optional[int] = None,
    D: Optional[int] = None,
    bs: Optional[int] = None,
    pool_blocks: Optional[int] = None,
    max_blocks: Optional[int] = None,
) -> DecodeBatch:
    """Decode inputs: sequences first_seq .. first_seq+B-1 of config cfg.

    Block tables are non-overlapping indices from one permutation of the pool
    (config 1 draws them from a fixed 512-block pool); unused table columns
    are 0, as ModelRunner.prepare_inputs pads them (model_runner.py:243-247).
    """
    sh = SHAPES.get(cfg, SHAPES[2])
    H = H or sh["H"]
    H_kv = H_kv or sh["H_kv"]
    D = D or sh["D"]
    bs = bs or sh["bs"]
    if ctx is None:
        ctx = [context_len(cfg, seed, first_seq + i) for i in range(B)]
    nblk = [max(1, -(-c // bs)) for c in ctx]
    need = sum(nblk)
    if pool_blocks is None:
        pool_blocks = max(need, 512 if cfg == 1 else need)
    if pool_blocks < need:
        raise ValueError("pool too small")
    mb = max(nblk) if max_blocks is None else max_blocks
    g = _gen(seed * 1000003 + first_seq, "cpu")
    perm = torch.randperm(pool_blocks, generator=g)
    bt = torch.zeros((B, mb), dtype=torch.int32)
    off = 0
    for i, n in enumerate(nblk):
        bt[i, :n] = perm[off : off + n].to(torch.int32)
        off += n
    slots = [int(bt[i, (c - 1) // bs]) * bs + (c - 1) % bs if c > 0 else -1 for i, c in enumerate(ctx)]
    base = (seed * 7919 + first_seq) * 16
    kc = _randn((pool_blocks, bs, H_kv, D), dtype, device, base + 1)
    vc = _randn((pool_blocks, bs, H_kv, D), dtype, device, base + 2)
    q = _randn((B, H, D), dtype, device, base + 3)
    k = _randn((B, H_kv, D), dtype, device, base + 4)
    v = _randn((B, H_kv, D), dtype, device, base + 5)
    return DecodeBatch(
        query=q,
        key=k,
        value=v,
        key_cache=kc,
        value_cache=vc,
        block_tables=bt.to(device),
        context_lens=torch.tensor(ctx, dtype=torch.int32).to(device),
        slot_mapping=torch.tensor(slots, dtype=torch.int64).to(device),
        ctx=list(ctx),
        scale=1.0 / math.sqrt(D),
    )


def make_logits(cfg: int, B: int, V: int, seed: int = 0, first_seq: int = 0,
                dtype=torch.bfloat16, device="cpu") -> torch.Tensor:
    """Logits [B, V]: N(0, 2^2) for config 1 (std 2), N(0, 1) otherwise."""
    std = 2.0 if cfg == 1 else 1.0
    return _randn((B, V), dtype, device, (seed * 7919 + first_seq) * 16 + 9, std=std)


def gumbel_noise(B: int, V: int, seed: int = 0, device="cpu") -> torch.Tensor:
    """Seeded fp32 Gumbel noise -log(-log(u)), u ~ U(0,1), for noise-given sampling."""
    g = _gen(seed * 31 + 17, "cpu")
    u = torch.rand((B, V), generator=g, dtype=torch.float64).clamp_(1e-12, 1 - 1e-12)
    return (-torch.log(-torch.log(u))).to(torch.float32).to(device)


def temperatures_for(cfg: int, B: int, device="cpu") -> torch.Tensor:
    """Per-row temperatures: config 1 rows 0-3 greedy / 4-7 at 0.7; config 2
    greedy; config 4 at 0.7; config 5 at 1.0."""
    if cfg == 1:
        t = [0.0 if i % 8 < 4 else 0.7 for i in range(B)]
    elif cfg == 2 or cfg == 3:
        t = [0.0] * B
    elif cfg == 4:
        t = [0.7] * B
    else:
        t = [1.0] * B
    return torch.tensor(t, dtype=torch.float32, device=device)


@dataclass
class PrefillBatch:
    query: torch.Tensor       # [T, H, D]
    key: torch.Tensor         # [T, H_kv, D]
    value: torch.Tensor
    key_cache: torch.Tensor
    value_cache: torch.Tensor
    block_tables: torch.Tensor
    context_lens: torch.Tensor  # prior + chunk
    cu_seqlens_q: torch.Tensor
    slot_mapping: torch.Tensor
    prior: list
    q_lens: list
    scale: float


def make_prefill_batch(
    q_lens: list,
    prior: list,
    seed: int = 0,
    H: int = 32,
    H_kv: int = 8,
    D: int = 128,
    bs: int = 16,
    dtype=torch.bfloat16,
    device="cpu",
    pool_slack: int = 0,
) -> PrefillBatch:
    """Chunks of q_lens[i] new tokens on top of prior[i] cached tokens.

    The prior keys are already in the pool; the chunk's own K/V are returned
    separately (key / value) together with the slot_mapping that stores them.
    """
    S = len(q_lens)
    ctx = [p + q for p, q in zip(prior, q_lens)]
    nblk = [max(1, -(-c // bs)) for c in ctx]
    pool = sum(nblk) + pool_slack
    g = _gen(seed * 1000003 + 7, "cpu")
    perm = torch.randperm(pool, generator=g)
    mb = max(nblk)
    bt = torch.zeros((S, mb), dtype=torch.int32)
    off = 0
    for i, n in enumerate(nblk):
        bt[i, :n] = perm[off : off + n].to(torch.int32)
        off += n
    slots = []
    for i in range(S):
        for pos in range(prior[i], ctx[i]):
            slots.append(int(bt[i, pos // bs]) * bs + pos % bs)
    T = sum(q_lens)
    base = seed * 104729 * 16
    cu = [0]
    for q in q_lens:
        cu.append(cu[-1] + q)
    return PrefillBatch(
        query=_randn((T, H, D), dtype, device, base + 3),
        key=_randn((T, H_kv, D), dtype, device, base + 4),
        value=_randn((T, H_kv, D), dtype, device, base + 5),
        key_cache=_randn((pool, bs, H_kv, D), dtype, device, base + 1),
        value_cache=_randn((pool, bs, H_kv, D), dtype, device, base + 2),
        block_tables=bt.to(device),
        context_lens=torch.tensor(ctx, dtype=torch.int32).to(device),
        cu_seqlens_q=torch.tensor(cu, dtype=torch.int32).to(device),
        slot_mapping=torch.tensor(slots, dtype=torch.int64).to(device),
        prior=list(prior),
        q_lens=list(q_lens),
        scale=1.0 / math.sqrt(D),
    )


def make_prefix_batch(B: int = 128, shared_blocks: int = 128, private_blocks: int = 16,
                      seed: int = 0, dtype=torch.bfloat16, device="cpu", H: int = 32,
                      H_kv: int = 8, D: int = 128, bs: int = 16, fork=None) -> DecodeBatch:
    """Config 4: every sequence's table starts with the same `shared_blocks`
    physical blocks (a common prefix), except that the last shared block is
    copy-on-write forked into a private copy per sequence, followed by
    `private_blocks` private blocks. `fork(caches, mapping)` performs the copy
    (the library's block copy); without it the copy is done with torch."""
    pool = (shared_blocks - 1) + B * (1 + private_blocks)
    ctx = (shared_blocks + private_blocks) * bs
    g = _gen(seed * 1000003 + 44, "cpu")
    perm = torch.randperm(pool, generator=g)
    shared = perm[: shared_blocks - 1]
    rest = perm[shared_blocks - 1:].view(B, 1 + private_blocks)
    bt = torch.empty((B, shared_blocks + private_blocks), dtype=torch.int32)
    bt[:, : shared_blocks - 1] = shared.to(torch.int32)
    bt[:, shared_blocks - 1:] = rest.to(torch.int32)
    base = (seed * 7919 + 4) * 16
    kc = _randn((pool, bs, H_kv, D), dtype, device, base + 1)
    vc = _randn((pool, bs, H_kv, D), dtype, device, base + 2)
    # the original last shared block lives at rest[0, 0]; fork it into rest[b, 0]
    if fork is not None:
        fork([(kc, vc)], [(int(rest[0, 0]), int(rest[b, 0])) for b in range(1, B)])
    else:
        for b in range(1, B):
            kc[int(rest[b, 0])] = kc[int(rest[0, 0])]
            vc[int(rest[b, 0])] = vc[int(rest[0, 0])]
    slots = [int(bt[i, (ctx - 1) // bs]) * bs + (ctx - 1) % bs for i in range(B)]
    return DecodeBatch(
        query=_randn((B, H, D), dtype, device, base + 3),
        key=_randn((B, H_kv, D), dtype, device, base + 4),
        value=_randn((B, H_kv, D), dtype, device, base + 5),
        key_cache=kc, value_cache=vc, block_tables=bt.to(device),
        context_lens=torch.full((B,), ctx, dtype=torch.int32).to(device),
        slot_mapping=torch.tensor(slots, dtype=torch.int64).to(device),
        ctx=[ctx] * B, scale=1.0 / math.sqrt(D))
