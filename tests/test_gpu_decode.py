"""Paged decode attention on the GPU vs the reference (golden) and the fp32 oracle."""

import math

import pytest
import torch

from litevllm_b200 import ops, workloads
from litevllm_b200.attention import Attention
from oracle import paged_attention as pa
from tests import golden_io
from tests.tolerance import assert_attn_close

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["store_decode.npz", "decode_g4.npz"])
def test_decode_matches_reference_golden(cuda, name):
    """Store + decode through the drop-in Attention.forward, as the reference's
    Attention.forward(..., is_prefill=False) ran them."""
    d = golden_io.decode_case(name)
    attn = Attention(int(d["H"]), int(d["D"]), int(d["H_kv"]))
    kc, vc = d["key_cache"].to(cuda), d["value_cache"].to(cuda)
    out = attn.forward(d["query"].to(cuda), d["key"].to(cuda), d["value"].to(cuda), kc, vc,
                       d["block_tables"].to(cuda), d["slot_mapping"].to(cuda),
                       d["context_lens"].to(cuda), is_prefill=False)
    assert out.dtype == torch.bfloat16 and out.shape == d["out"].shape
    assert_attn_close(out, d["out"])


def _check(b, rows=None, num_splits=0, dtype=torch.bfloat16):
    out = ops.paged_decode(b.query, b.key_cache, b.value_cache, b.block_tables, b.context_lens,
                           b.scale, num_splits=num_splits)
    ref = pa.decode(b.query.float(), b.key_cache.float(), b.value_cache.float(), b.block_tables,
                    b.context_lens, b.scale, rows=rows)
    got = out if rows is None else out[list(rows)]
    assert_attn_close(got, ref)
    return out


@pytest.mark.parametrize("ctx", [[1], [15], [16], [17], [1, 2, 3, 31, 32, 33, 255, 256, 257]])
def test_decode_edge_lengths(cuda, ctx):
    b = workloads.make_decode_batch(1, len(ctx), seed=5, ctx=ctx, H=16, H_kv=8, device=cuda)
    _check(b)


@pytest.mark.parametrize("H,H_kv", [(8, 8), (16, 8), (32, 8), (64, 8), (32, 4), (8, 2), (4, 1), (16, 16)])
def test_decode_gqa_ratios_and_head_groups(cuda, H, H_kv):
    b = workloads.make_decode_batch(2, 6, seed=H * 7 + H_kv, H=H, H_kv=H_kv, device=cuda,
                                    ctx=[5, 100, 333, 1024, 16, 700])
    _check(b)


@pytest.mark.parametrize("num_splits", [-1, 1, 2, 3, 7, 64])
def test_decode_split_kv_consistent(cuda, num_splits):
    b = workloads.make_decode_batch(2, 5, seed=11, device=cuda, ctx=[4096, 1, 2000, 17, 1023])
    _check(b, num_splits=num_splits)


def test_decode_repeated_calls_reuse_workspace(cuda):
    """Counters reset after each call: many back-to-back split calls agree."""
    b = workloads.make_decode_batch(2, 16, seed=12, device=cuda)
    first = ops.paged_decode(b.query, b.key_cache, b.value_cache, b.block_tables, b.context_lens,
                             b.scale, num_splits=8)
    for _ in range(5):
        again = ops.paged_decode(b.query, b.key_cache, b.value_cache, b.block_tables,
                                 b.context_lens, b.scale, num_splits=8)
        assert torch.equal(first, again)
    assert ops.decode_status() == 0


def test_decode_fp16(cuda):
    b = workloads.make_decode_batch(2, 8, seed=13, dtype=torch.float16, device=cuda)
    _check(b)


def test_decode_block_size_32(cuda):
    b = workloads.make_decode_batch(2, 6, seed=14, bs=32, device=cuda, ctx=[1, 31, 32, 33, 500, 64])
    _check(b)


def test_decode_zero_context_is_nan_like_reference(cuda):
    """The reference's softmax over an all -inf row yields NaN (attention.py:132-135)."""
    b = workloads.make_decode_batch(2, 3, seed=15, device=cuda, ctx=[5, 1, 9])
    b.context_lens[1] = 0
    out = ops.paged_decode(b.query, b.key_cache, b.value_cache, b.block_tables, b.context_lens,
                           b.scale)
    assert torch.isnan(out[1]).all() and not torch.isnan(out[[0, 2]]).any()
    lit = pa.decode_batched_reference(b.query.float().cpu(), b.key_cache.float().cpu(),
                                      b.value_cache.float().cpu(), b.block_tables.cpu(),
                                      b.context_lens.cpu(), b.scale)
    assert torch.isnan(lit[1]).all()


def test_decode_custom_scale_and_strided_query(cuda):
    b = workloads.make_decode_batch(2, 4, seed=16, device=cuda)
    big = torch.randn((4, 3, 32, 128), device=cuda).bfloat16()
    big[:, 1] = b.query
    q = big[:, 1]  # token stride 3*32*128
    out = ops.paged_decode(q, b.key_cache, b.value_cache, b.block_tables, b.context_lens, 0.05)
    ref = pa.decode(b.query.float(), b.key_cache.float(), b.value_cache.float(), b.block_tables,
                    b.context_lens, 0.05)
    assert_attn_close(out, ref)


def test_decode_config2_full_batch_sampled_rows(cuda):
    """Config 2 at full size (B=256); the oracle checks 24 rows incl. the longest."""
    b = workloads.make_decode_batch(2, 256, seed=0, device=cuda)
    longest = max(range(256), key=lambda i: b.ctx[i])
    rows = sorted(set(list(range(0, 256, 12)) + [longest]))
    _check(b, rows=rows)


def test_decode_config5_long_context_subset(cuda):
    """Config 5 shapes (32K-128K tokens, split-KV mandatory) on 2 sequences."""
    ctx = [workloads.context_len(5, 0, 0), 131072]
    b = workloads.make_decode_batch(5, 2, seed=0, device=cuda, ctx=ctx)
    _check(b)


def test_decode_config5_full_batch_eight_rows(cuda):
    """Config 5 at full size: 64 sequences of 32K-128K tokens (22 GB of bf16
    KV) in one split-KV launch; the oracle checks 8 rows, the longest among
    them, each on its own gathered blocks."""
    b = workloads.make_decode_batch(5, 64, seed=0, device=cuda)
    out = ops.paged_decode(b.query, b.key_cache, b.value_cache, b.block_tables, b.context_lens,
                           b.scale)
    longest = max(range(64), key=lambda i: b.ctx[i])
    rows = sorted(set(list(range(3, 64, 9)) + [longest]))
    assert len(rows) >= 8
    for i in rows:
        n = -(-b.ctx[i] // 16)
        blk = b.block_tables[i, :n].long()
        kc, vc = b.key_cache[blk].float(), b.value_cache[blk].float()
        bt = torch.arange(n, dtype=torch.int32, device=cuda)[None]
        ref = pa.decode(b.query[i:i + 1].float(), kc, vc, bt, b.context_lens[i:i + 1], b.scale)
        assert_attn_close(out[i:i + 1], ref)
        del kc, vc


def test_decode_two_streams_concurrently(cuda):
    """Split decodes on two streams at once: each stream has its own default
    workspace (counters, partials, ordering), so neither corrupts the other."""
    cases = [workloads.make_decode_batch(2, 64, seed=s, device=cuda) for s in (41, 42)]
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    for _ in range(3):
        outs = []
        for b, st in zip(cases, streams):
            with torch.cuda.stream(st):
                outs.append(ops.paged_decode(b.query, b.key_cache, b.value_cache, b.block_tables,
                                             b.context_lens, b.scale, num_splits=4))
    torch.cuda.synchronize()
    for b, out in zip(cases, outs):
        ref = pa.decode(b.query.float(), b.key_cache.float(), b.value_cache.float(),
                        b.block_tables, b.context_lens, b.scale)
        assert_attn_close(out, ref)


def test_decode_out_of_range_block_flags_status(cuda):
    b = workloads.make_decode_batch(2, 2, seed=17, device=cuda, ctx=[40, 40])
    nb = b.key_cache.shape[0]
    b.block_tables[1, 1] = nb + 5
    ws = torch.zeros(ops.decode_workspace_bytes(2, 32, 8, 128, -1), dtype=torch.uint8, device=cuda)
    ops.paged_decode(b.query, b.key_cache, b.value_cache, b.block_tables, b.context_lens, b.scale,
                     workspace=ws, num_splits=-1)
    assert ops.decode_status(ws) & 2


def test_decode_workspace_reused_across_batch_shapes(cuda):
    for B, splits in [(3, 5), (40, 7), (5, 64), (40, 7)]:
        b = workloads.make_decode_batch(2, B, seed=B, device=cuda)
        _check(b, num_splits=splits)


def test_persistent_many_tiny_sequences(cuda):
    """Hundreds of 1-40 token sequences: many units per CTA, ranges cutting units."""
    ctx = [1 + (i * 7) % 40 for i in range(1000)]
    b = workloads.make_decode_batch(2, len(ctx), seed=21, device=cuda, ctx=ctx)
    _check(b, num_splits=-1)
    _check(b)


def test_persistent_single_long_sequence_spans_all_ctas(cuda):
    """One 100K-token sequence is cut across every SM; the last CTA merges all."""
    b = workloads.make_decode_batch(5, 1, seed=22, device=cuda, ctx=[100_003])
    _check(b, num_splits=-1)
    _check(b)


def test_persistent_matches_split_kernel(cuda):
    b = workloads.make_decode_batch(2, 64, seed=23, device=cuda)
    a = ops.paged_decode(b.query, b.key_cache, b.value_cache, b.block_tables, b.context_lens,
                         b.scale, num_splits=-1)
    s = ops.paged_decode(b.query, b.key_cache, b.value_cache, b.block_tables, b.context_lens,
                         b.scale, num_splits=3)
    assert_attn_close(a, s.float(), max_abs=8e-3, mean_rel=2e-3)


def test_decode_shared_prefix_with_cow_fork(cuda):
    """Config 4: 128 sequences share a 2048-token prefix (127 shared blocks plus a
    copy-on-write fork of the last one, made with the library's block copy)."""
    b = workloads.make_prefix_batch(B=128, seed=1, device=cuda, fork=ops.copy_blocks)
    ref_b = workloads.make_prefix_batch(B=128, seed=1, device=cuda)  # torch fork
    assert torch.equal(b.key_cache, ref_b.key_cache) and torch.equal(b.value_cache, ref_b.value_cache)
    _check(b, rows=[0, 1, 64, 127])


@pytest.mark.parametrize("variant", ["LITEKERN_DECODE_ORDER=0", "LITEKERN_DECODE_HEADS_PER_CTA=4",
                                     "LITEKERN_DECODE_HEADS_PER_CTA=2",
                                     "LITEKERN_DECODE_HEADS_PER_CTA=1",
                                     "LITEKERN_DECODE_PREFETCH=8", "LITEKERN_DECODE_STREAM=1",
                                     "LITEKERN_PREFIX_RANGES=1", "LITEKERN_PREFIX_RANGES=16",
                                     "LITEKERN_PREFIX_SPP=8", "LITEKERN_PDL=0"])
def test_decode_kernel_options(variant):
    """The decode options (read once per process from the environment)
    against the oracle, in a child process."""
    import os
    import subprocess
    import sys
    key, val = variant.split("=")
    env = dict(os.environ, **{key: val})
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-m", "tests.decode_variant_check"], cwd=root, env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "ok" in r.stdout


def _shared_prefix_batch(cuda, B, prefix_blocks, suffix_lens, H=32, H_kv=8, dtype=torch.bfloat16,
                         seed=0, bs=16):
    g = torch.Generator().manual_seed(seed)
    priv = [-(-n // bs) for n in suffix_lens]
    pool = prefix_blocks + sum(priv) + 1
    perm = torch.randperm(pool, generator=g).tolist()
    shared, rest = perm[:prefix_blocks], perm[prefix_blocks:]
    mb = prefix_blocks + max(priv + [0])
    bt = torch.zeros((B, max(mb, 1)), dtype=torch.int32)
    off = 0
    for b in range(B):
        bt[b, :prefix_blocks] = torch.tensor(shared, dtype=torch.int32)
        bt[b, prefix_blocks:prefix_blocks + priv[b]] = torch.tensor(rest[off:off + priv[b]],
                                                                   dtype=torch.int32)
        off += priv[b]
    kc = torch.randn((pool, bs, H_kv, 128), generator=g).to(dtype).to(cuda)
    vc = torch.randn((pool, bs, H_kv, 128), generator=g).to(dtype).to(cuda)
    q = torch.randn((B, H, 128), generator=g).to(dtype).to(cuda)
    ctx = torch.tensor([prefix_blocks * bs + n for n in suffix_lens], dtype=torch.int32)
    return q, kc, vc, bt.to(cuda), ctx.to(cuda)


@pytest.mark.parametrize("B,prefix_blocks,H", [(128, 127, 32), (7, 8, 32), (1, 1, 32),
                                               (33, 25, 8), (16, 50, 16), (20, 9, 64)])
def test_shared_prefix_decode_matches_oracle(cuda, B, prefix_blocks, H):
    g = torch.Generator().manual_seed(B * 31 + prefix_blocks)
    suffix = torch.randint(0, 300, (B,), generator=g).tolist()
    suffix[0] = 0  # a row whose whole context is the prefix
    q, kc, vc, bt, ctx = _shared_prefix_batch(cuda, B, prefix_blocks, suffix, H=H, seed=B)
    scale = 128 ** -0.5
    out = ops.paged_decode_shared_prefix(q, kc, vc, bt, ctx, scale, prefix_blocks * 16)
    rows = list(range(min(B, 12)))
    ref = pa.decode(q.float(), kc.float(), vc.float(), bt, ctx, scale, rows=rows)
    assert_attn_close(out[rows], ref)
    # and the regular kernel on the same inputs agrees on every row
    out2 = ops.paged_decode(q, kc, vc, bt, ctx, scale)
    assert_attn_close(out, out2.float(), max_abs=1e-2, mean_rel=5e-3)


def test_shared_prefix_decode_config4_and_fp16(cuda):
    b = workloads.make_prefix_batch(128, seed=3, device=cuda)
    scale = b.scale
    out = ops.paged_decode_shared_prefix(b.query, b.key_cache, b.value_cache, b.block_tables,
                                         b.context_lens, scale, 127 * 16)
    ref = pa.decode(b.query.float(), b.key_cache.float(), b.value_cache.float(), b.block_tables,
                    b.context_lens, scale, rows=[0, 1, 64, 127])
    assert_attn_close(out[[0, 1, 64, 127]], ref)
    q, kc, vc, bt, ctx = _shared_prefix_batch(cuda, 9, 20, [5, 0, 100, 17, 64, 1, 2, 3, 250],
                                              dtype=torch.float16, seed=9)
    out = ops.paged_decode_shared_prefix(q, kc, vc, bt, ctx, 128 ** -0.5, 320)
    ref = pa.decode(q.float(), kc.float(), vc.float(), bt, ctx, 128 ** -0.5)
    assert_attn_close(out, ref)


def test_attention_forward_uses_the_shared_prefix_hint(cuda):
    """The engine hook's hint routes Attention.forward's decode to the
    shared-prefix kernel for that step's table only; results agree."""
    from litevllm_b200 import attention as att
    b = workloads.make_prefix_batch(32, seed=4, device=cuda)
    layer = att.Attention(32, 128, 8)
    plain = layer.forward(b.query, b.key, b.value, b.key_cache, b.value_cache, b.block_tables,
                          None, b.context_lens, is_prefill=False)
    att.set_shared_prefix_hint(b.block_tables, 127 * 16)
    try:
        hinted = layer.forward(b.query, b.key, b.value, b.key_cache, b.value_cache,
                               b.block_tables, None, b.context_lens, is_prefill=False)
        other = b.block_tables.clone()  # another tensor: the hint does not apply
        again = layer.forward(b.query, b.key, b.value, b.key_cache, b.value_cache, other, None,
                              b.context_lens, is_prefill=False)
    finally:
        att.set_shared_prefix_hint(None, 0)
    assert_attn_close(hinted, plain.float(), max_abs=1e-2, mean_rel=5e-3)
    assert torch.equal(again, plain)


def test_shared_prefix_decode_back_to_back_is_exact(cuda):
    """The suffix decode starts beside the prefix kernel and waits for it only
    before merging the prefix partials. Back-to-back calls alternating two
    query tensors (eagerly and from a CUDA graph) must each give the bits of
    a call made alone: a merge that read the other call's partials, or this
    call's before they were written, would not."""
    b = workloads.make_prefix_batch(128, seed=5, device=cuda)
    q2 = torch.flip(b.query, dims=[0]).contiguous()
    args = (b.key_cache, b.value_cache, b.block_tables, b.context_lens, b.scale, 127 * 16)
    want = []
    for q in (b.query, q2):
        want.append(ops.paged_decode_shared_prefix(q, *args).clone())
        torch.cuda.synchronize()
    outs = [torch.empty_like(b.query) for _ in range(16)]
    for i, o in enumerate(outs):
        ops.paged_decode_shared_prefix(b.query if i % 2 == 0 else q2, *args, out=o)
    torch.cuda.synchronize()
    for i, o in enumerate(outs):
        assert torch.equal(o, want[i % 2]), i
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for i, o in enumerate(outs):  # warm-up on the capture stream
            ops.paged_decode_shared_prefix(b.query if i % 2 == 0 else q2, *args, out=o)
        with torch.cuda.graph(g, stream=s):
            for i, o in enumerate(outs):
                ops.paged_decode_shared_prefix(b.query if i % 2 == 0 else q2, *args, out=o)
    torch.cuda.current_stream().wait_stream(s)
    for o in outs:
        o.zero_()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    for i, o in enumerate(outs):
        assert torch.equal(o, want[i % 2]), i


def test_shared_prefix_longer_than_a_row_is_flagged(cuda):
    q, kc, vc, bt, ctx = _shared_prefix_batch(cuda, 6, 10, [5, 40, 0, 7, 9, 30], seed=12)
    ctx[2] = 100  # shorter than the declared 160-token prefix
    ws = torch.zeros(ops.lib().lk_paged_decode_shared_prefix_workspace_bytes(
        6, 32, 8, 128, bt.shape[1], 16, 160), dtype=torch.uint8, device=cuda)
    ops.paged_decode_shared_prefix(q, kc, vc, bt, ctx, 128 ** -0.5, 160, workspace=ws)
    assert ops.decode_status(ws) & 8  # LK_STATUS_CTX_OOB


@pytest.mark.parametrize("H,H_kv", [(32, 4), (8, 2), (4, 1), (16, 16)])
def test_shared_prefix_decode_head_groupings(cuda, H, H_kv):
    suffix = [3, 0, 77, 250, 16, 1]
    q, kc, vc, bt, ctx = _shared_prefix_batch(cuda, 6, 12, suffix, H=H, H_kv=H_kv, seed=H + H_kv)
    out = ops.paged_decode_shared_prefix(q, kc, vc, bt, ctx, 128 ** -0.5, 12 * 16)
    ref = pa.decode(q.float(), kc.float(), vc.float(), bt, ctx, 128 ** -0.5)
    assert_attn_close(out, ref)
