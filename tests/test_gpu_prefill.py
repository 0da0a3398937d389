"""Chunked-prefill attention on the GPU vs the reference's _prefill (golden)
and the fp32 prior-context oracle."""

import pytest
import torch

from litevllm_b200 import ops, workloads
from litevllm_b200.attention import Attention
from oracle import paged_attention as pa
from tests import golden_io
from tests.tolerance import assert_attn_close

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("tag", ["g2", "g4"])
def test_prefill_matches_reference_golden(cuda, tag):
    """The reference path: Attention.forward(is_prefill=True) with no block
    table attends the new tokens only (attention.py:141-151)."""
    d = golden_io.load("prefill.npz")
    S, H, H_kv, D = (int(x) for x in d[f"{tag}_shape"])
    q, k, v = (golden_io.bf16(d[f"{tag}_{x}"]).to(cuda) for x in "qkv")
    attn = Attention(H, D, H_kv)
    out = attn.forward(q, k, v, None, None, None, None, None, is_prefill=True)
    assert_attn_close(out, torch.from_numpy(d[f"{tag}_out"]))


def _paged_case(cuda, q_lens, prior, H=32, H_kv=8, seed=0, dtype=torch.bfloat16, bs=16):
    b = workloads.make_prefill_batch(q_lens, prior, seed=seed, H=H, H_kv=H_kv, dtype=dtype,
                                     bs=bs, device=cuda)
    ops.store_kvcache(b.key, b.value, b.key_cache, b.value_cache, b.slot_mapping)
    out = ops.paged_prefill(b.query, b.key_cache, b.value_cache, b.cu_seqlens_q, max(q_lens),
                            b.scale, block_tables=b.block_tables, context_lens=b.context_lens)
    ref = pa.prefill(b.query.float(), b.key_cache.float(), b.value_cache.float(), b.block_tables,
                     b.context_lens, b.cu_seqlens_q, b.scale)
    assert_attn_close(out, ref)
    return b, out


@pytest.mark.parametrize("q_lens,prior", [
    ([1], [0]), ([16], [0]), ([17], [5]), ([64], [64]), ([200], [1000]),
    ([1, 33, 128, 7], [0, 15, 2000, 3]),
])
def test_prefill_paged_prior_context(cuda, q_lens, prior):
    _paged_case(cuda, q_lens, prior)


@pytest.mark.parametrize("H,H_kv", [(8, 8), (16, 8), (32, 8), (64, 8)])
def test_prefill_gqa_ratios(cuda, H, H_kv):
    _paged_case(cuda, [40, 130], [70, 0], H=H, H_kv=H_kv, seed=H)


def test_prefill_fp16(cuda):
    _paged_case(cuda, [90], [33], dtype=torch.float16, seed=3)


def test_prefill_prior_zero_equals_contiguous(cuda):
    """With no prior context the paged path equals the reference's _prefill path."""
    b, out = _paged_case(cuda, [77], [0], seed=4)
    cu = torch.tensor([0, 77], dtype=torch.int32, device=cuda)
    out2 = ops.paged_prefill(b.query, b.key, b.value, cu, 77, b.scale)
    assert_attn_close(out2, out.float(), max_abs=1e-2, mean_rel=5e-3)


def test_prefill_config3_chunks(cuda):
    """Config 3's four 512-token chunks on top of prior context ~U[0,3584]."""
    prior = [workloads.prefill_prior(0, i) for i in range(4)]
    _paged_case(cuda, [512] * 4, prior, seed=5)


def test_mixed_step_prefill_plus_decode(cuda):
    """One mixed step through Attention.forward_mixed: 2 chunks + 5 decode rows."""
    q_lens = [40, 70, 1, 1, 1, 1, 1]
    prior = [100, 0, 9, 300, 15, 16, 1000]
    b = workloads.make_prefill_batch(q_lens, prior, seed=6, device=cuda)
    attn = Attention(32, 128, 8)
    out = attn.forward_mixed(b.query, b.key, b.value, b.key_cache, b.value_cache,
                             b.block_tables, b.slot_mapping, b.context_lens, b.cu_seqlens_q,
                             num_prefill_seqs=2, num_prefill_tokens=110, max_q_len=70)
    ref = pa.prefill(b.query.float(), b.key_cache.float(), b.value_cache.float(), b.block_tables,
                     b.context_lens, b.cu_seqlens_q, b.scale)
    assert_attn_close(out, ref)


def test_mixed_step_overlapped_equals_sequential(cuda, monkeypatch):
    """forward_mixed's two-stream form (decode on a side stream next to the
    prefill) gives the same bits as running them one after the other, and is
    joined before returning (the result is read on the caller's stream)."""
    from litevllm_b200 import attention as attn_mod
    q_lens = [512, 300, 64] + [1] * 40
    prior = [1000, 2900, 0] + list(range(50, 50 + 40 * 37, 37))
    b = workloads.make_prefill_batch(q_lens, prior, seed=36, device=cuda)
    attn = Attention(32, 128, 8)
    args = (b.query, b.key, b.value, b.key_cache, b.value_cache, b.block_tables, b.slot_mapping,
            b.context_lens, b.cu_seqlens_q)
    kw = dict(num_prefill_seqs=3, num_prefill_tokens=876, max_q_len=512)
    monkeypatch.setattr(attn_mod, "MIXED_OVERLAP", True)
    over = attn.forward_mixed(*args, **kw)
    monkeypatch.setattr(attn_mod, "MIXED_OVERLAP", False)
    seq = attn.forward_mixed(*args, **kw)  # stores the same K/V again: idempotent
    assert torch.equal(over, seq)
    ref = pa.prefill(b.query.float(), b.key_cache.float(), b.value_cache.float(), b.block_tables,
                     b.context_lens, b.cu_seqlens_q, b.scale)
    assert_attn_close(over, ref)


def test_prefill_many_ragged_items(cuda):
    """Far more work items than SMs, ragged chunk lengths and priors: every
    item is taken once from the persistent kernel's counter, and the query
    hand-over between consecutive items of one CTA is exact."""
    g = torch.Generator().manual_seed(11)
    n = 40
    q_lens = torch.randint(1, 700, (n,), generator=g).tolist()
    prior = torch.randint(0, 1500, (n,), generator=g).tolist()
    _paged_case(cuda, q_lens, prior, seed=11)


def test_prefill_two_streams_concurrently(cuda):
    """Launches on two streams run at the same time; each stream has its own
    work-item counter."""
    cases = []
    for seed in (21, 22):
        b = workloads.make_prefill_batch([300, 520, 64], [900, 10, 2000], seed=seed, device=cuda)
        ops.store_kvcache(b.key, b.value, b.key_cache, b.value_cache, b.slot_mapping)
        cases.append(b)
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    outs = []
    for _ in range(3):
        outs = []
        for b, s in zip(cases, streams):
            with torch.cuda.stream(s):
                outs.append(ops.paged_prefill(b.query, b.key_cache, b.value_cache, b.cu_seqlens_q,
                                              520, b.scale, block_tables=b.block_tables,
                                              context_lens=b.context_lens))
    torch.cuda.synchronize()
    for b, out in zip(cases, outs):
        ref = pa.prefill(b.query.float(), b.key_cache.float(), b.value_cache.float(),
                         b.block_tables, b.context_lens, b.cu_seqlens_q, b.scale)
        assert_attn_close(out, ref)


def test_prefill_block_out_of_range_flags_status(cuda):
    """A block id past the pool is reported (LK_STATUS_BLOCK_OOB) and read as
    zeros instead of faulting; the other sequence is unaffected."""
    b = workloads.make_prefill_batch([50, 50], [100, 100], seed=31, device=cuda)
    ops.store_kvcache(b.key, b.value, b.key_cache, b.value_cache, b.slot_mapping)
    bt = b.block_tables.clone()
    bt[0, 2] = b.key_cache.shape[0] + 7
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = ops.paged_prefill(b.query, b.key_cache, b.value_cache, b.cu_seqlens_q, 50, b.scale,
                            block_tables=bt, context_lens=b.context_lens, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & 2  # LK_STATUS_BLOCK_OOB
    ref = pa.prefill(b.query.float(), b.key_cache.float(), b.value_cache.float(), b.block_tables,
                     b.context_lens, b.cu_seqlens_q, b.scale)
    assert_attn_close(out[50:], ref[50:])


@pytest.mark.parametrize("variant", ["LITEKERN_PREFILL_KERNEL=single",
                                     "LITEKERN_PREFILL_KERNEL=pingpong",
                                     "LITEKERN_PREFILL_MMA_SYNC=1",
                                     "LITEKERN_PREFILL_ORDER=0",
                                     "LITEKERN_PREFILL_SPLIT=0"])
def test_prefill_kernel_options(variant):
    """The kernels kept as options (chosen once per process from the
    environment) against the oracle, in a child process."""
    import os
    import subprocess
    import sys
    key, val = variant.split("=")
    env = dict(os.environ, **{key: val})
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-m", "tests.prefill_variant_check"], cwd=root, env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "ok" in r.stdout


def test_prefill_more_pairs_than_the_order_buffer(cuda):
    """More (sequence, query tile) pairs than the longest-first order buffer
    holds (16384): the kernel falls back to tile-major order. One-token
    sequences in contiguous mode attend to their own key only, so each output
    row is that token's value row exactly."""
    n, H = 16500, 8
    g = torch.Generator(device=cuda).manual_seed(12)
    q = torch.randn((n, H, 128), device=cuda, generator=g).bfloat16()
    k = torch.randn((n, H, 128), device=cuda, generator=g).bfloat16()
    v = torch.randn((n, H, 128), device=cuda, generator=g).bfloat16()
    cu = torch.arange(n + 1, dtype=torch.int32, device=cuda)
    out = ops.paged_prefill(q, k, v, cu, 1, 128 ** -0.5)
    assert torch.equal(out, v)
    # and just under the limit, ordered
    m = 16000
    out = ops.paged_prefill(q[:m], k[:m], v[:m], cu[: m + 1], 1, 128 ** -0.5)
    assert torch.equal(out, v[:m])


def _units_planned(dev):
    """Units of the last prefill plan on the current stream (workspace header)."""
    ws = ops.WORKSPACES.get(dev, f"prefill:{torch.cuda.current_stream(dev).cuda_stream}", 0)
    return int(ws[4:8].view(torch.int32).item())


@pytest.mark.parametrize("H,H_kv", [(32, 8), (8, 8), (64, 8), (16, 2)])
def test_prefill_key_split_tail(cuda, H, H_kv):
    """Few waves of items on very different priors: the plan cuts the late
    long pairs into two key-range pieces (more units than pairs) and the
    merged rows match the oracle, including rows that see no key of the
    second piece."""
    q_lens, prior = [512] * 4, [1986, 2952, 408, 2864]
    _paged_case(cuda, q_lens, prior, H=H, H_kv=H_kv, seed=H + H_kv)
    BQ = 256 // (H // H_kv)
    pairs = 4 * ((512 + BQ - 1) // BQ)
    sms = torch.cuda.get_device_properties(cuda).multi_processor_count
    if sms < pairs * H_kv <= 4 * sms:  # a second wave, at most four: the tail is cut
        assert _units_planned(cuda) > pairs
    else:
        assert _units_planned(cuda) == pairs


def test_prefill_key_split_is_deterministic(cuda):
    """Either piece may end second; the merge order is fixed, so repeated
    launches give identical bits."""
    b, out = _paged_case(cuda, [512] * 4, [1986, 2952, 408, 2864], seed=31)
    for _ in range(5):
        again = ops.paged_prefill(b.query, b.key_cache, b.value_cache, b.cu_seqlens_q, 512,
                                  b.scale, block_tables=b.block_tables,
                                  context_lens=b.context_lens)
        assert torch.equal(again, out)


def test_prefill_split_plan_is_deterministic_with_equal_lengths(cuda):
    """Eight chunks of 512 on equal 8K priors: many pairs share a key-tile
    count, so the plan's buckets are large and the first wave ends inside
    one. The cut is decided per bucket, not per position inside it (which
    the plan's atomics reorder between launches), so twenty launches give
    the same bits; and the result matches the oracle."""
    b, out = _paged_case(cuda, [512] * 8, [8192] * 8, seed=35)
    assert _units_planned(cuda) >= 8 * 8  # whole pairs and pieces
    for _ in range(20):
        again = ops.paged_prefill(b.query, b.key_cache, b.value_cache, b.cu_seqlens_q, 512,
                                  b.scale, block_tables=b.block_tables,
                                  context_lens=b.context_lens)
        assert torch.equal(again, out)


def test_prefill_workspace_too_small_raises(cuda):
    b = workloads.make_prefill_batch([64], [0], seed=32, device=cuda)
    small = torch.zeros(200 * 1024, dtype=torch.uint8, device=cuda)
    with pytest.raises(ValueError):
        ops.paged_prefill(b.query, b.key_cache, b.value_cache, b.cu_seqlens_q, 64, b.scale,
                          block_tables=b.block_tables, context_lens=b.context_lens,
                          workspace=small)


def test_prefill_entry_without_workspace(cuda):
    """lk_paged_prefill (no workspace: plan in the library's per-stream
    buffer, no key splits) on the tail-split case, straight through the C ABI."""
    from litevllm_b200._lib import LK_DTYPE_BF16, check, lib
    q_lens, prior = [512] * 4, [1986, 2952, 408, 2864]
    b = workloads.make_prefill_batch(q_lens, prior, seed=33, device=cuda)
    ops.store_kvcache(b.key, b.value, b.key_cache, b.value_cache, b.slot_mapping)
    out = torch.empty_like(b.query)
    nb, bs, H_kv, D = b.key_cache.shape
    check(lib().lk_paged_prefill(
        out.data_ptr(), b.query.data_ptr(), b.query.stride(0), b.key_cache.data_ptr(),
        b.value_cache.data_ptr(), nb, b.block_tables.data_ptr(), b.block_tables.stride(0),
        b.cu_seqlens_q.data_ptr(), b.context_lens.data_ptr(), 4, 512, b.query.shape[1], H_kv, D,
        bs, b.scale, LK_DTYPE_BF16, None, torch.cuda.current_stream().cuda_stream))
    ref = pa.prefill(b.query.float(), b.key_cache.float(), b.value_cache.float(), b.block_tables,
                     b.context_lens, b.cu_seqlens_q, b.scale)
    assert_attn_close(out, ref)


def test_prefill_block_size_32(cuda):
    """32-slot blocks: each block-table entry covers two 16-slot TMA boxes."""
    _paged_case(cuda, [100, 37, 300], [45, 500, 0], seed=34, bs=32)


def test_prefill_key_split_fp16(cuda):
    """The key-split merge in fp16 (pieces merged in fp32, rounded once)."""
    _paged_case(cuda, [512] * 4, [1986, 2952, 408, 2864], seed=35, dtype=torch.float16)
    assert _units_planned(cuda) > 32
