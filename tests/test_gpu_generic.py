"""The generic CUDA-core attention kernel (lk_paged_attention_generic) on the GPU.

It serves the shapes the tuned kernels do not take: an fp32 model (the
reference's own CPU configuration, config 1, run on the GPU in its dtype),
head dims other than 128 (Llama-3.2-1B / TinyLlama use 64), block sizes that
are not a multiple of 16, and GQA ratios other than 1/2/4/8. lk_paged_decode
and lk_paged_prefill route such shapes to it, so these tests go through the
same drop-in calls as the tuned kernels' tests, against the fp32 oracle (the
literal _decode_fast restatement for fp32 inputs) and the reference's golden
prefill outputs.
"""

import pytest
import torch

from litevllm_b200 import _lib, ops, workloads
from litevllm_b200.attention import Attention
from oracle import paged_attention as pa
from tests import golden_io
from tests.tolerance import assert_attn_close

pytestmark = pytest.mark.gpu

# fp32 in, fp32 out: only summation order and exp2 rounding differ from the
# fp32 reference.
FP32_MAX_ABS = 1e-4
FP32_MEAN_REL = 1e-5


def test_generic_decode_fp32_config1_through_attention_forward(cuda):
    """Config 1 (Qwen3-0.6B layer: 16 Q / 8 KV heads, D 128, block 16, batch 8,
    contexts in [1, 512], 512-block pool) in fp32: store + decode through the
    drop-in Attention.forward, against the literal _decode_fast restatement."""
    b = workloads.make_decode_batch(1, 8, seed=3, dtype=torch.float32, device=cuda)
    kc_ref, vc_ref = b.key_cache.clone().cpu(), b.value_cache.clone().cpu()
    attn = Attention(16, 128, 8)
    out = attn.forward(b.query, b.key, b.value, b.key_cache, b.value_cache, b.block_tables,
                       b.slot_mapping, b.context_lens, is_prefill=False)
    assert out.dtype == torch.float32
    # the reference's store (attention.py:79-84), then its decode, on the CPU
    slots = b.slot_mapping.cpu()
    kc_ref.view(-1, 8, 128)[slots] = b.key.cpu()
    vc_ref.view(-1, 8, 128)[slots] = b.value.cpu()
    assert torch.equal(b.key_cache.cpu(), kc_ref) and torch.equal(b.value_cache.cpu(), vc_ref)
    ref = pa.decode_batched_reference(b.query.cpu(), kc_ref, vc_ref, b.block_tables.cpu(),
                                      b.context_lens.cpu(), b.scale)
    assert_attn_close(out, ref, FP32_MAX_ABS, FP32_MEAN_REL)
    assert ops.decode_status() == 0


@pytest.mark.parametrize("H,H_kv,D,bs", [
    (32, 8, 64, 16),    # Llama-3.2-1B attention
    (32, 4, 64, 16),    # TinyLlama: G = 8, D = 64
    (32, 2, 128, 16),   # G = 16
    (16, 8, 128, 8),    # 8-slot blocks
    (12, 4, 96, 16),    # G = 3, D = 96
    (16, 8, 256, 16),
    (8, 8, 32, 32),
])
def test_generic_decode_shapes(cuda, H, H_kv, D, bs):
    ctx = [1, 15, 16, 17, 33, 300, 1000]
    b = workloads.make_decode_batch(2, len(ctx), seed=H + D + bs, ctx=ctx, H=H, H_kv=H_kv, D=D,
                                    bs=bs, device=cuda)
    out = ops.paged_decode(b.query, b.key_cache, b.value_cache, b.block_tables, b.context_lens,
                           b.scale)
    ref = pa.decode(b.query.float(), b.key_cache.float(), b.value_cache.float(), b.block_tables,
                    b.context_lens, b.scale)
    assert_attn_close(out, ref)
    assert ops.decode_status() == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_generic_decode_dtypes_long_context(cuda, dtype):
    b = workloads.make_decode_batch(2, 3, seed=21, ctx=[4097, 9000, 2], H=32, H_kv=8, D=64,
                                    dtype=dtype, device=cuda)
    out = ops.paged_decode(b.query, b.key_cache, b.value_cache, b.block_tables, b.context_lens,
                           b.scale)
    ref = pa.decode(b.query, b.key_cache, b.value_cache, b.block_tables, b.context_lens, b.scale)
    if dtype == torch.float32:
        assert_attn_close(out, ref, FP32_MAX_ABS, FP32_MEAN_REL)
    else:
        assert_attn_close(out, ref)


def test_generic_agrees_with_tuned_decode(cuda):
    """On a shape both take (bf16, D 128, G 4), the generic kernel called
    directly and the split kernel agree with the oracle and each other."""
    b = workloads.make_decode_batch(2, 16, seed=22, device=cuda)
    gen = ops.paged_attention_generic(b.query, b.key_cache, b.value_cache, b.scale,
                                      block_tables=b.block_tables, context_lens=b.context_lens)
    tuned = ops.paged_decode(b.query, b.key_cache, b.value_cache, b.block_tables,
                             b.context_lens, b.scale)
    ref = pa.decode(b.query.float(), b.key_cache.float(), b.value_cache.float(), b.block_tables,
                    b.context_lens, b.scale)
    assert_attn_close(gen, ref)
    assert_attn_close(gen, tuned.float())


def test_generic_decode_edge_rows(cuda):
    """Context 0 gives a NaN row (the reference's softmax over all -inf);
    contexts beyond the table are clamped and flagged; out-of-pool block ids
    read zeros and are flagged."""
    b = workloads.make_decode_batch(2, 3, seed=23, ctx=[0, 40, 40], H=16, H_kv=8, D=64,
                                    device=cuda)
    out = ops.paged_decode(b.query, b.key_cache, b.value_cache, b.block_tables, b.context_lens,
                           b.scale)
    assert torch.isnan(out[0]).all() and not torch.isnan(out[1:]).any()
    assert ops.decode_status() == 0
    ctx = b.context_lens.clone()
    ctx[1] = b.block_tables.shape[1] * 16 + 5
    out2 = ops.paged_decode(b.query, b.key_cache, b.value_cache, b.block_tables, ctx, b.scale)
    assert ops.decode_status() & _lib.LK_STATUS_CTX_OOB
    assert torch.equal(out2[1], ops.paged_decode(
        b.query, b.key_cache, b.value_cache, b.block_tables,
        torch.full_like(ctx, b.block_tables.shape[1] * 16), b.scale)[1])
    assert ops.decode_status() == 0
    bt = b.block_tables.clone()
    bt[2, 0] = b.key_cache.shape[0] + 3
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    ops.paged_attention_generic(b.query, b.key_cache, b.value_cache, b.scale, block_tables=bt,
                                context_lens=b.context_lens, status=status)
    assert int(status.item()) & _lib.LK_STATUS_BLOCK_OOB


@pytest.mark.parametrize("dtype,H,H_kv,D,bs", [
    (torch.float32, 16, 8, 128, 16),
    (torch.bfloat16, 32, 8, 64, 16),
    (torch.bfloat16, 24, 8, 128, 16),   # G = 3
    (torch.float16, 32, 8, 128, 8),
])
def test_generic_prefill_prior_context(cuda, dtype, H, H_kv, D, bs):
    q_lens, prior = [1, 17, 64, 33], [0, 5, 100, 250]
    b = workloads.make_prefill_batch(q_lens, prior, seed=24, H=H, H_kv=H_kv, D=D, bs=bs,
                                     dtype=dtype, device=cuda)
    ops.store_kvcache(b.key, b.value, b.key_cache, b.value_cache, b.slot_mapping)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = ops.paged_prefill(b.query, b.key_cache, b.value_cache, b.cu_seqlens_q, max(q_lens),
                            b.scale, block_tables=b.block_tables, context_lens=b.context_lens,
                            status=status)
    ref = pa.prefill(b.query.float(), b.key_cache.float(), b.value_cache.float(), b.block_tables,
                     b.context_lens, b.cu_seqlens_q, b.scale)
    if dtype == torch.float32:
        assert_attn_close(out, ref, FP32_MAX_ABS, FP32_MEAN_REL)
    else:
        assert_attn_close(out, ref)
    assert int(status.item()) == 0


@pytest.mark.parametrize("tag", ["g2", "g4"])
def test_generic_prefill_matches_reference_golden(cuda, tag):
    """Contiguous mode against the reference's own _prefill outputs: bf16 as
    stored, and the same inputs upcast to fp32 through Attention.forward
    (which routes fp32 to the generic kernel)."""
    d = golden_io.load("prefill.npz")
    S, H, H_kv, D = (int(x) for x in d[f"{tag}_shape"])
    q, k, v = (golden_io.bf16(d[f"{tag}_{x}"]).to(cuda) for x in "qkv")
    cu = torch.tensor([0, S], dtype=torch.int32, device=cuda)
    out = ops.paged_attention_generic(q, k, v, 1.0 / D**0.5, cu_seqlens_q=cu, max_q_len=S)
    assert_attn_close(out, torch.from_numpy(d[f"{tag}_out"]))
    out32 = Attention(H, D, H_kv).forward(q.float(), k.float(), v.float(), None, None, None,
                                          None, None, is_prefill=True)
    assert out32.dtype == torch.float32
    ref32 = pa.prefill_contiguous(q.float().cpu(), k.float().cpu(), v.float().cpu())
    assert_attn_close(out32, ref32, FP32_MAX_ABS, FP32_MEAN_REL)


def test_generic_fp32_engine_loop(cuda):
    """fp32 model, engine-shaped: a prefill of each prompt into the paged cache,
    then decode steps across a block boundary, all through Attention.forward,
    checked against the fp32 oracle every step."""
    H, H_kv, D, bs = 16, 8, 128, 16
    prompts = [5, 16, 30]
    n_steps = 4
    nblk = [-(-(p + n_steps) // bs) for p in prompts]
    pool = sum(nblk) + 2
    g = torch.Generator().manual_seed(25)
    kc = torch.zeros((pool, bs, H_kv, D), device=cuda)
    vc = torch.zeros_like(kc)
    bt = torch.zeros((len(prompts), max(nblk)), dtype=torch.int32)
    perm = torch.randperm(pool, generator=g)
    off = 0
    for i, n in enumerate(nblk):
        bt[i, :n] = perm[off:off + n].to(torch.int32)
        off += n
    bt = bt.to(cuda)
    attn = Attention(H, D, H_kv)

    def slot(i, pos):
        return int(bt[i, pos // bs]) * bs + pos % bs

    for i, p in enumerate(prompts):
        q = torch.randn((p, H, D), generator=g).to(cuda)
        k = torch.randn((p, H_kv, D), generator=g).to(cuda)
        v = torch.randn((p, H_kv, D), generator=g).to(cuda)
        sm = torch.tensor([slot(i, j) for j in range(p)], dtype=torch.int64, device=cuda)
        out = attn.forward(q, k, v, kc, vc, None, sm, None, is_prefill=True)
        assert_attn_close(out, pa.prefill_contiguous(q.cpu(), k.cpu(), v.cpu()), FP32_MAX_ABS,
                          FP32_MEAN_REL)
    lens = list(prompts)
    for _ in range(n_steps):
        B = len(prompts)
        q = torch.randn((B, H, D), generator=g).to(cuda)
        k = torch.randn((B, H_kv, D), generator=g).to(cuda)
        v = torch.randn((B, H_kv, D), generator=g).to(cuda)
        sm = torch.tensor([slot(i, lens[i]) for i in range(B)], dtype=torch.int64, device=cuda)
        lens = [n + 1 for n in lens]
        ctx = torch.tensor(lens, dtype=torch.int32, device=cuda)
        out = attn.forward(q, k, v, kc, vc, bt, sm, ctx, is_prefill=False)
        ref = pa.decode_batched_reference(q.cpu(), kc.cpu(), vc.cpu(), bt.cpu(), ctx.cpu(),
                                          attn.scale)
        assert_attn_close(out, ref, FP32_MAX_ABS, FP32_MEAN_REL)
    assert ops.decode_status() == 0


def test_generic_decode_unaligned_caches(cuda):
    """Caches that start 2 bytes past a 16-byte boundary take the kernel's
    element-wise tile loads instead of 16-byte vectors; same results."""
    b = workloads.make_decode_batch(2, 5, seed=26, ctx=[1, 17, 64, 300, 999], H=32, H_kv=8,
                                    D=64, device=cuda)
    n = b.key_cache.numel()
    kbuf = torch.empty(n + 1, dtype=b.key_cache.dtype, device=cuda)
    vbuf = torch.empty_like(kbuf)
    kc = kbuf[1:].view(b.key_cache.shape)
    vc = vbuf[1:].view(b.value_cache.shape)
    kc.copy_(b.key_cache)
    vc.copy_(b.value_cache)
    assert kc.data_ptr() % 16 != 0
    out = ops.paged_decode(b.query, kc, vc, b.block_tables, b.context_lens, b.scale)
    aligned = ops.paged_decode(b.query, b.key_cache, b.value_cache, b.block_tables,
                               b.context_lens, b.scale)
    ref = pa.decode(b.query.float(), b.key_cache.float(), b.value_cache.float(), b.block_tables,
                    b.context_lens, b.scale)
    assert_attn_close(out, ref)
    assert torch.equal(out, aligned)


@pytest.mark.parametrize("D,dtype,H,H_kv", [
    (64, torch.bfloat16, 32, 8), (64, torch.float32, 32, 8), (64, torch.float16, 32, 8),
    (32, torch.bfloat16, 32, 8), (96, torch.float16, 16, 4), (128, torch.float32, 32, 8),
    (256, torch.bfloat16, 16, 8), (128, torch.bfloat16, 32, 2), (128, torch.float16, 64, 4)])
def test_generic_split_decode_matches_single_pass(cuda, D, dtype, H, H_kv):
    """lk_paged_decode splits long contexts across CTAs for the generic kernel
    (partials merged by a second launch); lk_paged_attention_generic runs one
    CTA per row. Both match the oracle, an empty split included (row 3 is far
    shorter than the table), over head dims 32-256, three dtypes and G = 16
    (the split kernel takes G <= 8 only)."""
    b = workloads.make_decode_batch(2, 5, seed=27 + D, ctx=[5000, 700, 31, 2048, 0], H=H,
                                    H_kv=H_kv, D=D, dtype=dtype, device=cuda)
    mb = b.block_tables.shape[1]
    assert _lib.lib().lk_paged_attention_generic_workspace_bytes(5, H, D, mb, 16) > 256
    split = ops.paged_decode(b.query, b.key_cache, b.value_cache, b.block_tables,
                             b.context_lens, b.scale)
    single = ops.paged_attention_generic(b.query, b.key_cache, b.value_cache, b.scale,
                                         block_tables=b.block_tables,
                                         context_lens=b.context_lens)
    ref = pa.decode(b.query.float(), b.key_cache.float(), b.value_cache.float(), b.block_tables,
                    b.context_lens, b.scale)
    tol = (FP32_MAX_ABS, FP32_MEAN_REL) if dtype == torch.float32 else ()
    assert_attn_close(split, ref, *tol)
    assert_attn_close(single, ref, *tol)
    assert torch.isnan(split[4]).all()
    assert ops.decode_status() == 0


def test_generic_decode_with_small_caller_workspace(cuda):
    """A caller workspace sized for the split kernel only (below the generic
    kernel's full split size) gives fewer splits, not an error; same results."""
    b = workloads.make_decode_batch(2, 4, seed=28, ctx=[6000, 1, 513, 4096], H=32, H_kv=8,
                                    D=64, device=cuda)
    mb = b.block_tables.shape[1]
    ns = ops.decode_num_splits(4, 8, mb, 16)
    small = ops.decode_workspace_bytes(4, 32, 8, 64, ns)
    full = _lib.lib().lk_paged_attention_generic_workspace_bytes(4, 32, 64, mb, 16)
    assert small < full
    ws = torch.zeros(small, dtype=torch.uint8, device=cuda)
    out = ops.paged_decode(b.query, b.key_cache, b.value_cache, b.block_tables, b.context_lens,
                           b.scale, workspace=ws)
    ref = pa.decode(b.query.float(), b.key_cache.float(), b.value_cache.float(), b.block_tables,
                    b.context_lens, b.scale)
    assert_attn_close(out, ref)
    assert ops.decode_status(ws) == 0


def test_generic_split_then_tuned_decode_share_a_workspace(cuda):
    """The generic split partials sit after the split kernel's counter region:
    a tuned decode that reuses the same workspace after a generic split decode
    still finds its counters zero and matches the oracle."""
    g = workloads.make_decode_batch(2, 8, seed=29, ctx=[4096] * 8, H=32, H_kv=8, D=64,
                                    device=cuda)
    t = workloads.make_decode_batch(2, 32, seed=30, device=cuda)
    need = max(_lib.lib().lk_paged_attention_generic_workspace_bytes(8, 32, 64, 256, 16),
               ops.decode_workspace_bytes(32, 32, 8, 128, 8))
    ws = torch.zeros(need, dtype=torch.uint8, device=cuda)
    for _ in range(2):
        ops.paged_decode(g.query, g.key_cache, g.value_cache, g.block_tables, g.context_lens,
                         g.scale, workspace=ws)
        out = ops.paged_decode(t.query, t.key_cache, t.value_cache, t.block_tables,
                               t.context_lens, t.scale, num_splits=8, workspace=ws)
        ref = pa.decode(t.query.float(), t.key_cache.float(), t.value_cache.float(),
                        t.block_tables, t.context_lens, t.scale)
        assert_attn_close(out, ref)
    assert ops.decode_status(ws) == 0
