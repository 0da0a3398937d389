"""The engine hooks on the GPU: a merged step (engine_hooks.prepare_inputs_mixed
-> the drop-in Attention.forward -> engine_hooks.process_outputs with the
drop-in Sampler) over stand-in engine objects with the reference's fields
(Sequence / SequenceGroup / BlockManager, litevllm/engine/sequence.py,
cache/block_manager.py). The metadata is the reference's per-group
prepare_inputs data (shown on CPU against the reference itself by
tests/test_engine_hooks_cpu.py); here every row's attention is checked
against the fp32 oracle: decode rows against _decode_fast's restatement,
prefill chunks against the prior-context prefill (which is the reference's
_prefill for chunks starting at position 0), and the sampled tokens against
the oracle's greedy argmax."""

import sys
import types

import numpy as np
import pytest
import torch

from litevllm_b200 import attention, engine_hooks, workloads
from litevllm_b200.attention import Attention
from oracle import paged_attention as pa
from oracle import sampler as osamp
from tests.tolerance import assert_attn_close

pytestmark = pytest.mark.gpu


class InputMetadata:
    """The reference InputMetadata's fields (engine/model_runner.py:84-103)."""

    def __init__(self, **kw):
        self.__dict__.update(kw)


def _seq(seq_id, prompt, generated, computed):
    toks = list(prompt) + list(generated)
    data = types.SimpleNamespace(prompt_len=len(prompt), prompt_token_ids=list(prompt),
                                 all_token_ids=toks, total_len=len(toks),
                                 output_token_ids=list(generated))
    data.append_token = lambda t, d=data: (d.all_token_ids.append(t), d.output_token_ids.append(t))
    return types.SimpleNamespace(seq_id=seq_id, data=data, num_computed_tokens=computed,
                                 is_prefill=computed < len(prompt))


def _group(seq, temperature=0.0):
    sp = types.SimpleNamespace(temperature=temperature, top_k=-1, top_p=1.0,
                               repetition_penalty=1.0)
    return types.SimpleNamespace(seqs=[seq], get_unfinished_seqs=lambda s=seq: [s],
                                 sampling_params=sp)


def test_merged_step_matches_oracle_per_row(cuda, monkeypatch):
    H, H_kv, D, bs = 32, 8, 128, 16
    gen = torch.Generator().manual_seed(31)
    rng = np.random.default_rng(31)
    # prefill: two first chunks and one later chunk (64 prior tokens computed)
    specs = [("p", 37, 0), ("p", 300, 0), ("p", 150, 64)]
    # decode: contexts across block boundaries
    specs += [("d", c, None) for c in (1, 16, 17, 700, 2049)]
    total_blocks = sum(-(-(n + 1) // bs) for _, n, _ in specs) + 4
    perm = rng.permutation(total_blocks)
    tables, groups_p, groups_d, off = {}, [], [], 0
    for i, (kind, n, computed) in enumerate(specs):
        if kind == "p":
            seq = _seq(i, rng.integers(0, 1000, n).tolist(), [], computed)
            nb = -(-n // bs)
        else:
            seq = _seq(i, rng.integers(0, 1000, max(1, n - 1)).tolist(), [7] if n > 1 else [], n)
            seq.num_computed_tokens = seq.data.prompt_len
            seq.is_prefill = False
            nb = -(-seq.data.total_len // bs)
        tables[i] = perm[off:off + nb].tolist()
        off += nb
        (groups_p if kind == "p" else groups_d).append(_group(seq))
    bm = types.SimpleNamespace(get_block_table=lambda sid: types.SimpleNamespace(
        physical_block_ids=tables[sid]))
    runner = types.SimpleNamespace(config=types.SimpleNamespace(
        cache_config=types.SimpleNamespace(block_size=bs)), device=str(cuda))
    monkeypatch.setattr(sys.modules[type(runner).__module__], "InputMetadata", InputMetadata,
                        raising=False)
    md = engine_hooks.prepare_inputs_mixed(runner, groups_p, groups_d, bm)
    N = md.input_ids.numel()
    kc = torch.randn((total_blocks, bs, H_kv, D), generator=gen).bfloat16().to(cuda)
    vc = torch.randn((total_blocks, bs, H_kv, D), generator=gen).bfloat16().to(cuda)
    q = torch.randn((N, H, D), generator=gen).bfloat16().to(cuda)
    k = torch.randn((N, H_kv, D), generator=gen).bfloat16().to(cuda)
    v = torch.randn((N, H_kv, D), generator=gen).bfloat16().to(cuda)
    attn = Attention(H, D, H_kv)
    out = attn.forward(q, k, v, kc, vc, md.block_tables, md.slot_mapping, md.context_lens,
                       md.is_prefill)
    torch.cuda.synchronize()
    # the stored slots hold this step's K / V
    flat_k = kc.view(-1, H_kv, D)
    assert torch.equal(flat_k[md.slot_mapping], k)
    hint = attention._MIXED_STEP
    P, TP = hint["P"], hint["TP"]
    ref_p = pa.prefill(q[:TP].float(), kc.float(), vc.float(), md.block_tables[:P],
                       md.context_lens[:P], hint["cu_seqlens_q"], attn.scale)
    assert_attn_close(out[:TP], ref_p)
    ref_d = pa.decode(q[TP:].float(), kc.float(), vc.float(), md.block_tables[P:],
                      md.context_lens[P:], attn.scale)
    assert_attn_close(out[TP:], ref_d)
    # chunks from position 0: the reference's own _prefill over the chunk alone
    cu = hint["cu_seqlens_q"].tolist()
    for b in (0, 1):
        s0, s1 = cu[b], cu[b + 1]
        assert_attn_close(out[s0:s1], pa.prefill_contiguous(q[s0:s1].cpu(), k[s0:s1].cpu(),
                                                            v[s0:s1].cpu()))

    # sampling the step's logits through the batched output hook (greedy rows)
    V = 5000
    logits = torch.randn((N, V), generator=gen).bfloat16().to(cuda)
    stops = []
    eng = types.SimpleNamespace(sampler=None,
                                _should_stop=lambda seq, p, tok: stops.append(seq.seq_id))
    engine_hooks.process_outputs(eng, logits, groups_p + groups_d)
    want = osamp.greedy(logits.float().cpu().numpy())
    rows = [c - 1 for c in cu[1:]] + list(range(TP, N))
    got = [g.seqs[0].data.all_token_ids[-1] for g in groups_p + groups_d]
    assert got == [int(want[r]) for r in rows]
    assert all(g.seqs[0].num_computed_tokens == g.seqs[0].data.prompt_len for g in groups_p)
    attention.set_mixed_step_hint(None)
