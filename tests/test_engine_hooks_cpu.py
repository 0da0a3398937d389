"""Engine hooks vs the reference engine methods, on CPU: the vectorised
prepare_inputs must build exactly the reference's tensors, and the batched
process_outputs must leave sequences exactly as the reference's per-sequence
loop does (greedy rows; the GPU sampler is replaced by argmax here)."""

import os
import sys
import types
from pathlib import Path

import pytest
import torch

# the reference checkout: LITEVLLM_REFERENCE, else a "reference" directory
# beside this repository
REF = Path(os.environ.get("LITEVLLM_REFERENCE")
           or Path(__file__).resolve().parent.parent.parent / "reference")
pytestmark = pytest.mark.skipif(not (REF / "litevllm").exists(),
                                reason="reference checkout not present")


@pytest.fixture(scope="module")
def ref():
    sys.path.insert(0, str(REF))
    from litevllm.cache.block_manager import BlockManager
    from litevllm.config import CacheConfig, SamplingParams, SchedulerConfig
    from litevllm.engine import llm_engine, model_runner
    from litevllm.engine.scheduler import Scheduler
    from litevllm.engine.sequence import SequenceGroup

    yield types.SimpleNamespace(BlockManager=BlockManager, CacheConfig=CacheConfig,
                                SamplingParams=SamplingParams, SchedulerConfig=SchedulerConfig,
                                Scheduler=Scheduler, SequenceGroup=SequenceGroup,
                                ModelRunner=model_runner.ModelRunner,
                                LLMEngine=llm_engine.LLMEngine)
    sys.path.remove(str(REF))


def _schedule(ref, prompts, steps_of_decode=0, block_size=16):
    cache = ref.CacheConfig(block_size=block_size, num_gpu_blocks=256)
    sched = ref.Scheduler(ref.SchedulerConfig(max_num_seqs=16, max_num_batched_tokens=4096,
                                              chunked_prefill=False, chunk_size=4096),
                          cache, ref.BlockManager(block_size=block_size, num_gpu_blocks=256))
    for i, p in enumerate(prompts):
        sched.add_request(ref.SequenceGroup.create(f"r{i}", p, ref.SamplingParams(temperature=0.0)))
    return sched


def _runner(ref, block_size=16):
    return types.SimpleNamespace(config=types.SimpleNamespace(
        cache_config=types.SimpleNamespace(block_size=block_size)), device="cpu")


def _same(a, b):
    assert a.is_prefill == b.is_prefill and a.seq_ids == b.seq_ids
    for name in ("input_ids", "positions", "slot_mapping", "block_tables", "context_lens"):
        x, y = getattr(a, name), getattr(b, name)
        if x is None or y is None:
            assert x is None and y is None, name
        else:
            assert x.dtype == y.dtype and torch.equal(x, y), name


def test_prepare_inputs_matches_reference_prefill_and_decode(ref, monkeypatch):
    from litevllm_b200 import engine_hooks

    sched = _schedule(ref, [list(range(3, 40)), list(range(7, 12)), list(range(1, 70))])
    out = sched.schedule()
    groups = out.scheduled_seq_groups
    runner = _runner(ref)
    runner.prepare_inputs = types.MethodType(engine_hooks.prepare_inputs, runner)
    # prepare_inputs finds InputMetadata in the module of the runner's class;
    # the stand-in runner's class lives in `types`
    import litevllm.engine.model_runner as mr
    monkeypatch.setattr(sys.modules[type(runner).__module__], "InputMetadata", mr.InputMetadata,
                        raising=False)
    want = ref.ModelRunner.prepare_inputs(runner, groups, sched.block_manager)
    got = engine_hooks.prepare_inputs(runner, groups, sched.block_manager)
    _same(got, want)
    assert got.is_prefill
    # move every sequence to decode and grow it across a block boundary
    for sg in groups:
        for seq in sg.get_unfinished_seqs():
            seq.num_computed_tokens = seq.data.prompt_len
            for t in range(12):
                seq.data.append_token(100 + t)
                table = sched.block_manager.get_block_table(seq.seq_id)
                if seq.get_num_blocks(16) > len(table):
                    sched.block_manager.append_slot(seq.seq_id)
    want = ref.ModelRunner.prepare_inputs(runner, groups, sched.block_manager)
    got = engine_hooks.prepare_inputs(runner, groups, sched.block_manager)
    _same(got, want)
    assert not got.is_prefill and got.block_tables.shape[0] == 3
    # the shared-prefix hint belongs to this step's table (no shared blocks here)
    from litevllm_b200 import attention
    assert attention._SHARED_PREFIX["table"] is got.block_tables
    assert attention._SHARED_PREFIX["tokens"] == 0


def test_process_outputs_matches_reference(ref, monkeypatch):
    from litevllm_b200 import engine_hooks
    from litevllm_b200.sampler import Sampler

    monkeypatch.setattr(Sampler, "sample_batch",
                        staticmethod(lambda logits, temps=None, **kw: logits.argmax(-1)))
    # (greedy rows; the filter arguments stay None)
    prompts = [list(range(3, 20)), list(range(5, 9)), list(range(2, 40))]
    logits = torch.randn(17 + 4 + 38, 50)

    def run(fn):
        sched = _schedule(ref, prompts)
        groups = sched.schedule().scheduled_seq_groups
        eng = types.SimpleNamespace(
            sampler=types.SimpleNamespace(sample=lambda lg, p: lg.argmax(-1)),
            _should_stop=lambda seq, p, tok: ref.LLMEngine._should_stop(eng, seq, p, tok),
            tokenizer=types.SimpleNamespace(eos_token_id=7, decode=lambda ids, **k: ""))
        fn(eng, logits, groups)
        return [(s.data.output_token_ids, s.num_computed_tokens, s.status)
                for g in groups for s in g.seqs]

    assert run(engine_hooks.process_outputs) == run(ref.LLMEngine._process_outputs)


def test_shared_prefix_tokens_counts_whole_shared_filled_blocks():
    import numpy as np
    from litevllm_b200.engine_hooks import shared_prefix_tokens

    a = np.array([5, 9, 2, 7, 1])
    b = np.array([5, 9, 2, 8])
    c = np.array([5, 9, 2, 7, 4, 6])
    assert shared_prefix_tokens([a, b, c], [80, 64, 90], 16) == 48      # 3 shared blocks
    assert shared_prefix_tokens([a, b, c], [80, 40, 90], 16) == 32      # row 1 filled only 2
    assert shared_prefix_tokens([a, c], [80, 90], 16) == 64             # 4 shared, all filled
    assert shared_prefix_tokens([a], [80], 16) == 0                     # one row: nothing shared
    assert shared_prefix_tokens([a, np.array([6, 9])], [80, 32], 16) == 0


def test_prepare_inputs_mixed_matches_reference_per_group(ref, monkeypatch):
    """One merged step (prefill chunks, then decodes) carries exactly the
    token data of the reference's per-group prepare_inputs calls
    (llm_engine.py:127-138), plus a table and context length for every row
    and cu_seqlens_q for the chunks."""
    import numpy as np

    from litevllm_b200 import attention, engine_hooks
    import litevllm.engine.model_runner as mr

    sched = _schedule(ref, [list(range(3, 40)), list(range(7, 30))])
    first = sched.schedule().scheduled_seq_groups
    for sg in first:  # both become decodes that have crossed a block boundary
        for seq in sg.get_unfinished_seqs():
            seq.num_computed_tokens = seq.data.prompt_len
            for t in range(5):
                seq.data.append_token(200 + t)
                if seq.get_num_blocks(16) > len(sched.block_manager.get_block_table(seq.seq_id)):
                    sched.block_manager.append_slot(seq.seq_id)
    sched.update_running(first)
    for i, p in enumerate([list(range(50, 83)), list(range(9, 14))]):
        sched.add_request(ref.SequenceGroup.create(f"n{i}", p, ref.SamplingParams(temperature=0.0)))
    groups = sched.schedule().scheduled_seq_groups
    prefill = [g for g in groups if any(s.is_prefill for s in g.get_unfinished_seqs())]
    decode = [g for g in groups if not any(s.is_prefill for s in g.get_unfinished_seqs())]
    assert len(prefill) == 2 and len(decode) == 2
    runner = _runner(ref)
    monkeypatch.setattr(sys.modules[type(runner).__module__], "InputMetadata", mr.InputMetadata,
                        raising=False)
    bm = sched.block_manager
    got = engine_hooks.prepare_inputs_mixed(runner, prefill, decode, bm)
    want_p = [ref.ModelRunner.prepare_inputs(runner, [g], bm) for g in prefill]
    want_d = ref.ModelRunner.prepare_inputs(runner, decode, bm)
    for name in ("input_ids", "positions", "slot_mapping"):
        want = torch.cat([getattr(w, name) for w in want_p] + [getattr(want_d, name)])
        assert torch.equal(getattr(got, name), want), name
    assert got.seq_ids == sum((w.seq_ids for w in want_p), []) + want_d.seq_ids
    P = len(prefill)
    # decode rows: the reference's tables (zero padded further) and lengths
    mb = want_d.block_tables.shape[1]
    assert torch.equal(got.block_tables[P:, :mb], want_d.block_tables)
    assert not got.block_tables[P:, mb:].any()
    assert torch.equal(got.context_lens[P:], want_d.context_lens)
    # prefill rows: their whole tables, context = prior + chunk = prompt length
    for i, g in enumerate(prefill):
        seq = g.get_unfinished_seqs()[0]
        ids = bm.get_block_table(seq.seq_id).physical_block_ids
        assert got.block_tables[i, :len(ids)].tolist() == ids
        assert int(got.context_lens[i]) == seq.data.prompt_len
    hint = attention._MIXED_STEP
    q_lens = [w.input_ids.numel() for w in want_p]
    assert hint["table"] is got.block_tables and hint["P"] == P
    assert hint["TP"] == sum(q_lens) and hint["max_q_len"] == max(q_lens)
    assert hint["cu_seqlens_q"].tolist() == [0] + np.cumsum(q_lens).tolist()
    # a step without chunks is the plain decode metadata, hint cleared
    plain = engine_hooks.prepare_inputs_mixed(runner, [], decode, bm)
    _same(plain, want_d)
    assert attention._MIXED_STEP["table"] is None
