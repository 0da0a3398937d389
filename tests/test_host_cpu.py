"""Host-side logic on CPU: workload keying, request sharding (2 gloo ranks),
and the drop-in install into the reference package."""

import os
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

from litevllm_b200 import sharding, workloads

# the reference checkout: LITEVLLM_REFERENCE, else a "reference" directory
# beside this repository
REF = Path(os.environ.get("LITEVLLM_REFERENCE")
           or Path(__file__).resolve().parent.parent.parent / "reference")


def test_shards_partition_the_batch():
    for G in (1, 7, 64, 256, 257):
        for W in (1, 2, 3, 8):
            got = [i for r in range(W) for i in sharding.shard(G, W, r)]
            assert got == list(range(G))


def test_balanced_shards_partition_and_balance():
    for G, W in ((64, 8), (2048, 8), (64, 3), (10, 4), (5, 8)):
        lens = [workloads.context_len(5, 0, i) for i in range(G)]
        parts = [sharding.balanced_shard(lens, W, r) for r in range(W)]
        assert sorted(i for p in parts for i in p) == list(range(G))
        counts = [len(p) for p in parts]
        assert max(counts) - min(counts) <= 1
        if G % W == 0 and G >= 2 * W:
            sums = [sum(lens[i] for i in p) for p in parts]
            contiguous = [sum(lens[i] for i in sharding.shard(G, W, r)) for r in range(W)]
            # the slowest rank carries less than with contiguous blocks
            assert max(sums) <= max(contiguous)
            assert max(sums) - min(sums) <= max(lens) - min(lens)


def test_context_lengths_keyed_by_global_index():
    full = [workloads.context_len(2, 0, i) for i in range(64)]
    assert all(16 <= c <= 4096 for c in full)
    assert 700 < sorted(full)[32] < 1500  # median near 1024
    for W in (2, 4, 8):
        parts = []
        for r in range(W):
            parts += [workloads.context_len(2, 0, i) for i in sharding.shard(64, W, r)]
        assert parts == full
    c5 = [workloads.context_len(5, 0, i) for i in range(16)]
    assert all(32768 <= c <= 131072 for c in c5)


def test_decode_batch_tables_are_disjoint():
    b = workloads.make_decode_batch(2, 32, seed=1, device="cpu", dtype=torch.float32)
    used = []
    for i, c in enumerate(b.ctx):
        n = -(-c // 16)
        used += b.block_tables[i, :n].tolist()
        assert (b.block_tables[i, n:] == 0).all()
        assert b.slot_mapping[i] == b.block_tables[i, (c - 1) // 16] * 16 + (c - 1) % 16
    assert len(used) == len(set(used))


def _rank_main(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = list(sharding.shard(10, world, rank))
        ctx = [workloads.context_len(2, 0, i) for i in mine]
        # rank-dependent "step time": the max over ranks must come back everywhere
        m = sharding.max_over_ranks([1.0 + rank, 5.0 - rank])
        out = [None] * world
        torch.distributed.all_gather_object(out, (mine, ctx))
        q.put((rank, m, out))
    finally:
        torch.distributed.destroy_process_group()


def test_two_rank_gloo_sharding_and_max_timing():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, m, out in res:
        assert m == [2.0, 5.0]
        idx = out[0][0] + out[1][0]
        assert idx == list(range(10))
        assert out[0][1] + out[1][1] == [workloads.context_len(2, 0, i) for i in range(10)]


@pytest.mark.skipif(not (REF / "litevllm").exists(), reason="reference checkout not present")
def test_install_patches_reference_namespace():
    sys.path.insert(0, str(REF))
    try:
        import litevllm.layers as L
        import litevllm.layers.attention as LA
        import litevllm.layers.sampler as LS

        from litevllm_b200 import install
        from litevllm_b200.attention import Attention
        from litevllm_b200.sampler import Sampler

        sites = install()
        assert LA.Attention is Attention and L.Attention is Attention
        assert LS.Sampler is Sampler
        assert "litevllm.layers.attention.Attention" in sites
        import litevllm.models.qwen3 as Q

        assert Q.Attention is Attention
        # the optional hooks: engine methods, merged steps, fused norm + RoPE + store
        import litevllm.engine.llm_engine as E
        import litevllm.engine.model_runner as MR
        import litevllm.models.llama as LL

        from litevllm_b200 import engine_hooks, model_hooks

        saved = (MR.ModelRunner.prepare_inputs, E.LLMEngine._process_outputs, E.LLMEngine.step,
                 Q.Qwen3Attention.forward, LL.LlamaAttention.forward)
        try:
            sites = install(engine_hooks=True, merged_steps=True, fused_rope=True)
            assert MR.ModelRunner.prepare_inputs is engine_hooks.prepare_inputs
            assert E.LLMEngine._process_outputs is engine_hooks.process_outputs
            assert E.LLMEngine.step is engine_hooks.merged_step
            assert Q.Qwen3Attention.forward is model_hooks.fused_forward
            assert LL.LlamaAttention.forward is model_hooks.fused_forward
            assert "litevllm.models.qwen3.Qwen3Attention.forward" in sites
            # the unfused forward stays reachable for shapes the kernel does not take
            assert model_hooks._ORIGINAL[Q.Qwen3Attention] is saved[3]
        finally:
            (MR.ModelRunner.prepare_inputs, E.LLMEngine._process_outputs, E.LLMEngine.step,
             Q.Qwen3Attention.forward, LL.LlamaAttention.forward) = saved
    finally:
        sys.path.remove(str(REF))


def _rank_dies(rank, world, port, q):
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world,
                                         timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # a worker that leaves between steps, nothing in flight
    try:
        torch.distributed.barrier()
        q.put((rank, "no error"))
    except Exception as e:  # the survivor learns of it on the host
        q.put((rank, type(e).__name__))


def test_dead_rank_is_detected_by_timed_barrier():
    """A rank that exits between steps: the other rank's next barrier fails
    within the process-group timeout instead of hanging."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank_dies, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    rank, outcome = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert rank == 0 and outcome != "no error"
