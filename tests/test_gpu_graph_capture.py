"""A decode step (KV store, ordering + decode, greedy sampler) captured in a
CUDA graph and replayed with new inputs gives the eager results: no entry point
on the step allocates, synchronises or reads host state that changes between
steps, so engines can capture it as they capture their decode steps."""

import pytest
import torch

from litevllm_b200 import ops, workloads

pytestmark = pytest.mark.gpu


def test_decode_step_graph_replay_matches_eager(cuda):
    b = workloads.make_decode_batch(2, 64, seed=8, device=cuda)
    V = 32000
    logits = torch.randn((64, V), device=cuda).bfloat16()
    out = torch.empty_like(b.query)
    ids = torch.empty(64, dtype=torch.int64, device=cuda)
    nsplit = ops.decode_num_splits(64, 8, b.block_tables.shape[1], 16)

    def step():
        ops.store_kvcache(b.key, b.value, b.key_cache, b.value_cache, b.slot_mapping)
        ops.paged_decode(b.query, b.key_cache, b.value_cache, b.block_tables, b.context_lens,
                         b.scale, num_splits=nsplit, out=out)
        ops.sample(logits, None, out=ids)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()  # first calls on the capture stream: workspaces, tensor maps, function attributes
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g):
            step()
    torch.cuda.synchronize()
    for it in range(3):
        # new step inputs into the captured buffers
        b.query.copy_(torch.randn_like(b.query.float()).bfloat16())
        b.key.copy_(torch.randn_like(b.key.float()).bfloat16())
        b.context_lens.copy_(torch.clamp(b.context_lens - it, min=1))
        logits.copy_(torch.randn_like(logits.float()).bfloat16())
        g.replay()
        torch.cuda.synchronize()
        got_out, got_ids = out.clone(), ids.clone()
        step()
        torch.cuda.synchronize()
        assert torch.equal(got_out, out), it
        assert torch.equal(got_ids, ids), it


def test_shared_prefix_decode_graph_replay(cuda):
    b = workloads.make_prefix_batch(32, seed=6, device=cuda)
    out = torch.empty_like(b.query)

    def step():
        ops.paged_decode_shared_prefix(b.query, b.key_cache, b.value_cache, b.block_tables,
                                       b.context_lens, b.scale, 127 * 16, out=out)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g):
            step()
    torch.cuda.synchronize()
    b.query.copy_(torch.randn_like(b.query.float()).bfloat16())
    g.replay()
    torch.cuda.synchronize()
    got = out.clone()
    step()
    torch.cuda.synchronize()
    assert torch.equal(got, out)
