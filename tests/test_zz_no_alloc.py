"""The allocation-free sampler entry point, lk_sample_noalloc.

Some callers cannot call cudaMalloc when they sample (the allocator is owned
by someone else at that moment, device allocation is forbidden after
start-up, or a plugin is handed only its input and output buffers). This
entry point keeps its scratch in a static device array instead of a
workspace. The test calls it through the C ABI and checks it against the
workspace entry point, lk_sample, on two calls in a row (the second call
finds the array as the first left it). It is collected last so that a run
that stops at the first failure has run everything else, and it passes both
alone in a fresh process and after the other tests.
"""

import ctypes

import numpy as np
import pytest
import torch

from litevllm_b200 import _lib, ops, workloads

pytestmark = pytest.mark.gpu

LK_ERR_TOO_LARGE = -7


def _noalloc(logits, temps=None, noise=None, seed=0, offset=0):
    B, V = logits.shape
    out = torch.full((B,), -1, dtype=torch.int64, device=logits.device)
    code = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[logits.dtype]
    rc = _lib.lib().lk_sample_noalloc(
        out.data_ptr(), logits.data_ptr(), B, V, logits.stride(0),
        None if temps is None else temps.data_ptr(),
        None if noise is None else noise.data_ptr(), 0 if noise is None else noise.stride(0),
        seed, offset, None, code, torch.cuda.current_stream().cuda_stream)
    return rc, out


@pytest.mark.parametrize("B,V", [(8, 151936), (256, 128256), (3, 1000)])
def test_noalloc_matches_workspace_entry_two_calls(cuda, B, V):
    for call in range(2):
        x = workloads.make_logits(1, B, V, seed=40 + call, dtype=torch.bfloat16, device=cuda)
        t = workloads.temperatures_for(1, B, device=cuda)
        n = workloads.gumbel_noise(B, V, seed=50 + call, device=cuda)
        rc, got = _noalloc(x, t, n)
        assert rc == 0, _lib.lib().lk_status_string(rc)
        want = ops.sample(x, t, noise=n)
        assert torch.equal(got, want), f"call {call}"
        # in-kernel noise: same seed / offset -> same ids as the workspace entry
        rc, got = _noalloc(x, t, None, seed=7, offset=call)
        assert rc == 0
        assert torch.equal(got, ops.sample(x, t, seed=7, offset=call))


def test_noalloc_rejects_oversized_problem(cuda):
    x = torch.zeros((9000, 16), device=cuda)
    rc, out = _noalloc(x)
    assert rc == LK_ERR_TOO_LARGE
    assert b"static scratch" in _lib.lib().lk_status_string(rc)
    assert (out == -1).all()


def _noalloc_dump(logits, temps, seed, offset):
    B, V = logits.shape
    out = torch.full((B,), -1, dtype=torch.int64, device=logits.device)
    dump = torch.zeros((B, V), device=logits.device)
    code = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[logits.dtype]
    rc = _lib.lib().lk_sample_noalloc(
        out.data_ptr(), logits.data_ptr(), B, V, logits.stride(0), temps.data_ptr(), None, 0,
        seed, offset, dump.data_ptr(), code, torch.cuda.current_stream().cuda_stream)
    return rc, out, dump


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("B,V", [(256, 128256), (8, 151936), (64, 4000)])
def test_noalloc_greedy_matches_oracle_two_calls(cuda, dtype, B, V):
    """temperatures == NULL: the all-greedy path (cluster merge for 16-bit
    logits, the general kernel for fp32) against the oracle's argmax, with
    planted ties across the row, on two calls in a row."""
    from oracle import sampler as osamp

    for call in range(2):
        x = workloads.make_logits(2, B, V, seed=60 + call, dtype=dtype, device=cuda)
        x[:, V // 3] = x.max() + 1           # a tie between two far-apart columns
        x[:, V - 5] = x[:, V // 3]
        rc, got = _noalloc(x)
        assert rc == 0, _lib.lib().lk_status_string(rc)
        want = osamp.greedy(x.float().cpu().numpy())
        assert got.cpu().numpy().tolist() == want.tolist(), f"call {call}"
        assert (got.cpu().numpy() == V // 3).all()
        assert torch.equal(got, ops.sample(x, None))


@pytest.mark.parametrize("B,V", [(256, 524288), (300, 524288)])
def test_noalloc_in_kernel_noise_at_the_scratch_limit(cuda, B, V):
    """In-kernel noise with the noise dumped: the ids equal the oracle's given
    the dump. 256 rows x 64 chunks fill the 16384 partial slots exactly; 300
    rows make the entry lengthen its chunks to stay within them."""
    from oracle import sampler as osamp

    for call in range(2):
        x = workloads.make_logits(4, B, V, seed=70 + call, device=cuda)
        t = torch.full((B,), 0.8, device=cuda)
        t[::5] = 0.0
        rc, got, dump = _noalloc_dump(x, t, seed=123, offset=call)
        assert rc == 0, _lib.lib().lk_status_string(rc)
        want = osamp.gumbel(x.float().cpu().numpy(), t.cpu().numpy(), dump.cpu().numpy())
        assert np.array_equal(got.cpu().numpy(), want), f"call {call}"
        del dump


def test_noalloc_allocates_nothing(cuda):
    """After a first call (which loads the kernels and looks up the scratch
    address), further calls change neither torch's allocator nor the device's
    free memory: every buffer here is allocated before the first call."""
    B, V = 128, 151936
    x = workloads.make_logits(4, B, V, seed=5, device=cuda)
    t = torch.full((B,), 0.7, device=cuda)
    out = torch.empty(B, dtype=torch.int64, device=cuda)
    stream = torch.cuda.current_stream().cuda_stream

    def call(temps, offset):
        rc = _lib.lib().lk_sample_noalloc(
            out.data_ptr(), x.data_ptr(), B, V, V, None if temps is None else temps.data_ptr(),
            None, 0, 1, offset, None, 2, stream)
        assert rc == 0

    call(t, 1)
    call(None, 1)
    torch.cuda.synchronize()
    before = (torch.cuda.memory_allocated(cuda), torch.cuda.mem_get_info(cuda)[0])
    for i in range(3):
        call(t, 2 + i)
        call(None, 2 + i)
    torch.cuda.synchronize()
    after = (torch.cuda.memory_allocated(cuda), torch.cuda.mem_get_info(cuda)[0])
    assert after == before
