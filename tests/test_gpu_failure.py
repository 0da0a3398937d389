"""Failure detection on the GPU without a fault: a bounded wait that nothing
satisfies returns an error status within its limit, and the context keeps
working afterwards."""

import time

import pytest
import torch

from litevllm_b200 import _lib, ops, workloads

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_reports(cuda):
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    t = time.perf_counter()
    rc = _lib.lib().lk_selftest_wait_timeout(status.data_ptr(), 5_000_000,  # 5 ms
                                             torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert time.perf_counter() - t < 5.0
    assert int(status.item()) == _lib.LK_STATUS_WAIT_TIMEOUT
    # the context is still usable: a decode right after matches its oracle-checked twin
    b = workloads.make_decode_batch(2, 4, seed=3, device=cuda)
    a = ops.paged_decode(b.query, b.key_cache, b.value_cache, b.block_tables, b.context_lens, b.scale)
    c = ops.paged_decode(b.query, b.key_cache, b.value_cache, b.block_tables, b.context_lens, b.scale)
    assert torch.equal(a, c) and not torch.isnan(a).any()


def test_selftest_rejects_unbounded_limits(cuda):
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    assert _lib.lib().lk_selftest_wait_timeout(status.data_ptr(), 0, None) == -1
    assert _lib.lib().lk_selftest_wait_timeout(status.data_ptr(), 10**12, None) == -1


def test_mma_rate_selftest_completes(cuda):
    """The tensor-core issue-rate probe finishes every shape within its bounded
    wait and reports positive cycles on every SM."""
    nsm = torch.cuda.get_device_properties(cuda).multi_processor_count
    cycles = torch.zeros(nsm, dtype=torch.int64, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    for shape in range(16):
        rc = _lib.lib().lk_selftest_mma_rate(256, shape, cycles.data_ptr(), status.data_ptr(),
                                            None)
        assert rc == 0
        torch.cuda.synchronize()
        assert int(status.item()) == 0 and (cycles > 0).all()
    assert _lib.lib().lk_selftest_mma_rate(0, 0, cycles.data_ptr(), None, None) == -1
    assert _lib.lib().lk_selftest_mma_rate(16, 16, cycles.data_ptr(), None, None) == -1
