"""Block copies (copy-on-write and swaps) vs the reference's per-block copy_
loops (litevllm/cache/kv_cache.py:74-102): bit-exact."""

import pytest
import torch

from litevllm_b200 import ops

pytestmark = pytest.mark.gpu


def _caches(L, nb, device, seed, pin=False, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(L):
        k = torch.randn((nb, 16, 8, 128), generator=g).to(dtype)
        v = torch.randn((nb, 16, 8, 128), generator=g).to(dtype)
        if device == "cpu":
            k, v = (k.pin_memory(), v.pin_memory()) if pin else (k, v)
        else:
            k, v = k.to(device), v.to(device)
        out.append((k, v))
    return out


def _reference_copy(src, dst, mapping):
    for s, d in mapping.items():
        for (ks, vs), (kd, vd) in zip(src, dst):
            kd[d].copy_(ks[s].to(kd.device))
            vd[d].copy_(vs[s].to(vd.device))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_copy_on_write_fork(cuda, dtype):
    gpu = _caches(3, 40, cuda, 1, dtype=dtype)
    ref = [(k.clone(), v.clone()) for k, v in gpu]
    mapping = {3: 17, 5: 6, 39: 0, 12: 30}
    ops.copy_blocks(gpu, mapping)
    _reference_copy(ref, ref, mapping)
    for (k, v), (kr, vr) in zip(gpu, ref):
        assert torch.equal(k, kr) and torch.equal(v, vr)


def test_swap_in_and_out_with_pinned_host_caches(cuda):
    gpu = _caches(2, 32, cuda, 2)
    cpu = _caches(2, 24, "cpu", 3, pin=True)
    ref_gpu = [(k.clone(), v.clone()) for k, v in gpu]
    ops.swap_in(gpu, cpu, {0: 5, 23: 31, 7: 0})
    _reference_copy(cpu, ref_gpu, {0: 5, 23: 31, 7: 0})
    torch.cuda.synchronize()
    for (k, v), (kr, vr) in zip(gpu, ref_gpu):
        assert torch.equal(k, kr) and torch.equal(v, vr)
    ref_cpu = [(k.clone(), v.clone()) for k, v in cpu]
    ops.swap_out(gpu, cpu, {31: 2, 1: 20})
    _reference_copy(gpu, ref_cpu, {31: 2, 1: 20})
    for (k, v), (kr, vr) in zip(cpu, ref_cpu):
        assert torch.equal(k, kr) and torch.equal(v, vr)


def test_unpinned_host_cache_is_refused(cuda):
    gpu = _caches(1, 4, cuda, 4)
    cpu = _caches(1, 4, "cpu", 5, pin=False)
    with pytest.raises(RuntimeError, match="pinned"):
        ops.swap_in(gpu, cpu, {0: 1})


def test_out_of_range_pairs_flagged(cuda):
    gpu = _caches(1, 8, cuda, 6)
    before = [(k.clone(), v.clone()) for k, v in gpu]
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    ops.copy_blocks_between(gpu, gpu, torch.tensor([[0, 99], [1, 2]]), status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & 2
    assert torch.equal(gpu[0][0][2], before[0][0][1])
    assert torch.equal(gpu[0][0][0], before[0][0][0])
