"""KV store on the GPU vs the reference / oracle: bit-exact."""

import numpy as np
import pytest
import torch

from litevllm_b200 import ops, workloads
from oracle import store_kv as ostore
from tests import golden_io

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["store_decode.npz", "decode_g4.npz"])
def test_store_matches_reference_golden(cuda, name):
    d = golden_io.decode_case(name)
    kc, vc = d["key_cache"].to(cuda), d["value_cache"].to(cuda)
    kc0 = kc.clone()
    ops.store_kvcache(d["key"].to(cuda), d["value"].to(cuda), kc, vc, d["slot_mapping"].to(cuda))
    H_kv, D = int(d["H_kv"]), int(d["D"])
    slots = d["slot_mapping"].to(cuda)
    assert torch.equal(kc.view(-1, H_kv, D)[slots].cpu().view(torch.int16), d["stored_k"].view(torch.int16))
    assert torch.equal(vc.view(-1, H_kv, D)[slots].cpu().view(torch.int16), d["stored_v"].view(torch.int16))
    mask = torch.ones(kc.numel() // (H_kv * D), dtype=torch.bool, device=cuda)
    mask[slots] = False
    assert torch.equal(kc.view(-1, H_kv, D)[mask], kc0.view(-1, H_kv, D)[mask])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("T,H_kv,D", [(1, 8, 128), (300, 8, 128), (77, 2, 64), (5, 3, 40), (9, 3, 36)])
def test_store_matches_oracle_whole_pool(cuda, dtype, T, H_kv, D):
    g = torch.Generator().manual_seed(T * 131 + H_kv)
    nb, bs = 64, 16
    slots = torch.randperm(nb * bs, generator=g)[:T].to(torch.int64)
    kc = torch.randn((nb, bs, H_kv, D), generator=g).to(dtype)
    vc = torch.randn((nb, bs, H_kv, D), generator=g).to(dtype)
    k = torch.randn((T, H_kv, D), generator=g).to(dtype)
    v = torch.randn((T, H_kv, D), generator=g).to(dtype)
    view = torch.int16 if dtype != torch.float32 else torch.int32
    ek, ev = kc.view(view).numpy().copy(), vc.view(view).numpy().copy()
    ostore.store_kv(k.view(view).numpy(), v.view(view).numpy(), ek, ev, slots.numpy())
    gk, gv = kc.to(cuda), vc.to(cuda)
    ops.store_kvcache(k.to(cuda), v.to(cuda), gk, gv, slots.to(cuda))
    assert np.array_equal(gk.cpu().view(view).numpy(), ek)
    assert np.array_equal(gv.cpu().view(view).numpy(), ev)


def test_store_strided_key_view(cuda):
    """key/value as views of a fused qkv projection output (token stride > H_kv*D)."""
    T, H, H_kv, D = 33, 32, 8, 128
    qkv = torch.randn((T, (H + 2 * H_kv) * D), device=cuda).bfloat16()
    k = qkv[:, H * D:(H + H_kv) * D].view(T, H_kv, D)
    v = qkv[:, (H + H_kv) * D:].view(T, H_kv, D)
    kc = torch.zeros((8, 16, H_kv, D), device=cuda, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slots = torch.randperm(128, device=cuda)[:T]
    ops.store_kvcache(k, v, kc, vc, slots)
    assert torch.equal(kc.view(-1, H_kv, D)[slots], k)
    assert torch.equal(vc.view(-1, H_kv, D)[slots], v)


def test_store_padding_and_out_of_range_slots(cuda):
    H_kv, D = 8, 128
    kc = torch.zeros((4, 16, H_kv, D), device=cuda, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    k = torch.ones((3, H_kv, D), device=cuda, dtype=torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    slots = torch.tensor([-1, 5, 64], device=cuda)  # padding, valid, past the pool
    ops.store_kvcache(k, k, kc, vc, slots, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 1  # LK_STATUS_SLOT_OOB for slot 64 only
    assert kc.view(-1, H_kv, D)[5].eq(1).all()
    assert kc.view(-1, H_kv, D).sum().item() == H_kv * D


def test_store_config2_full_size_roundtrip(cuda):
    """Config 2 size (B=256 tokens into a >1 GB pool): write, read back the slots."""
    b = workloads.make_decode_batch(2, 256, seed=3, device=cuda)
    ops.store_kvcache(b.key, b.value, b.key_cache, b.value_cache, b.slot_mapping)
    H_kv, D = b.key.shape[1:]
    assert torch.equal(b.key_cache.view(-1, H_kv, D)[b.slot_mapping], b.key)
    assert torch.equal(b.value_cache.view(-1, H_kv, D)[b.slot_mapping], b.value)
