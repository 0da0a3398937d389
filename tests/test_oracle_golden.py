"""Pin the CPU oracle to the reference: every restatement in oracle/ must
reproduce the outputs the reference's own functions produced
(tests/golden/, written by tests/golden/make_golden.py)."""

import numpy as np
import pytest
import torch

from oracle import paged_attention as pa
from oracle import sampler as osamp
from oracle import store_kv as ostore
from tests import golden_io


@pytest.mark.parametrize("name", ["store_decode.npz", "decode_g4.npz"])
def test_store_oracle_matches_reference(name):
    d = golden_io.decode_case(name)
    kc = d["key_cache"].view(torch.int16).numpy().copy()
    vc = d["value_cache"].view(torch.int16).numpy().copy()
    ostore.store_kv(d["key"].view(torch.int16).numpy(), d["value"].view(torch.int16).numpy(),
                    kc, vc, d["slot_mapping"].numpy())
    H_kv, D = int(d["H_kv"]), int(d["D"])
    slots = d["slot_mapping"].numpy()
    assert np.array_equal(kc.reshape(-1, H_kv, D)[slots], d["stored_k"].view(torch.int16).numpy())
    assert np.array_equal(vc.reshape(-1, H_kv, D)[slots], d["stored_v"].view(torch.int16).numpy())
    assert d["untouched_equal"]


@pytest.mark.parametrize("name", ["store_decode.npz", "decode_g4.npz"])
def test_decode_oracle_matches_reference(name):
    d = golden_io.decode_case(name)
    kc, vc = d["key_cache"].float().clone(), d["value_cache"].float().clone()
    bs = int(d["bs"])
    kc.view(-1, *kc.shape[2:])[d["slot_mapping"]] = d["key"].float()
    vc.view(-1, *vc.shape[2:])[d["slot_mapping"]] = d["value"].float()
    got = pa.decode(d["query"].float(), kc, vc, d["block_tables"], d["context_lens"], float(d["scale"]))
    torch.testing.assert_close(got, d["out"], atol=2e-5, rtol=1e-5)
    lit = pa.decode_batched_reference(d["query"].float(), kc, vc, d["block_tables"],
                                      d["context_lens"], float(d["scale"]))
    torch.testing.assert_close(lit, d["out"], atol=1e-6, rtol=1e-6)
    assert bs == 16


@pytest.mark.parametrize("tag", ["g2", "g4"])
def test_prefill_oracle_matches_reference(tag):
    d = golden_io.load("prefill.npz")
    q, k, v = (golden_io.bf16(d[f"{tag}_{x}"]).float() for x in "qkv")
    got = pa.prefill_contiguous(q, k, v)
    torch.testing.assert_close(got, torch.from_numpy(d[f"{tag}_out"]), atol=2e-5, rtol=1e-5)


def test_paged_prefill_oracle_reduces_to_contiguous():
    """With prior = 0 and the chunk stored in the cache, the paged restatement
    equals the reference's _prefill restatement."""
    d = golden_io.load("prefill.npz")
    q, k, v = (golden_io.bf16(d[f"g4_{x}"]).float() for x in "qkv")
    S, H, H_kv, D = (int(x) for x in d["g4_shape"])
    bs = 16
    nb = -(-S // bs) + 2
    perm = torch.randperm(nb, generator=torch.Generator().manual_seed(0))[: -(-S // bs)]
    kc = torch.zeros((nb, bs, H_kv, D))
    vc = torch.zeros((nb, bs, H_kv, D))
    slots = torch.tensor([int(perm[p // bs]) * bs + p % bs for p in range(S)])
    kc.view(-1, H_kv, D)[slots] = k
    vc.view(-1, H_kv, D)[slots] = v
    got = pa.prefill_one(q, kc, vc, perm.int(), 0, 1.0 / D**0.5)
    torch.testing.assert_close(got, torch.from_numpy(d["g4_out"]), atol=2e-5, rtol=1e-5)


def test_greedy_oracle_matches_reference():
    d = golden_io.load("sampler.npz")
    assert np.array_equal(osamp.greedy(d["logits"]), d["greedy"])
    assert d["greedy"][1] == 100 and d["greedy"][2] == 0 and d["greedy"][5] == 17
    # reference tests/test_sampler.py:11-17
    assert osamp.greedy(d["ref_vec"]).tolist() == [1, 0] == d["ref_vec_out"].tolist()


def test_gumbel_oracle_properties():
    d = golden_io.load("sampler.npz")
    x = d["logits"]
    t = np.array([0.0, 0.7, 0.0, 1.0, 0.0, 0.5], dtype=np.float32)
    g = np.zeros_like(x, dtype=np.float32)
    ids = osamp.gumbel(x, t, g)
    # zero noise: temperature does not move the argmax; greedy rows are greedy
    assert np.array_equal(ids, d["greedy"])
    # a dominant noise spike wins
    g[1, 7] = 1e6
    assert osamp.gumbel(x, t, g)[1] == 7
    # NaN key wins (torch.argmax semantics), first NaN index
    y = x.copy()
    y[0, 9] = np.nan
    y[0, 11] = np.nan
    assert osamp.greedy(y)[0] == 9


def test_gumbel_oracle_is_the_softmax_distribution():
    """argmax(x/T + Gumbel) is distributed as softmax(x/T) — the distribution the
    reference samples with torch.multinomial (sampler.py:178, :187)."""
    rng = np.random.default_rng(0)
    V, N, T = 8, 40000, 0.7
    x = rng.normal(size=V).astype(np.float32)
    u = rng.uniform(1e-7, 1 - 1e-7, size=(N, V))
    g = (-np.log(-np.log(u))).astype(np.float32)
    ids = osamp.gumbel(np.repeat(x[None], N, 0), np.full(N, T, np.float32), g)
    hist = np.bincount(ids, minlength=V) / N
    p = torch.softmax(torch.from_numpy(x) / T, 0).numpy()
    assert np.abs(hist - p).max() < 0.01


def test_philox_known_answers():
    """Philox4x32-10 known-answer vectors of the Random123 distribution."""
    out = osamp.philox4x32_10(np.zeros((1, 4), np.uint32), 0, 0)[0]
    assert [hex(int(v)) for v in out] == ["0x6627e8d5", "0xe169c58d", "0xbc57ac4c", "0x9b00dbd8"]
    out = osamp.philox4x32_10(np.full((1, 4), 0xFFFFFFFF, np.uint32), 0xFFFFFFFF, 0xFFFFFFFF)[0]
    assert [hex(int(v)) for v in out] == ["0x408f276d", "0x41c83b0e", "0xa20bc7c6", "0x6d5451fd"]
    ctr = np.array([[0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344]], np.uint32)
    out = osamp.philox4x32_10(ctr, 0xA4093822, 0x299F31D0)[0]
    assert [hex(int(v)) for v in out] == ["0xd16cfe09", "0x94fdcceb", "0x5001e420", "0x24126ea1"]


def test_uniform_mapping_open_interval():
    u = osamp.uniform_bits_to_u(np.array([0, 0xFFFFFFFF], np.uint32))
    assert 0.0 < u[0] < 1e-6 and 1 - 1e-6 < u[1] < 1.0
    g = osamp.gumbel_from_u(u)
    assert np.all(np.isfinite(g))


def test_rope_oracle_matches_reference():
    from oracle import rope as orope

    d = golden_io.load("rope.npz")
    q, k = golden_io.bf16(d["q"]), golden_io.bf16(d["k"])
    cos, sin = torch.from_numpy(d["cos"]), torch.from_numpy(d["sin"])
    qw, kw = golden_io.bf16(d["q_w"]), golden_io.bf16(d["k_w"])
    eps = float(d["eps"])
    assert torch.equal(orope.norm_rope(q, cos, sin, qw, eps), torch.from_numpy(d["q_out"]))
    assert torch.equal(orope.norm_rope(k, cos, sin, kw, eps), torch.from_numpy(d["k_out"]))


@pytest.mark.parametrize("tag,pen", [("p13", 1.3), ("p08", 0.8)])
def test_repetition_penalty_oracle_matches_reference(tag, pen):
    """The oracle's penalty is bit-exact with the reference's
    _apply_repetition_penalty on fp32 and bf16 logits (duplicates, negative
    ids, a zero score, the row max penalised)."""
    d = golden_io.load("penalty.npz")
    got = osamp.repetition_penalty(d["logits"], d["past"], pen, "f32")
    assert np.array_equal(got.view(np.uint32), d[f"{tag}_f32"].view(np.uint32))
    lb = (d["logits_bf16"].astype(np.uint32) << 16).view(np.float32)
    got = osamp.repetition_penalty(lb, d["past"], pen, "bf16")
    assert np.array_equal(got.view(np.uint32) >> 16, d[f"{tag}_bf16"].astype(np.uint32))
    assert np.array_equal(osamp.greedy(osamp.repetition_penalty(d["logits"], d["past"], pen)),
                          d[f"{tag}_greedy"])
