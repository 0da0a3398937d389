"""Sampler on the GPU vs the reference (golden, its own test vectors) and the
oracle: greedy and noise-given ids bit-exact, in-kernel noise reproducible."""

import numpy as np
import pytest
import torch

from litevllm_b200 import ops, workloads
from litevllm_b200.sampler import Sampler
from oracle import sampler as osamp
from tests import golden_io

pytestmark = pytest.mark.gpu


class SP:
    """Minimal stand-in with the reference SamplingParams fields the sampler reads
    (litevllm/config/config.py:159-170)."""

    def __init__(self, temperature=1.0, top_p=1.0, top_k=-1, repetition_penalty=1.0, seed=None):
        self.temperature, self.top_p, self.top_k = temperature, top_p, top_k
        self.repetition_penalty, self.seed = repetition_penalty, seed


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_greedy_matches_reference_golden(cuda, dtype):
    d = golden_io.load("sampler.npz")
    x = torch.from_numpy(d["logits"]).to(dtype)
    got = ops.sample(x.to(cuda)).cpu().numpy()
    want = osamp.greedy(x.float().numpy())
    assert np.array_equal(got, want)
    if dtype == torch.float32:
        assert np.array_equal(got, d["greedy"])


def test_reference_test_sampler_vectors(cuda):
    """litevllm tests/test_sampler.py, through the drop-in Sampler on the GPU."""
    logits = torch.tensor([[1.0, 5.0, 3.0, 0.5], [4.0, 0.0, 2.0, 1.0]], device=cuda)
    assert Sampler.sample(logits, SP(temperature=0.0)).tolist() == [1, 0]
    torch.manual_seed(0)
    out = Sampler.sample(torch.randn(4, 32, device=cuda), SP(temperature=1.0))
    assert out.shape == (4,) and (out >= 0).all() and (out < 32).all()
    logits = torch.zeros(1, 8, device=cuda)
    logits[0, 3] = 100.0
    assert Sampler.sample(logits, SP(temperature=1.0, top_k=1)).tolist() == [3]
    logits = torch.tensor([[10.0, 9.5, -100.0, -100.0]], device=cuda)
    assert Sampler.sample(logits, SP(temperature=1.0, top_p=0.9)).tolist()[0] in (0, 1)


def test_softmax_temp_matches_reference_golden(cuda):
    d = golden_io.load("sampler.npz")
    x = torch.from_numpy(d["logits"][:2]).to(cuda)
    p = ops.softmax_temp(x, torch.full((2,), 0.7, device=cuda))
    torch.testing.assert_close(p.cpu(), torch.from_numpy(d["probs07"]), atol=1e-6, rtol=1e-4)


@pytest.mark.parametrize("B,V", [(1, 7), (3, 1000), (8, 151936), (64, 128256), (5, 151937)])
def test_greedy_ties_across_chunks(cuda, B, V):
    g = torch.Generator().manual_seed(B * 7 + V)
    x = torch.randn((B, V), generator=g).bfloat16()
    # plant exact ties in far-apart chunks; the lower index must win
    for b in range(B):
        i, j = sorted(torch.randint(0, V, (2,), generator=g).tolist())
        x[b, j] = 30.0
        x[b, i] = 30.0
    got = ops.sample(x.to(cuda)).cpu().numpy()
    assert np.array_equal(got, osamp.greedy(x.float().numpy()))


def test_greedy_unaligned_row_stride(cuda):
    x = torch.randn((6, 1001), device=cuda).bfloat16()
    view = x[:, :999]  # row stride 1001 elements: not 16-byte aligned
    got = ops.sample(view).cpu().numpy()
    assert np.array_equal(got, osamp.greedy(view.float().cpu().numpy()))


def test_greedy_nan_wins_like_torch_argmax(cuda):
    x = torch.randn((2, 5000), device=cuda)
    x[1, 4321] = float("nan")
    x[1, 4400] = float("nan")
    got = ops.sample(x).tolist()
    assert got[1] == 4321 == int(torch.argmax(x[1].cpu()))


@pytest.mark.parametrize("cfg", [1, 4, 5])
def test_gumbel_noise_given_bit_exact(cuda, cfg):
    B, V = (8, 151936) if cfg == 1 else (16, 151936)
    x = workloads.make_logits(cfg, B, V, seed=cfg, dtype=torch.bfloat16)
    t = workloads.temperatures_for(cfg, B)
    n = workloads.gumbel_noise(B, V, seed=cfg)
    got = ops.sample(x.to(cuda), t.to(cuda), noise=n.to(cuda)).cpu().numpy()
    want = osamp.gumbel(x.float().numpy(), t.numpy(), n.numpy())
    assert np.array_equal(got, want)


def test_in_kernel_noise_dump_and_philox(cuda):
    """In-kernel noise: the dumped noise reproduces the ids bit-exactly, its
    uniforms are the oracle's Philox4x32-10 stream, and the same (seed, offset)
    gives the same ids."""
    B, V = 4, 50000
    x = torch.randn((B, V)).bfloat16()
    t = torch.tensor([0.7, 1.0, 0.0, 1.3])
    dump = torch.zeros((B, V), device=cuda)
    seed, offset = 0x1234_5678_9ABC, 77
    ids = ops.sample(x.to(cuda), t.to(cuda), seed=seed, offset=offset, noise_dump=dump)
    dump_np = dump.cpu().numpy()
    assert np.array_equal(ids.cpu().numpy(), osamp.gumbel(x.float().numpy(), t.numpy(), dump_np))
    for b in (0, 1, 3):
        g = osamp.gumbel_from_u(osamp.philox_uniforms(b, V, seed, offset))
        np.testing.assert_allclose(dump_np[b], g, rtol=2e-6, atol=2e-6)
    again = ops.sample(x.to(cuda), t.to(cuda), seed=seed, offset=offset)
    assert torch.equal(ids, again)


def test_gumbel_in_kernel_distribution_chi_square(cuda):
    """Histogram of in-kernel Gumbel-max draws vs the reference's softmax(x / T)."""
    V, N, T = 32, 60_000, 0.7
    x = torch.randn(V, generator=torch.Generator().manual_seed(9)) * 2
    logits = x.repeat(N, 1).to(cuda)
    ids = ops.sample(logits, torch.full((N,), T, device=cuda), seed=2024, offset=1).cpu()
    counts = torch.bincount(ids, minlength=V).double()
    p = torch.softmax(x.double() / T, 0)
    exp = p * N
    keep = exp > 5
    chi2 = (((counts - exp) ** 2) / exp)[keep].sum().item()
    dof = int(keep.sum()) - 1
    # 99.9th percentile of chi-square is below dof + 4.5 sqrt(2 dof) for these dof
    assert chi2 < dof + 4.5 * (2 * dof) ** 0.5, (chi2, dof)


def test_sample_batch_mixed_rows(cuda):
    """One launch, per-row temperatures: greedy rows equal argmax."""
    x = workloads.make_logits(1, 8, 151936, seed=1, dtype=torch.float32).to(cuda)
    t = workloads.temperatures_for(1, 8).to(cuda)
    ids = Sampler.sample_batch(x, t, seed=5, offset=9).cpu().numpy()
    assert np.array_equal(ids[:4], osamp.greedy(x[:4].cpu().numpy()))
    assert ((ids >= 0) & (ids < 151936)).all()


def test_workspace_reused_across_batch_shapes(cuda):
    """Calls with different B / V share one workspace; each must find the
    counters zeroed whatever the previous call's layout was."""
    for B, V in [(8, 151936), (256, 128256), (3, 50000), (64, 151936), (256, 128256)]:
        x = torch.randn((B, V), device=cuda).bfloat16()
        got = ops.sample(x).cpu().numpy()
        assert np.array_equal(got, osamp.greedy(x.float().cpu().numpy())), (B, V)


@pytest.mark.parametrize("tag,pen", [("p13", 1.3), ("p08", 0.8)])
def test_repetition_penalty_matches_reference_golden(cuda, tag, pen):
    """Fused penalty vs the reference's _apply_repetition_penalty: bit-exact on
    fp32 and bf16 logits; Sampler.sample with past ids gives the reference's
    greedy ids."""
    d = golden_io.load("penalty.npz")
    past = torch.from_numpy(d["past"]).to(cuda)
    x = torch.from_numpy(d["logits"]).to(cuda)
    got = ops.repetition_penalty_(x.clone(), past, pen).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), d[f"{tag}_f32"].view(np.uint32))
    xb = golden_io.bf16(d["logits_bf16"]).to(cuda)
    gotb = ops.repetition_penalty_(xb.clone(), past, pen).cpu().view(torch.int16).numpy()
    assert np.array_equal(gotb.view(np.uint16), d[f"{tag}_bf16"])
    ids = Sampler.sample(x, SP(temperature=0.0, repetition_penalty=pen), past_token_ids=past)
    assert np.array_equal(ids.cpu().numpy(), d[f"{tag}_greedy"])
    assert torch.equal(x, torch.from_numpy(d["logits"]).to(cuda))  # caller's logits untouched


@pytest.mark.parametrize("dtype,tag", [(torch.float32, "f32"), (torch.bfloat16, "bf16"),
                                       (torch.float16, "f16")])
def test_repetition_penalty_per_row_and_large(cuda, dtype, tag):
    """Per-row penalties (1.0 leaves a row alone), long histories with many
    duplicates, a vocabulary of 151936, against the oracle."""
    g = torch.Generator().manual_seed(77)
    B, V, L = 6, 151936, 3000
    x = (torch.randn((B, V), generator=g) * 4).to(dtype)
    past = torch.randint(-V, V, (B, L), generator=g)
    past[:, ::7] = past[:, :1]  # many repeats of one id
    pens = torch.tensor([1.3, 1.0, 0.7, 2.0, 1.05, 1.0])
    got = ops.repetition_penalty_(x.to(cuda), past.to(cuda), pens.to(cuda)).float().cpu().numpy()
    want = x.float().numpy().copy()
    for b in range(B):
        if pens[b].item() != 1.0:
            row = osamp.repetition_penalty(x[b:b + 1].float().numpy(), past[b:b + 1].numpy(),
                                           pens[b].item(), "bf16" if tag == "bf16" else "f32")
            if tag == "f16":
                row = row.astype(np.float16).astype(np.float32)
            want[b] = row[0]
    assert np.array_equal(got, want)


def test_repetition_penalty_out_of_range_ids_flagged(cuda):
    x = torch.randn((2, 100), device=cuda)
    past = torch.tensor([[3, 100, 5], [-101, 7, 7]], device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    want = osamp.repetition_penalty(x.cpu().numpy(), [[3, 5], [7]], 1.5)
    got = ops.repetition_penalty_(x.clone(), past, 1.5, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & 16  # LK_STATUS_TOKEN_OOB
    assert np.array_equal(got.cpu().numpy(), want)


@pytest.mark.parametrize("variant", ["LITEKERN_SAMPLE_UNROLL=0", "LITEKERN_SAMPLE_UNROLL=4",
                                     "LITEKERN_SAMPLE_UNROLL=16", "LITEKERN_SAMPLE_CHUNKS=5", "LITEKERN_PDL=0"])
def test_sampler_kernel_options(variant):
    """The greedy kernels kept as options (chosen once per process from the
    environment) against the oracle, in a child process."""
    import os
    import subprocess
    import sys
    key, val = variant.split("=")
    env = dict(os.environ, **{key: val})
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-m", "tests.sampler_variant_check"], cwd=root, env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "ok" in r.stdout


def _all_16bit_values():
    """Every finite and non-finite bf16 and fp16 value, as fp32 (NaNs dropped)."""
    bits = torch.arange(65536, dtype=torch.int32).to(torch.int16)
    v = torch.cat([bits.view(torch.bfloat16).float(), bits.view(torch.float16).float()])
    return v[~torch.isnan(v)]


def test_sampler_division_is_ieee_for_every_16bit_value(cuda):
    """The in-kernel-noise kernel's x / T (Markstein's correction, IEEE division
    outside its range) equals IEEE fp32 division for every 16-bit logit and a
    spread of temperatures, including ones that force the fallback."""
    x = _all_16bit_values()
    gen = torch.Generator().manual_seed(3)
    temps = torch.cat([
        torch.tensor([0.7, 1.0, 1.3, 0.1, 2.0, 1e-3, 37.5, 3e-5, 1e5, 1e-30, 1e30, 0.5, 0.999999,
                      1.0000001, 2.0 ** -60, 2.0 ** 60, 2.0 ** -61, 2.0 ** 61]),
        torch.rand(96, generator=gen) * 2 + 0.01,
        torch.exp(torch.randn(32, generator=gen) * 6),
    ]).float()
    out = torch.empty((temps.numel(), x.numel()), device=cuda)
    from litevllm_b200 import _lib
    xd, td = x.to(cuda), temps.to(cuda)
    _lib.check(_lib.lib().lk_selftest_sampler_div(out.data_ptr(), xd.data_ptr(), x.numel(),
                                                   td.data_ptr(), temps.numel(), None))
    want = (x.numpy()[None, :] / temps.numpy()[:, None]).astype(np.float32)
    got = out.cpu().numpy()
    both_nan = np.isnan(got) & np.isnan(want)
    bad = (got.view(np.int32) != want.view(np.int32)) & ~both_nan
    assert not bad.any(), (np.argwhere(bad)[:5], got[bad][:5], want[bad][:5])


def test_gumbel_map_every_uniform(cuda):
    """The noise map over all 2^23 uniforms the kernel can draw (random low
    bits below them) is -ln(-ln u) to 1e-6 relative (2e-6 absolute)."""
    k = np.arange(2 ** 23, dtype=np.uint64)
    low = np.random.default_rng(1).integers(0, 512, size=k.size, dtype=np.uint64)
    bits = ((k << np.uint64(9)) | low).astype(np.uint32)
    out = torch.empty(bits.size, device=cuda)
    from litevllm_b200 import _lib
    bd = torch.from_numpy(bits.view(np.int32)).to(cuda)
    _lib.check(_lib.lib().lk_selftest_gumbel(out.data_ptr(), bd.data_ptr(), bits.size, None))
    u = (k.astype(np.float64) + 0.5) * 2.0 ** -23
    want = -np.log(-np.log(u))
    got = out.cpu().numpy().astype(np.float64)
    err = np.abs(got - want)
    assert (err <= 2e-6 + 1e-6 * np.abs(want)).all(), (err.max(), int(err.argmax()))
    # the oracle's fp32 map agrees within the noise-dump tolerance
    g32 = osamp.gumbel_from_u(osamp.uniform_bits_to_u(bits[:: 97]))
    np.testing.assert_allclose(out.cpu().numpy()[:: 97], g32, rtol=2e-6, atol=2e-6)


@pytest.mark.parametrize("B,V,dtype", [(128, 151936, torch.bfloat16), (64, 151936, torch.bfloat16),
                                       (5, 32003, torch.float16), (300, 4096, torch.bfloat16)])
def test_in_kernel_noise_configs_bit_exact_given_dump(cuda, B, V, dtype):
    """Config 4 / 5 shapes (and a ragged V, fp16, many rows) through the
    in-kernel-noise kernel: ids equal the oracle's given the dumped noise."""
    x = workloads.make_logits(4, B, V, seed=B, dtype=dtype, device=cuda)
    t = (torch.rand(B, generator=torch.Generator().manual_seed(B)) * 1.5 + 0.2).to(cuda)
    t[::7] = 0.0  # greedy rows inside a sampled batch
    dump = torch.zeros((B, V), device=cuda)
    ids = ops.sample(x, t, seed=99, offset=B, noise_dump=dump).cpu().numpy()
    want = osamp.gumbel(x.float().cpu().numpy(), t.cpu().numpy(), dump.cpu().numpy())
    assert np.array_equal(ids, want)


def test_in_kernel_noise_edge_values(cuda):
    """-inf masks, +inf, NaN, zeros, subnormals and extreme temperatures in the
    in-kernel-noise kernel: the same ids as the oracle given the dumped noise."""
    B, V = 12, 20000
    gen = torch.Generator().manual_seed(12)
    x = torch.randn((B, V), generator=gen)
    x[0, ::2] = float("-inf")                     # masked vocabulary
    x[1, :] = float("-inf")                       # fully masked row -> index 0
    x[2, 777] = float("inf")
    x[3, 1234] = float("nan")
    x[4, :] = 0.0
    x[5, ::3] = -0.0
    x[6, :100] = 1e-39                            # bf16 subnormals
    x[7, 5] = 3.0e38
    x = x.bfloat16()
    t = torch.tensor([0.7, 1.0, 0.9, 1.2, 1.0, 0.5, 1e-30, 0.25, 1e30, 3e-5, 1e5, 0.0])
    dump = torch.zeros((B, V), device=cuda)
    ids = ops.sample(x.to(cuda), t.to(cuda), seed=5, offset=6, noise_dump=dump).cpu().numpy()
    want = osamp.gumbel(x.float().numpy(), t.numpy(), dump.cpu().numpy())
    assert np.array_equal(ids, want), (ids, want)
    assert ids[1] == 0 and ids[2] == 777 and ids[3] == 1234


@pytest.mark.parametrize("B,V,T,spread", [(128, 151936, 0.7, 1.0), (64, 151936, 1.0, 1.0),
                                          (16, 32000, 0.05, 1.0), (8, 4096, 30.0, 1.0),
                                          (32, 151936, 0.7, 8.0), (8, 128256, 1.0, 20.0),
                                          (1, 151936, 0.7, 1.0), (3, 151936, 0.7, 1.0),
                                          (300, 4104, 0.7, 1.0)])
def test_in_kernel_noise_vector_skip_is_exact(cuda, B, V, T, spread):
    """Without a noise dump the kernel skips vectors whose key bound cannot beat
    the running best (wide logit spreads also skip the noise of most vectors);
    with a dump it computes every key. Same (seed, offset): the same ids, equal
    to the oracle's given the dumped noise — planted masks, ties and NaN
    included."""
    x = (workloads.make_logits(4, B, V, seed=B + V, device=cuda).float() * spread).to(torch.bfloat16)
    x[0, ::3] = float("-inf")
    if B > 1:
        x[1, 100] = x[1, V - 50] = x[1].max() + 2   # a tie in logits far apart
    if B > 2:
        x[2, V // 2] = float("nan")
    t = torch.full((B,), T, device=cuda)
    for offset in (1, 2):
        dump = torch.zeros((B, V), device=cuda)
        full = ops.sample(x, t, seed=77, offset=offset, noise_dump=dump)
        skip = ops.sample(x, t, seed=77, offset=offset)
        assert torch.equal(full, skip)
        want = osamp.gumbel(x.float().cpu().numpy(), t.cpu().numpy(), dump.cpu().numpy())
        assert np.array_equal(skip.cpu().numpy(), want)
        if B > 2:
            assert int(skip[2]) == V // 2
