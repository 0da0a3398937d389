"""Fused top-k / top-p sampling vs the reference's filter (oracle restatement of
_apply_top_k_top_p, litevllm/layers/sampler.py:204-225): bit-exact ids given the
noise, the reference's own test vectors, and the sampled distribution."""

import numpy as np
import pytest
import torch

from litevllm_b200 import ops
from litevllm_b200.sampler import Sampler
from oracle import sampler as osamp

pytestmark = pytest.mark.gpu


class SP:
    def __init__(self, temperature=1.0, top_p=1.0, top_k=-1, repetition_penalty=1.0, seed=None):
        self.temperature, self.top_p, self.top_k = temperature, top_p, top_k
        self.repetition_penalty, self.seed = repetition_penalty, seed


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("V", [1000, 8192, 151936])
def test_filtered_noise_given_matches_oracle(cuda, V, dtype):
    g = torch.Generator().manual_seed(V)
    B = 12
    x = (torch.randn((B, V), generator=g) * 2).to(dtype)
    temps = torch.tensor([0.7, 1.0, 1.3, 0.5] * 3)
    ks = torch.tensor([1, 5, 50, 0, 0, 0, 20, 1000, 3, 0, 7, 0], dtype=torch.int32)
    ps = torch.tensor([1.0, 1.0, 1.0, 0.9, 0.5, 0.1, 0.8, 0.95, 1.0, 0.999, 0.3, 1.0])
    noise = torch.from_numpy(-np.log(-np.log(np.random.default_rng(V).uniform(1e-7, 1 - 1e-7,
                                                                            (B, V))))).float()
    got = ops.sample_filtered(x.to(cuda), temps.to(cuda), ks.to(cuda), ps.to(cuda),
                              noise=noise.to(cuda)).cpu().tolist()
    xf = x.float().numpy()
    want = [osamp.filtered_gumbel(xf[b], float(temps[b]), int(ks[b]), float(ps[b]), noise[b].numpy())
            for b in range(B)]
    assert got == want


def test_reference_top_k_top_p_vectors(cuda):
    """litevllm tests/test_sampler.py:28-46, bf16 logits through Sampler.sample."""
    logits = torch.zeros(1, 8, device=cuda, dtype=torch.bfloat16)
    logits[0, 3] = 100.0
    for _ in range(5):
        assert Sampler.sample(logits, SP(temperature=1.0, top_k=1)).tolist() == [3]
    logits = torch.tensor([[10.0, 9.5, -100.0, -100.0]], device=cuda, dtype=torch.bfloat16)
    for _ in range(20):
        assert Sampler.sample(logits, SP(temperature=1.0, top_p=0.9)).tolist()[0] in (0, 1)


def test_reference_top_k_top_p_vectors_fp32(cuda):
    """The same vectors as the reference's tests use them, fp32 logits: the
    fused kernel, no torch sort / multinomial."""
    logits = torch.zeros(1, 8, device=cuda)
    logits[0, 3] = 100.0
    for _ in range(5):
        assert Sampler.sample(logits, SP(temperature=1.0, top_k=1)).tolist() == [3]
    logits = torch.tensor([[10.0, 9.5, -100.0, -100.0]], device=cuda)
    for _ in range(20):
        assert Sampler.sample(logits, SP(temperature=1.0, top_p=0.9)).tolist()[0] in (0, 1)


def test_fp32_top_k_keeps_probability_ties(cuda):
    """fp32 logits one ulp apart have the same probability after rounding;
    the reference keeps every token whose probability equals the k-th
    largest, so top_k=1 over such a pair must be able to draw either."""
    x = torch.full((1, 64), -30.0)
    x[0, 10] = 1e-3
    x[0, 20] = float(np.nextafter(np.float32(1e-3), np.float32(0.0)))
    kept, _ = osamp.filtered_kept(x[0].numpy(), 1.0, 1, 1.0)
    assert kept[10] and kept[20]  # the reference keeps both
    N = 4000
    ids = ops.sample_filtered(x.repeat(N, 1).to(cuda), torch.ones(N, device=cuda),
                              torch.ones(N, dtype=torch.int32, device=cuda), None,
                              seed=3, offset=1).cpu()
    assert set(ids.tolist()) == {10, 20}


@pytest.mark.parametrize("k,p", [(5, 1.0), (0, 0.7), (10, 0.6)])
def test_filtered_distribution_chi_square(cuda, k, p):
    V, N, T = 32, 60_000, 0.8
    x = (torch.randn(V, generator=torch.Generator().manual_seed(4)) * 2).bfloat16()
    kept, probs = osamp.filtered_kept(x.float().numpy(), T, k, p)
    target = np.where(kept, probs, 0.0)
    target = target / target.sum()
    logits = x.repeat(N, 1).to(cuda)
    ids = ops.sample_filtered(logits, torch.full((N,), T, device=cuda),
                              torch.full((N,), k, dtype=torch.int32, device=cuda),
                              torch.full((N,), p, device=cuda), seed=11, offset=2).cpu().numpy()
    assert kept[ids].all(), "a filtered-out token was drawn"
    counts = np.bincount(ids, minlength=V).astype(np.float64)
    exp = target * N
    m = exp > 5
    chi2 = (((counts - exp) ** 2) / np.where(m, exp, 1))[m].sum()
    dof = int(m.sum()) - 1
    assert chi2 < dof + 4.5 * (2 * max(dof, 1)) ** 0.5 + 5, (chi2, dof)


def test_greedy_rows_ignore_filters(cuda):
    x = torch.randn((4, 5000), device=cuda).bfloat16()
    ids = ops.sample_filtered(x, torch.zeros(4, device=cuda),
                              torch.full((4,), 3, dtype=torch.int32, device=cuda),
                              torch.full((4,), 0.2, device=cuda))
    assert torch.equal(ids.cpu(), x.float().cpu().argmax(-1))
