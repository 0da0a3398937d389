"""Attention tolerance of the parity contract: bf16 outputs within 2e-2
max-abs and 1e-2 mean-relative of the fp32 reference."""

import torch

MAX_ABS = 2e-2
MEAN_REL = 1e-2


def assert_attn_close(got: torch.Tensor, ref: torch.Tensor, max_abs=MAX_ABS, mean_rel=MEAN_REL):
    got = got.detach().float().cpu()
    ref = ref.detach().float().cpu()
    assert got.shape == ref.shape, (got.shape, ref.shape)
    nan_g, nan_r = torch.isnan(got), torch.isnan(ref)
    assert torch.equal(nan_g, nan_r), "NaN pattern differs"
    got, ref = got[~nan_r], ref[~nan_r]
    if ref.numel() == 0:
        return
    diff = (got - ref).abs()
    ma = diff.max().item()
    mr = (diff.mean() / ref.abs().mean().clamp_min(1e-12)).item()
    assert ma <= max_abs, f"max-abs {ma:.3e} > {max_abs}"
    assert mr <= mean_rel, f"mean-rel {mr:.3e} > {mean_rel}"
