"""Sampler oracles (numpy). Test infrastructure only.

greedy():  argmax over fp32 logits, first index wins ties — the reference's
           greedy branch (litevllm/layers/sampler.py:174-175 -> _argmax_kernel
           :60-84, strict '>' at :80; torch.argmax on CPU, :113). NaN counts as
           the maximum (torch.argmax semantics).
gumbel():  argmax(fp32(x) / T + g) with IEEE fp32 division and addition,
           first index on ties: the Gumbel-max form of the temperature branch
           (:178 softmax(x / T), :187 categorical draw) for a given noise g.
repetition_penalty(): _apply_repetition_penalty (sampler.py:190-201): each
           distinct past id (negative ids index from the row's end) of a row
           gets s / p if s > 0 else s * p, in fp32 (IEEE, p as fp32), rounded
           to the logits dtype ("f32", "bf16" round-to-nearest-even).
philox4x32_10(): Philox4x32-10 (Salmon et al., SC'11), the generator the
           sampler kernel uses for in-kernel noise; uniform_bits_to_u()
           restates its bits -> u mapping.
"""

from __future__ import annotations

import numpy as np


def _first_argmax(keys: np.ndarray) -> np.ndarray:
    """Row-wise argmax, NaN is the maximum, lowest index on ties."""
    keys = np.asarray(keys, dtype=np.float32)
    out = np.empty(keys.shape[0], dtype=np.int64)
    for b in range(keys.shape[0]):
        row = keys[b]
        nan = np.flatnonzero(np.isnan(row))
        out[b] = nan[0] if nan.size else int(np.argmax(row))  # np.argmax: first max
    return out


def greedy(logits) -> np.ndarray:
    return _first_argmax(np.asarray(logits, dtype=np.float32))


def gumbel(logits, temperatures, noise) -> np.ndarray:
    """Rows with T == 0 are greedy; others argmax(x / T + g) in fp32."""
    x = np.asarray(logits, dtype=np.float32)
    t = np.asarray(temperatures, dtype=np.float32)
    g = np.asarray(noise, dtype=np.float32)[:, : x.shape[1]]
    out = np.empty(x.shape[0], dtype=np.int64)
    with np.errstate(invalid="ignore", over="ignore"):
        for b in range(x.shape[0]):
            if not t[b] > 0:
                out[b] = _first_argmax(x[b : b + 1])[0]
            else:
                key = (x[b] / np.float32(t[b])).astype(np.float32) + g[b]
                out[b] = _first_argmax(key.astype(np.float32)[None])[0]
    return out


M0, M1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
W0, W1 = np.uint32(0x9E3779B9), np.uint32(0xBB67AE85)
MASK = np.uint64(0xFFFFFFFF)


def philox4x32_10(ctr: np.ndarray, k0: int, k1: int) -> np.ndarray:
    """ctr uint32 [N, 4] -> uint32 [N, 4]; 10 rounds, key bumped by the Weyl constants."""
    c = np.asarray(ctr, dtype=np.uint64).copy()
    k0 = np.uint64(k0 & 0xFFFFFFFF)
    k1 = np.uint64(k1 & 0xFFFFFFFF)
    for _ in range(10):
        p0 = M0 * c[:, 0]
        p1 = M1 * c[:, 2]
        hi0, lo0 = p0 >> np.uint64(32), p0 & MASK
        hi1, lo1 = p1 >> np.uint64(32), p1 & MASK
        c = np.stack([hi1 ^ c[:, 1] ^ k0, lo1, hi0 ^ c[:, 3] ^ k1, lo0], axis=1)
        k0 = (k0 + np.uint64(W0)) & MASK
        k1 = (k1 + np.uint64(W1)) & MASK
    return c.astype(np.uint32)


def uniform_bits_to_u(r: np.ndarray) -> np.ndarray:
    """u = ((r >> 9) + 0.5) * 2^-23 in fp32 (exact), u in (0, 1)."""
    return ((np.asarray(r, dtype=np.uint32) >> np.uint32(9)).astype(np.float32) + np.float32(0.5)) * np.float32(2.0**-23)


def philox_uniforms(b: int, V: int, seed: int, offset: int) -> np.ndarray:
    """The kernel's u[b, 0..V-1]: counter (v // 4, b, offset lo, offset hi), word v % 4."""
    n = (V + 3) // 4
    ctr = np.zeros((n, 4), dtype=np.uint32)
    ctr[:, 0] = np.arange(n, dtype=np.uint32)
    ctr[:, 1] = b
    ctr[:, 2] = offset & 0xFFFFFFFF
    ctr[:, 3] = (offset >> 32) & 0xFFFFFFFF
    r = philox4x32_10(ctr, seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF).reshape(-1)[:V]
    return uniform_bits_to_u(r)


def gumbel_from_u(u: np.ndarray) -> np.ndarray:
    u = np.asarray(u, dtype=np.float32)
    return (-np.log(-np.log(u))).astype(np.float32)


def filtered_kept(logits, temperature: float, top_k: int, top_p: float):
    """Tokens the reference keeps: softmax(x / T) in fp32, then the masking of
    _apply_top_k_top_p (litevllm/layers/sampler.py:204-225) before its
    renormalisation; returns (kept bool [V], probs fp32 [V]). Torch on CPU."""
    import torch

    x = torch.as_tensor(np.asarray(logits, dtype=np.float32))
    probs = torch.softmax(x / np.float32(temperature), dim=-1)
    p = probs.clone()
    if top_k > 0:
        k = min(top_k, p.size(-1))
        kth = torch.topk(p, k, dim=-1).values[..., -1, None]
        p = torch.where(p < kth, torch.zeros_like(p), p)
    if top_p < 1.0:
        sp, si = torch.sort(p, descending=True, dim=-1)
        cum = torch.cumsum(sp, dim=-1)
        sp = torch.where(cum - sp > top_p, torch.zeros_like(sp), sp)
        p = torch.zeros_like(p).scatter_(-1, si, sp)
    return (p > 0).numpy(), probs.numpy()


def filtered_gumbel(logits, temperature: float, top_k: int, top_p: float, noise) -> int:
    """argmax over kept tokens of fp32(x) / T + g (IEEE fp32), lowest index on ties."""
    kept, _ = filtered_kept(logits, temperature, top_k, top_p)
    x = np.asarray(logits, dtype=np.float32)
    key = (x / np.float32(temperature)).astype(np.float32) + np.asarray(noise, np.float32)
    key = np.where(kept, key.astype(np.float32), -np.inf)
    return int(np.argmax(key))


def round_bf16(x) -> np.ndarray:
    """fp32 -> nearest bf16 (ties to even), returned as fp32 values."""
    b = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def repetition_penalty(logits, past, penalty: float, dtype: str = "f32") -> np.ndarray:
    """Restates _apply_repetition_penalty (sampler.py:190-201) row by row."""
    out = np.array(logits, dtype=np.float32, copy=True)
    V = out.shape[1]
    p = np.float32(penalty)
    for i in range(out.shape[0]):
        ids = np.asarray(past[i], dtype=np.int64)
        ids = np.unique(np.where(ids < 0, ids + V, ids))
        s = out[i, ids]
        v = np.where(s > 0, s / p, s * p).astype(np.float32)
        out[i, ids] = round_bf16(v) if dtype == "bf16" else v
    return out
