"""Generate tests/golden/*.npz by running the REFERENCE implementation on CPU.

    python tests/golden/make_golden.py /path/to/lite-vllm-checkout

Imports litevllm from the given checkout (read only) and records, for small
seeded inputs, what its own functions return:

  store_decode.npz   Attention.forward(..., is_prefill=False)   (store + _decode_fast,
                     litevllm/layers/attention.py:77-139), config-1 head shapes
                     (16 Q / 8 KV heads, D=128, bs=16), context lengths 1, 15, 16,
                     17, 40, 100 (one block, block edges, partial last block).
  decode_g4.npz      same, 32 Q / 8 KV heads (Llama-3-8B GQA ratio 4).
  prefill.npz        Attention.forward(..., is_prefill=True)    (store + _prefill,
                     :141-151) for G=2 and G=4.
  rope.npz           LlamaRMSNorm (litevllm/models/llama.py:18-27) on q and k, then
                     RotaryEmbedding + apply_rotary_emb (layers/rotary_emb.py) at Qwen3
                     settings (theta 1e6), as Qwen3Attention.forward does (qwen3.py:76-84);
                     the cos / sin rows of the used positions are stored with it.
  sampler.npz        Sampler.sample greedy ids (litevllm/layers/sampler.py:151-175)
                     with planted ties, and the temperature softmax the reference
                     computes before its multinomial draw (:178 / :133-135).
  penalty.npz        _apply_repetition_penalty (sampler.py:190-201) on fp32 and bf16
                     logits for penalties 1.3 and 0.8, past ids with duplicates and
                     negative (wrapping) ids, and Sampler.sample's greedy ids after it
                     (:168-175). Written by penalty_fixture() (own generator).

Inputs are stored next to outputs (bf16 inputs as uint16 bit patterns), so
the fixtures do not depend on any random generator.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from litevllm.config import SamplingParams
    from litevllm.layers.attention import Attention
    from litevllm.layers.sampler import Sampler, _triton_softmax_temp

    torch.manual_seed(1234)
    g = torch.Generator().manual_seed(20260101)

    def decode_case(name, H, H_kv, ctx):
        D, bs = 128, 16
        B = len(ctx)
        nblk = [max(1, -(-c // bs)) for c in ctx]
        pool = sum(nblk) + 1
        perm = torch.randperm(pool, generator=g)
        mb = max(nblk)
        bt = torch.zeros((B, mb), dtype=torch.int32)
        off = 0
        for i, n in enumerate(nblk):
            bt[i, :n] = perm[off : off + n].int()
            off += n
        slots = torch.tensor([int(bt[i, (c - 1) // bs]) * bs + (c - 1) % bs for i, c in enumerate(ctx)])
        kc = torch.randn((pool, bs, H_kv, D), generator=g).bfloat16()
        vc = torch.randn((pool, bs, H_kv, D), generator=g).bfloat16()
        q = torch.randn((B, H, D), generator=g).bfloat16()
        k = torch.randn((B, H_kv, D), generator=g).bfloat16()
        v = torch.randn((B, H_kv, D), generator=g).bfloat16()
        kc32, vc32 = kc.float().clone(), vc.float().clone()
        attn = Attention(H, D, H_kv)
        out = attn.forward(q.float(), k.float(), v.float(), kc32, vc32, bt, slots,
                           torch.tensor(ctx, dtype=torch.int32), is_prefill=False)
        np.savez_compressed(
            HERE / name,
            H=H, H_kv=H_kv, D=D, bs=bs, scale=attn.scale,
            ctx=np.array(ctx, dtype=np.int32), block_tables=bt.numpy(), slot_mapping=slots.numpy(),
            key_cache=bf16_bits(kc), value_cache=bf16_bits(vc), query=bf16_bits(q),
            key=bf16_bits(k), value=bf16_bits(v),
            # the rows the store wrote, read back from the reference's cache
            stored_k=bf16_bits(kc32.view(-1, H_kv, D)[slots].bfloat16()),
            stored_v=bf16_bits(vc32.view(-1, H_kv, D)[slots].bfloat16()),
            untouched_equal=np.array(bool(
                torch.equal(kc32.view(-1, H_kv, D)[[i for i in range(pool * bs) if i not in set(slots.tolist())]],
                            kc.float().view(-1, H_kv, D)[[i for i in range(pool * bs) if i not in set(slots.tolist())]]))),
            out=out.float().numpy(),
        )

    decode_case("store_decode.npz", 16, 8, [1, 15, 16, 17, 40, 100])
    decode_case("decode_g4.npz", 32, 8, [3, 64, 129])

    # prefill: reference _prefill over the new tokens only
    pre = {}
    for tag, H, H_kv, S in (("g2", 16, 8, 37), ("g4", 32, 8, 33)):
        D = 128
        q = torch.randn((S, H, D), generator=g).bfloat16()
        k = torch.randn((S, H_kv, D), generator=g).bfloat16()
        v = torch.randn((S, H_kv, D), generator=g).bfloat16()
        attn = Attention(H, D, H_kv)
        out = attn.forward(q.float(), k.float(), v.float(), None, None, None, None, None,
                           is_prefill=True)
        pre.update({f"{tag}_q": bf16_bits(q), f"{tag}_k": bf16_bits(k), f"{tag}_v": bf16_bits(v),
                    f"{tag}_out": out.float().contiguous().numpy(), f"{tag}_shape": np.array([S, H, H_kv, D])})
    np.savez_compressed(HERE / "prefill.npz", **pre)

    # sampler: greedy with planted ties + the temperature softmax
    V = 4096
    logits = torch.randn((6, V), generator=g) * 2.0
    logits[1, 100] = logits[1, 3000] = 50.0          # tie: lowest index wins
    logits[2, :] = 1.0                               # all equal -> index 0
    logits[3, V - 1] = 60.0                          # max at the last index
    logits[4, 0] = 70.0                              # max at the first index
    logits[5, 17] = logits[5, 18] = logits[5, 4000] = 55.0
    greedy = Sampler.sample(logits, SamplingParams(temperature=0.0, max_tokens=8))
    probs07 = _triton_softmax_temp(logits[:2], 0.7)
    # the four vectors of the reference's own tests/test_sampler.py
    ref_vec = torch.tensor([[1.0, 5.0, 3.0, 0.5], [4.0, 0.0, 2.0, 1.0]])
    ref_vec_out = Sampler.sample(ref_vec, SamplingParams(temperature=0.0, max_tokens=8))
    np.savez_compressed(
        HERE / "sampler.npz",
        logits=logits.numpy(), greedy=greedy.numpy(), probs07=probs07.numpy(),
        ref_vec=ref_vec.numpy(), ref_vec_out=ref_vec_out.numpy(),
    )
    # q/k RMSNorm + RoPE, as in Qwen3Attention.forward
    from litevllm.layers.rotary_emb import RotaryEmbedding, apply_rotary_emb
    from litevllm.models.llama import LlamaRMSNorm

    T, H, H_kv, D = 9, 16, 8, 128
    rope = RotaryEmbedding(D, 40960, 1000000.0, None)
    positions = torch.randint(0, 40960, (T,), generator=g)
    qn, kn = LlamaRMSNorm(D), LlamaRMSNorm(D)
    with torch.no_grad():
        qn.weight.copy_(1 + 0.1 * torch.randn(D, generator=g))
        kn.weight.copy_(1 + 0.1 * torch.randn(D, generator=g))
    qn, kn = qn.bfloat16(), kn.bfloat16()
    q = torch.randn((T, H, D), generator=g).bfloat16()
    k = torch.randn((T, H_kv, D), generator=g).bfloat16()
    with torch.no_grad():
        cos, sin = rope(positions)
        q_ref = apply_rotary_emb(qn(q), cos.unsqueeze(1), sin.unsqueeze(1))
        k_ref = apply_rotary_emb(kn(k), cos.unsqueeze(1), sin.unsqueeze(1))
    np.savez_compressed(
        HERE / "rope.npz", q=bf16_bits(q), k=bf16_bits(k), positions=positions.numpy(),
        cos=cos.numpy(), sin=sin.numpy(), q_w=bf16_bits(qn.weight.detach()),
        k_w=bf16_bits(kn.weight.detach()), eps=np.float32(qn.eps),
        q_out=q_ref.float().numpy(), k_out=k_ref.float().numpy(),
        q_out_dtype=str(q_ref.dtype),
    )
    penalty_fixture(ref_root)
    attention_block_fixture(ref_root)
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


def attention_block_fixture(ref_root: str) -> None:
    """The reference's own Qwen3Attention (q/k RMSNorm) and LlamaAttention
    blocks in bf16 (Attention from the reference too): a 20-token prefill that
    stores its K/V into a paged cache, then one decode step over that cache.
    Weights, inputs, the bf16 cos / sin tables and both outputs are saved."""
    sys.path.insert(0, ref_root)
    from litevllm.models.llama import LlamaAttention
    from litevllm.models.qwen3 import Qwen3Attention

    g = torch.Generator().manual_seed(777)
    hidden, H, H_kv, D, bs, S = 256, 8, 2, 128, 16, 20
    out = {}
    for tag, cls, kw in (("qwen3", Qwen3Attention, dict(rope_theta=1000000.0, use_qk_norm=True)),
                         ("llama", LlamaAttention, dict(rope_theta=500000.0))):
        torch.manual_seed(5)
        m = cls(hidden, H, H_kv, D, max_position_embeddings=4096, **kw)
        with torch.no_grad():
            for name, prm in m.named_parameters():
                if name.endswith("norm.weight"):
                    prm.copy_(1 + 0.1 * torch.randn(prm.shape, generator=g))
                else:
                    prm.copy_(torch.randn(prm.shape, generator=g) * prm.shape[-1] ** -0.5)
        m = m.to(torch.bfloat16)
        kc = torch.zeros((8, bs, H_kv, D), dtype=torch.bfloat16)
        vc = torch.zeros_like(kc)
        blocks = [3, 5]
        x = torch.randn((S, hidden), generator=g).bfloat16()
        pos = torch.arange(S)
        slots = torch.tensor([blocks[p // bs] * bs + p % bs for p in range(S)])
        x2 = torch.randn((1, hidden), generator=g).bfloat16()
        with torch.no_grad():
            y = m(x, pos, (kc, vc), slots, None, None, True)
            y2 = m(x2, torch.tensor([S]), (kc, vc), torch.tensor([blocks[S // bs] * bs + S % bs]),
                   torch.tensor([blocks], dtype=torch.int32),
                   torch.tensor([S + 1], dtype=torch.int32), False)
        sd = {k: bf16_bits(v) for k, v in m.state_dict().items() if v.dtype == torch.bfloat16}
        out.update({f"{tag}.{k}": v for k, v in sd.items()})
        out.update({f"{tag}.x": bf16_bits(x), f"{tag}.x2": bf16_bits(x2),
                    f"{tag}.y": y.float().numpy(), f"{tag}.y2": y2.float().numpy(),
                    # the rows of the positions used (the test's tables stop there)
                    f"{tag}.cos": bf16_bits(m.rotary_emb.cos_cached[:64]),
                    f"{tag}.sin": bf16_bits(m.rotary_emb.sin_cached[:64]),
                    f"{tag}.k_cache": bf16_bits(kc), f"{tag}.v_cache": bf16_bits(vc),
                    f"{tag}.eps": np.float32(getattr(getattr(m, "q_norm", None), "eps", 1e-6))})
    out["shape"] = np.array([hidden, H, H_kv, D, bs, S])
    out["blocks"] = np.array([3, 5])
    np.savez_compressed(HERE / "attn_block.npz", **out)


def penalty_fixture(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from litevllm.config import SamplingParams
    from litevllm.layers.sampler import Sampler, _apply_repetition_penalty

    g = torch.Generator().manual_seed(20261201)
    B, V, L = 4, 1000, 12
    logits = torch.randn((B, V), generator=g) * 3.0
    past = torch.randint(0, V, (B, L), generator=g)
    past[0, 3] = past[0, 7] = past[0, 1]     # duplicates: penalised once
    past[1, 0] = -1                          # wraps to V - 1
    past[1, 5] = -V                          # wraps to 0
    past[2, :] = 42                          # one id only
    logits[2, 42] = 0.0                      # score 0: multiplied (not > 0)
    logits[3, past[3, 0]] = 80.0             # the row's max, penalised
    out = {"logits": logits.numpy(), "past": past.numpy(),
           "logits_bf16": bf16_bits(logits.bfloat16())}
    for tag, pen in (("p13", 1.3), ("p08", 0.8)):
        out[f"{tag}_f32"] = _apply_repetition_penalty(logits.clone(), past, pen).numpy()
        out[f"{tag}_bf16"] = bf16_bits(_apply_repetition_penalty(logits.bfloat16(), past, pen))
        out[f"{tag}_greedy"] = Sampler.sample(
            logits, SamplingParams(temperature=0.0, repetition_penalty=pen, max_tokens=8),
            past_token_ids=past).numpy()
    np.savez_compressed(HERE / "penalty.npz", **out)


if __name__ == "__main__":
    # the reference checkout: argument, LITEVLLM_REFERENCE, else a "reference"
    # directory beside this repository; "--only NAME" writes one fixture
    args = [a for a in sys.argv[1:] if not a.startswith("--only")]
    root = args[0] if args else (os.environ.get("LITEVLLM_REFERENCE")
                                 or str(HERE.parent.parent.parent / "reference"))
    only = [a.split("=", 1)[1] for a in sys.argv[1:] if a.startswith("--only=")]
    if only == ["attn_block"]:
        attention_block_fixture(root)
    else:
        main(root)
