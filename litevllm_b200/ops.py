"""PyTorch-facing wrappers of the liblitekern C ABI.

Every function validates dtype / device / layout, then calls one C entry
point on the current CUDA stream of the tensors' device. Nothing here
computes on the host: a CPU tensor or a missing library raises.
"""

from __future__ import annotations

import contextlib
import ctypes
import math
from typing import Optional

import torch

from ._lib import LK_DTYPE_BF16, LK_DTYPE_F16, LK_DTYPE_F32, check, lib

_DTYPES = {torch.float32: LK_DTYPE_F32, torch.float16: LK_DTYPE_F16, torch.bfloat16: LK_DTYPE_BF16}


def _dtype_code(t: torch.Tensor, allowed=(torch.float16, torch.bfloat16)) -> int:
    if t.dtype not in allowed:
        raise TypeError(f"dtype {t.dtype} not supported here (allowed: {allowed})")
    return _DTYPES[t.dtype]


def _cuda(*ts: Optional[torch.Tensor]) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("litevllm_b200 kernels run on CUDA tensors only (no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} vs {t.device}")
    assert dev is not None
    return dev


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


_NULL = contextlib.nullcontext()


def _on(dev: torch.device):
    """Make dev current for the call (a no-op when it already is)."""
    return _NULL if dev.index == torch.cuda.current_device() else torch.cuda.device(dev)


class _Workspaces:
    """Zero-initialised scratch buffers, one per (device, purpose, stream).

    The kernels leave their counter regions zero after every call, so a
    buffer is reused across calls on one stream without re-clearing; calls on
    different streams may run at the same time, so each stream has its own.
    """

    def __init__(self) -> None:
        self._bufs: dict[tuple, torch.Tensor] = {}

    def get(self, dev: torch.device, name: str, nbytes: int) -> torch.Tensor:
        key = (dev.index, name)
        buf = self._bufs.get(key)
        if buf is None or buf.numel() < nbytes:
            size = max(nbytes, 1 << 16)
            if buf is not None:
                size = max(size, buf.numel() * 2)
            buf = torch.zeros(size, dtype=torch.uint8, device=dev)
            self._bufs[key] = buf
        return buf


WORKSPACES = _Workspaces()


# --------------------------------------------------------------- KV store ---
def store_kvcache(
    key: torch.Tensor,
    value: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
    status: Optional[torch.Tensor] = None,
) -> None:
    """key_cache[slot // bs, slot % bs] = key[t] (and value), for every t.

    key/value: [T, H_kv, D]; caches [num_blocks, bs, H_kv, D] contiguous;
    slot_mapping int64 [T]. Mirrors litevllm/layers/attention.py:79-84.
    """
    dev = _cuda(key, value, key_cache, value_cache, slot_mapping, status)
    if key.dim() != 3 or value.shape != key.shape:
        raise ValueError("key/value must be [T, H_kv, D] with equal shapes")
    T, H_kv, D = key.shape
    if key_cache.dim() != 4 or key_cache.shape[2:] != (H_kv, D) or value_cache.shape != key_cache.shape:
        raise ValueError("caches must be [num_blocks, block_size, H_kv, D]")
    if not (key_cache.is_contiguous() and value_cache.is_contiguous()):
        raise ValueError("caches must be contiguous")
    for t in (key, value):
        if t.stride(2) != 1 or t.stride(1) != D:
            raise ValueError("key/value must have unit d-stride and head stride D")
    if key.dtype != key_cache.dtype or value.dtype != key_cache.dtype:
        raise TypeError("key/value dtype must match the cache dtype")
    if slot_mapping.dtype != torch.int64 or slot_mapping.numel() != T:
        raise TypeError("slot_mapping must be int64 [T]")
    slot_mapping = slot_mapping.contiguous()
    code = _dtype_code(key_cache, (torch.float32, torch.float16, torch.bfloat16))
    num_slots = key_cache.shape[0] * key_cache.shape[1]
    with _on(dev):
        check(
            lib().lk_store_kv(
                key.data_ptr(), value.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(),
                slot_mapping.data_ptr(), T, H_kv, D, key.stride(0), value.stride(0), num_slots,
                code, _ptr(status), _stream(dev),
            )
        )


# ----------------------------------------------------------- paged decode ---
def decode_num_splits(B: int, H_kv: int, max_blocks: int, block_size: int) -> int:
    return int(lib().lk_paged_decode_num_splits(B, H_kv, max_blocks, block_size))


def decode_workspace_bytes(B: int, H: int, H_kv: int, D: int, num_splits: int) -> int:
    return int(lib().lk_paged_decode_workspace_bytes(B, H, H_kv, D, num_splits))


def paged_decode(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    block_tables: torch.Tensor,
    context_lens: torch.Tensor,
    scale: float,
    num_splits: int = 0,
    out: Optional[torch.Tensor] = None,
    workspace: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Single-token paged attention; mirrors Attention._decode_fast
    (litevllm/layers/attention.py:91-139). query [B, H, D] -> [B, H, D]."""
    dev = _cuda(query, key_cache, value_cache, block_tables, context_lens, out, workspace)
    if query.dim() != 3:
        raise ValueError("query must be [B, H, D]")
    B, H, D = query.shape
    nb, bs, H_kv, Dk = key_cache.shape
    if Dk != D or value_cache.shape != key_cache.shape:
        raise ValueError("cache shape mismatch")
    if not (key_cache.is_contiguous() and value_cache.is_contiguous()):
        raise ValueError("caches must be contiguous")
    if query.dtype != key_cache.dtype:
        raise TypeError("query dtype must match the cache dtype")
    if query.stride(2) != 1 or query.stride(1) != D:
        raise ValueError("query must have unit d-stride and head stride D")
    if block_tables.dtype != torch.int32 or block_tables.dim() != 2 or block_tables.shape[0] != B:
        raise TypeError("block_tables must be int32 [B, max_blocks]")
    if block_tables.stride(1) != 1:
        block_tables = block_tables.contiguous()
    if context_lens.dtype != torch.int32 or context_lens.numel() != B:
        raise TypeError("context_lens must be int32 [B]")
    context_lens = context_lens.contiguous()
    code = _dtype_code(query, (torch.float32, torch.float16, torch.bfloat16))
    if out is None:
        out = torch.empty((B, H, D), dtype=query.dtype, device=dev)
    elif out.shape != (B, H, D) or out.dtype != query.dtype or out.stride(2) != 1 or out.stride(1) != D:
        raise ValueError("bad out tensor")
    if B == 0:
        return out
    max_blocks = block_tables.shape[1]
    plan_key = (B, H, H_kv, D, bs, max_blocks, query.dtype, int(num_splits))
    plan = _DECODE_PLANS.get(plan_key)
    if plan is None:
        num_splits = int(num_splits)
        if num_splits == 0:  # auto split count; -1 selects the persistent kernel
            num_splits = decode_num_splits(B, H_kv, max_blocks, bs)
        need = decode_workspace_bytes(B, H, H_kv, D, num_splits)
        want = need
        if not _decode_takes_split_kernel(query.dtype, D, bs, H // H_kv):
            # room for the generic kernel's split-KV partials (less only means fewer splits)
            want = max(need, int(lib().lk_paged_attention_generic_workspace_bytes(
                B, H, D, max_blocks, bs)))
        plan = _DECODE_PLANS[plan_key] = (num_splits, need, want)
    num_splits, need, want = plan
    stream = _stream(dev)
    if workspace is None:
        workspace = WORKSPACES.get(dev, f"decode:{stream}", want)
    elif workspace.numel() * workspace.element_size() < need:
        raise ValueError(f"workspace too small: need {need} bytes")
    with _on(dev):
        check(
            lib().lk_paged_decode(
                out.data_ptr(), out.stride(0), query.data_ptr(), query.stride(0),
                key_cache.data_ptr(), value_cache.data_ptr(), nb, block_tables.data_ptr(),
                block_tables.stride(0), context_lens.data_ptr(), B, H, H_kv, D, bs, max_blocks,
                float(scale), num_splits, workspace.data_ptr(),
                workspace.numel() * workspace.element_size(), code, stream,
            )
        )
    return out


# (B, H, H_kv, D, block_size, max_blocks, dtype, num_splits argument) ->
# (split count, workspace bytes the kernel needs, bytes to allocate): the
# library's answers for a shape, asked once per shape instead of per call.
_DECODE_PLANS: dict = {}


def paged_decode_shared_prefix(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    block_tables: torch.Tensor,
    context_lens: torch.Tensor,
    scale: float,
    prefix_tokens: int,
    out: Optional[torch.Tensor] = None,
    workspace: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """paged_decode for a batch whose rows share their first prefix_tokens
    tokens (the same physical blocks at the start of every block-table row):
    the shared part runs once, on the tensor cores, for all rows. Same result
    as paged_decode (Attention._decode_fast, litevllm/layers/attention.py:91-139)."""
    dev = _cuda(query, key_cache, value_cache, block_tables, context_lens, out, workspace)
    if query.dim() != 3:
        raise ValueError("query must be [B, H, D]")
    B, H, D = query.shape
    nb, bs, H_kv, Dk = key_cache.shape
    if Dk != D or value_cache.shape != key_cache.shape:
        raise ValueError("cache shape mismatch")
    if not (key_cache.is_contiguous() and value_cache.is_contiguous()):
        raise ValueError("caches must be contiguous")
    if query.dtype != key_cache.dtype:
        raise TypeError("query dtype must match the cache dtype")
    if query.stride(2) != 1 or query.stride(1) != D:
        raise ValueError("query must have unit d-stride and head stride D")
    if block_tables.dtype != torch.int32 or block_tables.dim() != 2 or block_tables.shape[0] != B:
        raise TypeError("block_tables must be int32 [B, max_blocks]")
    block_tables = block_tables.contiguous()
    if context_lens.dtype != torch.int32 or context_lens.numel() != B:
        raise TypeError("context_lens must be int32 [B]")
    context_lens = context_lens.contiguous()
    code = _dtype_code(query)
    if out is None:
        out = torch.empty((B, H, D), dtype=query.dtype, device=dev)
    if B == 0:
        return out
    max_blocks = block_tables.shape[1]
    need = int(lib().lk_paged_decode_shared_prefix_workspace_bytes(B, H, H_kv, D, max_blocks, bs,
                                                                    int(prefix_tokens)))
    if need == 0:
        raise ValueError("invalid shared-prefix decode shape")
    if workspace is None:
        workspace = WORKSPACES.get(dev, f"decode:{_stream(dev)}", need)
    elif workspace.numel() * workspace.element_size() < need:
        raise ValueError(f"workspace too small: need {need} bytes")
    with _on(dev):
        check(
            lib().lk_paged_decode_shared_prefix(
                out.data_ptr(), out.stride(0), query.data_ptr(), query.stride(0),
                key_cache.data_ptr(), value_cache.data_ptr(), nb, block_tables.data_ptr(),
                block_tables.stride(0), context_lens.data_ptr(), B, H, H_kv, D, bs, max_blocks,
                float(scale), int(prefix_tokens), workspace.data_ptr(),
                workspace.numel() * workspace.element_size(), code, _stream(dev),
            )
        )
    return out


def decode_status(workspace: Optional[torch.Tensor] = None, device=None) -> int:
    """Read (and clear) the LK_STATUS_* bits the decode kernels left in their
    workspace (by default the current stream's). Synchronises the current stream."""
    if workspace is None:
        dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        workspace = WORKSPACES.get(dev, f"decode:{_stream(dev)}", 256)
    v = int(workspace[:4].view(torch.int32).item())
    workspace[:4].zero_()
    return v


# --------------------------------------------------------- paged prefill ---
def paged_prefill(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    cu_seqlens_q: torch.Tensor,
    max_q_len: int,
    scale: float,
    block_tables: Optional[torch.Tensor] = None,
    context_lens: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
    status: Optional[torch.Tensor] = None,
    workspace: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Causal attention for prefill chunks over prior paged context.

    query [T, H, D] packed by cu_seqlens_q (int32 [S+1]). Paged mode
    (block_tables given): caches [num_blocks, bs, H_kv, D], context_lens =
    prior + chunk length per sequence. Contiguous mode (block_tables None):
    key_cache/value_cache are the chunk's own [T, H_kv, D] keys/values and
    every sequence starts at position 0 (Attention._prefill,
    litevllm/layers/attention.py:141-151).
    """
    dev = _cuda(query, key_cache, value_cache, cu_seqlens_q, block_tables, context_lens, out, status, workspace)
    if query.dim() != 3:
        raise ValueError("query must be [T, H, D]")
    T, H, D = query.shape
    if query.stride(2) != 1 or query.stride(1) != D:
        raise ValueError("query must have unit d-stride and head stride D")
    if block_tables is not None:
        nb, bs, H_kv, Dk = key_cache.shape
        if not (key_cache.is_contiguous() and value_cache.is_contiguous()):
            raise ValueError("caches must be contiguous")
        if block_tables.dtype != torch.int32 or block_tables.stride(1) != 1:
            raise TypeError("block_tables must be int32 with unit column stride")
        if context_lens is None or context_lens.dtype != torch.int32:
            raise TypeError("context_lens must be int32 in paged mode")
        context_lens = context_lens.contiguous()
        bt_stride = block_tables.stride(0)
        num = nb
    else:
        if key_cache.dim() != 3:
            raise ValueError("contiguous mode wants key/value [T, H_kv, D]")
        key_cache = key_cache.contiguous()
        value_cache = value_cache.contiguous()
        Tk, H_kv, Dk = key_cache.shape
        bs, bt_stride, num = 16, 0, Tk
        context_lens = None
    if Dk != D or value_cache.shape != key_cache.shape:
        raise ValueError("key/value shape mismatch")
    if query.dtype != key_cache.dtype:
        raise TypeError("query dtype must match the cache dtype")
    if cu_seqlens_q.dtype != torch.int32:
        raise TypeError("cu_seqlens_q must be int32")
    cu_seqlens_q = cu_seqlens_q.contiguous()
    S = cu_seqlens_q.numel() - 1
    code = _dtype_code(query, (torch.float32, torch.float16, torch.bfloat16))
    if out is None:
        out = torch.empty((T, H, D), dtype=query.dtype, device=dev)
    elif out.shape != (T, H, D) or not out.is_contiguous():
        raise ValueError("bad out tensor")
    if S <= 0 or T == 0:
        return out
    need = int(lib().lk_paged_prefill_workspace_bytes())
    if workspace is None:
        # one per stream: the plan and the split partials belong to one launch at a time
        workspace = WORKSPACES.get(dev, f"prefill:{_stream(dev)}", need)
    elif workspace.numel() * workspace.element_size() < need:
        raise ValueError(f"workspace too small: need {need} bytes")
    with _on(dev):
        check(
            lib().lk_paged_prefill_ws(
                out.data_ptr(), query.data_ptr(), query.stride(0), key_cache.data_ptr(),
                value_cache.data_ptr(), num, _ptr(block_tables), bt_stride,
                cu_seqlens_q.data_ptr(), _ptr(context_lens), S, int(max_q_len), H, H_kv, D, bs,
                float(scale), code, workspace.data_ptr(),
                workspace.numel() * workspace.element_size(), _ptr(status), _stream(dev),
            )
        )
    return out


def _decode_takes_split_kernel(dtype: torch.dtype, head_dim: int, block_size: int, G: int) -> bool:
    """lk_paged_decode's own routing: 16-bit caches, head_dim 128, block sizes
    that are multiples of 16 and G <= 8 run the split kernel (G need not be a
    power of two there); everything else the generic kernel, whose split-KV
    partials want a larger workspace."""
    return (dtype in (torch.float16, torch.bfloat16) and head_dim == 128
            and block_size % 16 == 0 and G <= 8)


def tuned_attention_shape(dtype: torch.dtype, head_dim: int, block_size: int, G: int) -> bool:
    """True when the tuned prefill and shared-prefix kernels take this shape
    (their tensor-core tiles hold 128 / G positions, so G is 1, 2, 4 or 8);
    other shapes run the generic CUDA-core kernel (fp32 caches, head dims
    other than 128, block sizes not a multiple of 16, other G). The decode
    split kernel takes every G <= 8 (_decode_takes_split_kernel)."""
    return (dtype in (torch.float16, torch.bfloat16) and head_dim == 128
            and block_size % 16 == 0 and G in (1, 2, 4, 8))


def paged_attention_generic(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    scale: float,
    block_tables: Optional[torch.Tensor] = None,
    context_lens: Optional[torch.Tensor] = None,
    cu_seqlens_q: Optional[torch.Tensor] = None,
    max_q_len: Optional[int] = None,
    status: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """The generic CUDA-core kernel called directly (lk_paged_attention_generic).

    cu_seqlens_q None: decode, one query per row at position
    context_lens[b] - 1 (Attention._decode_fast). Otherwise prefill chunks as in
    paged_prefill: paged when block_tables is given, else key_cache /
    value_cache are the chunk's own [T, H_kv, D] keys / values.
    """
    dev = _cuda(query, key_cache, value_cache, block_tables, context_lens, cu_seqlens_q, status)
    T, H, D = query.shape
    if query.stride(2) != 1 or query.stride(1) != D:
        raise ValueError("query must have unit d-stride and head stride D")
    if query.dtype != key_cache.dtype or value_cache.shape != key_cache.shape:
        raise TypeError("query / cache dtype or shape mismatch")
    key_cache, value_cache = key_cache.contiguous(), value_cache.contiguous()
    if block_tables is not None:
        nb, bs, H_kv, _ = key_cache.shape
        if block_tables.dtype != torch.int32 or block_tables.stride(1) != 1:
            raise TypeError("block_tables must be int32 with unit column stride")
        bt_stride, max_blocks = block_tables.stride(0), block_tables.shape[1]
    else:
        nb, H_kv, _ = key_cache.shape
        bs, bt_stride, max_blocks = 16, 0, 0
    if context_lens is not None:
        context_lens = context_lens.contiguous()
    if cu_seqlens_q is None:
        S, mq = T, 1
    else:
        cu_seqlens_q = cu_seqlens_q.contiguous()
        S = cu_seqlens_q.numel() - 1
        # without max_q_len, the row count bounds every chunk (no device read)
        mq = int(max_q_len) if max_q_len is not None else T
    code = _dtype_code(query, (torch.float32, torch.float16, torch.bfloat16))
    out = torch.empty((T, H, D), dtype=query.dtype, device=dev)
    with _on(dev):
        check(
            lib().lk_paged_attention_generic(
                out.data_ptr(), out.stride(0), query.data_ptr(), query.stride(0),
                key_cache.data_ptr(), value_cache.data_ptr(), nb, _ptr(block_tables), bt_stride,
                _ptr(cu_seqlens_q), _ptr(context_lens), S, mq, H, H_kv, D, bs, max_blocks,
                float(scale), code, _ptr(status), _stream(dev),
            )
        )
    return out


# ---------------------------------------------------------------- sampler ---
def sample(
    logits: torch.Tensor,
    temperatures: Optional[torch.Tensor] = None,
    noise: Optional[torch.Tensor] = None,
    seed: int = 0,
    offset: int = 0,
    noise_dump: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
    workspace: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Greedy / Gumbel-max token ids, int64 [B].

    temperatures: fp32 [B] (0 = greedy row) or None (all greedy).
    noise: fp32 [B, >=V] Gumbel noise, or None for in-kernel Philox noise
    keyed by (seed, offset); noise_dump (fp32 [B, V]) receives that noise.
    """
    if logits.dim() == 1:
        logits = logits.unsqueeze(0)
    dev = _cuda(logits, temperatures, noise, noise_dump, out, workspace)
    B, V = logits.shape
    if logits.stride(1) != 1:
        logits = logits.contiguous()
    code = _dtype_code(logits, (torch.float32, torch.float16, torch.bfloat16))
    if temperatures is not None:
        if temperatures.dtype != torch.float32 or temperatures.numel() != B:
            raise TypeError("temperatures must be fp32 [B]")
        temperatures = temperatures.contiguous()
    noise_ld = 0
    if noise is not None:
        if noise.dtype != torch.float32 or noise.shape[0] != B or noise.shape[1] < V or noise.stride(1) != 1:
            raise TypeError("noise must be fp32 [B, >=V] with unit column stride")
        noise_ld = noise.stride(0)
    if noise_dump is not None:
        if noise_dump.dtype != torch.float32 or noise_dump.shape != (B, V) or not noise_dump.is_contiguous():
            raise TypeError("noise_dump must be contiguous fp32 [B, V]")
    if out is None:
        out = torch.empty(B, dtype=torch.int64, device=dev)
    if B == 0:
        return out
    need = _SAMPLE_WS.get((B, V))
    if need is None:
        need = _SAMPLE_WS[(B, V)] = int(lib().lk_sample_workspace_bytes(B, V))
    stream = _stream(dev)
    if workspace is None:
        workspace = WORKSPACES.get(dev, f"sample:{stream}", need)
    with _on(dev):
        check(
            lib().lk_sample(
                out.data_ptr(), logits.data_ptr(), B, V, logits.stride(0), _ptr(temperatures),
                _ptr(noise), noise_ld, seed & (2**64 - 1), offset & (2**64 - 1), _ptr(noise_dump),
                workspace.data_ptr(), workspace.numel() * workspace.element_size(), code, stream,
            )
        )
    return out


_SAMPLE_WS: dict = {}  # (B, V) -> lk_sample_workspace_bytes, asked once per shape


def sample_filtered(
    logits: torch.Tensor,
    temperatures: torch.Tensor,
    top_k: Optional[torch.Tensor] = None,
    top_p: Optional[torch.Tensor] = None,
    noise: Optional[torch.Tensor] = None,
    seed: int = 0,
    offset: int = 0,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Top-k / top-p filtered Gumbel-max sampling (fp32 / f16 / bf16 logits), int64 [B].
    Mirrors Sampler.sample's filtered branch (litevllm/layers/sampler.py:178-225)."""
    if logits.dim() == 1:
        logits = logits.unsqueeze(0)
    dev = _cuda(logits, temperatures, top_k, top_p, noise, out)
    B, V = logits.shape
    if logits.stride(1) != 1:
        logits = logits.contiguous()
    code = _dtype_code(logits, (torch.float32, torch.float16, torch.bfloat16))
    temperatures = temperatures.to(torch.float32).contiguous()
    if top_k is not None:
        top_k = top_k.to(torch.int32).contiguous()
    if top_p is not None:
        top_p = top_p.to(torch.float32).contiguous()
    noise_ld = 0
    if noise is not None:
        if noise.dtype != torch.float32 or noise.shape[0] != B or noise.shape[1] < V or noise.stride(1) != 1:
            raise TypeError("noise must be fp32 [B, >=V]")
        noise_ld = noise.stride(0)
    if out is None:
        out = torch.empty(B, dtype=torch.int64, device=dev)
    if B == 0:
        return out
    with _on(dev):
        check(
            lib().lk_sample_filtered(
                out.data_ptr(), logits.data_ptr(), B, V, logits.stride(0), temperatures.data_ptr(),
                _ptr(top_k), _ptr(top_p), _ptr(noise), noise_ld, seed & (2**64 - 1),
                offset & (2**64 - 1), code, _stream(dev),
            )
        )
    return out


def softmax_temp(logits: torch.Tensor, temperatures: torch.Tensor) -> torch.Tensor:
    """fp32 softmax(logits / T) per row (the top-k / top-p path)."""
    if logits.dim() == 1:
        logits = logits.unsqueeze(0)
    dev = _cuda(logits, temperatures)
    B, V = logits.shape
    logits = logits.contiguous()
    code = _dtype_code(logits, (torch.float32, torch.float16, torch.bfloat16))
    temperatures = temperatures.to(torch.float32).contiguous()
    probs = torch.empty((B, V), dtype=torch.float32, device=dev)
    with _on(dev):
        check(
            lib().lk_softmax_temp(
                probs.data_ptr(), V, logits.data_ptr(), B, V, V, temperatures.data_ptr(), code,
                _stream(dev),
            )
        )
    return probs


def repetition_penalty_(
    logits: torch.Tensor,
    past_token_ids: torch.Tensor,
    penalty,
    status: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """In place: each distinct id of past_token_ids[b] gets s / p if s > 0 else
    s * p on row b of logits, p = penalty (a float, or fp32 [B] per row; 1.0
    leaves the row alone). The reference's _apply_repetition_penalty
    (litevllm/layers/sampler.py:190-201) on a caller-owned tensor."""
    if logits.dim() == 1:
        logits = logits.unsqueeze(0)
    if past_token_ids.dim() == 1:
        past_token_ids = past_token_ids.unsqueeze(0)
    dev = _cuda(logits, past_token_ids, status)
    B, V = logits.shape
    if logits.stride(1) != 1:
        raise ValueError("logits must have unit column stride")
    code = _dtype_code(logits, (torch.float32, torch.float16, torch.bfloat16))
    past = past_token_ids.to(device=dev, dtype=torch.int64)
    if past.shape[0] != B:
        raise ValueError("past_token_ids must have one row per logits row")
    if past.shape[1] > 0 and past.stride(1) != 1:
        past = past.contiguous()
    if isinstance(penalty, torch.Tensor):
        pens = penalty.to(device=dev, dtype=torch.float32).contiguous()
        if pens.numel() != B:
            raise ValueError("per-row penalties must have B entries")
    else:
        pens = torch.full((B,), float(penalty), dtype=torch.float32, device=dev)
    with _on(dev):
        check(
            lib().lk_repetition_penalty(
                logits.data_ptr(), B, V, logits.stride(0), past.data_ptr(),
                past.stride(0) if past.shape[1] > 0 else 0, past.shape[1], pens.data_ptr(),
                _ptr(status), code, _stream(dev),
            )
        )
    return logits


# ------------------------------------------------ norm + RoPE + KV store ---
def rope_store_kvcache(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    key_cache: Optional[torch.Tensor],
    value_cache: Optional[torch.Tensor],
    slot_mapping: Optional[torch.Tensor],
    positions: torch.Tensor,
    cos_cached: torch.Tensor,
    sin_cached: torch.Tensor,
    q_norm_weight: Optional[torch.Tensor] = None,
    k_norm_weight: Optional[torch.Tensor] = None,
    eps: float = 1e-6,
    status: Optional[torch.Tensor] = None,
    key_out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """In one launch: optional q/k RMSNorm, RoPE on q (in place) and k, and the
    store of k / v into the paged cache. Mirrors Qwen3Attention.forward
    (litevllm/models/qwen3.py:76-92) up to the attention call; returns query.
    key_out ([T, H_kv, D], may be key itself) receives the rotated k."""
    dev = _cuda(query, key, value, key_cache, value_cache, slot_mapping, positions, cos_cached,
                sin_cached, q_norm_weight, k_norm_weight, status, key_out)
    if key_out is not None and (key_out.shape != key.shape or key_out.dtype != key.dtype
                                or key_out.stride(2) != 1 or key_out.stride(1) != key.shape[2]):
        raise ValueError("key_out must match key's shape and dtype, unit d-stride, head stride D")
    T, H, D = query.shape
    H_kv = key.shape[1]
    for t in (query, key, value):
        if t.stride(2) != 1 or t.stride(1) != D:
            raise ValueError("q/k/v must have unit d-stride and head stride D")
    code = _dtype_code(query)
    if key.dtype != query.dtype or value.dtype != query.dtype:
        raise TypeError("q, k, v must share a dtype")
    if cos_cached.dtype != torch.float32 or sin_cached.dtype != torch.float32:
        raise TypeError("cos / sin tables must be fp32 (RotaryEmbedding buffers)")
    cos_cached, sin_cached = cos_cached.contiguous(), sin_cached.contiguous()
    positions = positions.to(torch.int64).contiguous()
    for w in (q_norm_weight, k_norm_weight):
        if w is not None and (w.dtype != query.dtype or w.numel() != D):
            raise TypeError("norm weights must be [D] in the activation dtype")
    num_slots = 0
    if slot_mapping is not None:
        if key_cache is None or value_cache is None or not key_cache.is_contiguous():
            raise ValueError("a slot mapping needs contiguous caches")
        slot_mapping = slot_mapping.to(torch.int64).contiguous()
        num_slots = key_cache.shape[0] * key_cache.shape[1]
    with _on(dev):
        check(
            lib().lk_rope_store_kv(
                query.data_ptr(), query.stride(0), key.data_ptr(), key.stride(0), value.data_ptr(),
                value.stride(0), _ptr(key_out), 0 if key_out is None else key_out.stride(0),
                _ptr(key_cache), _ptr(value_cache), num_slots, _ptr(slot_mapping),
                positions.data_ptr(), cos_cached.data_ptr(), sin_cached.data_ptr(),
                cos_cached.shape[0], _ptr(q_norm_weight), _ptr(k_norm_weight), float(eps), T, H,
                H_kv, D, code, _ptr(status), _stream(dev),
            )
        )
    return query


# ------------------------------------------------------------- block copies ---
def _device_address(t: torch.Tensor) -> int:
    if t.is_cuda:
        return t.data_ptr()
    if not t.is_pinned():
        raise RuntimeError("host caches must be pinned (page-locked) for device-side swaps")
    out = ctypes.c_uint64(0)
    check(lib().lk_host_device_pointer(t.data_ptr(), ctypes.byref(out)))
    return out.value


def copy_blocks_between(src_caches, dst_caches, mapping, device=None,
                        status: Optional[torch.Tensor] = None) -> None:
    """dst[layer][d] = src[layer][s] for every (s, d) in mapping and every layer,
    K and V, in one launch. src_caches / dst_caches: lists of (key_cache,
    value_cache) per layer ([num_blocks, bs, H_kv, D], contiguous); CUDA tensors
    or pinned host tensors. mapping: dict {src: dst}, list of pairs or int64
    [n, 2] tensor. Mirrors KVCache.swap_in / swap_out and blocks_to_copy
    (litevllm/cache/kv_cache.py:74-102, engine/scheduler.py:25-27)."""
    if len(src_caches) != len(dst_caches) or not src_caches:
        raise ValueError("need the same, non-zero number of layers on both sides")
    k0 = src_caches[0][0]
    for kc, vc in list(src_caches) + list(dst_caches):
        if kc.shape[1:] != k0.shape[1:] or vc.shape != kc.shape or kc.dtype != k0.dtype:
            raise ValueError("all caches must share block shape and dtype")
        if not (kc.is_contiguous() and vc.is_contiguous()):
            raise ValueError("caches must be contiguous")
    if device is None:
        devs = [t.device for pair in list(src_caches) + list(dst_caches) for t in pair if t.is_cuda]
        if not devs:
            raise RuntimeError("at least one side must be on a CUDA device")
        device = devs[0]
    device = torch.device(device)
    if isinstance(mapping, dict):
        pairs = list(mapping.items())
    elif isinstance(mapping, torch.Tensor):
        pairs = None
    else:
        pairs = list(mapping)
    if pairs is not None:
        if not pairs:
            return
        mapping = torch.tensor(pairs, dtype=torch.int64)
    mapping = mapping.to(device=device, dtype=torch.int64).contiguous().view(-1, 2)
    n = mapping.shape[0]
    if n == 0:
        return
    src_ptrs = torch.tensor([_device_address(t) for pair in src_caches for t in pair],
                            dtype=torch.uint64).to(device)
    dst_ptrs = torch.tensor([_device_address(t) for pair in dst_caches for t in pair],
                            dtype=torch.uint64).to(device)
    block_bytes = k0[0].numel() * k0.element_size()
    with _on(device):
        check(
            lib().lk_copy_blocks(
                src_ptrs.data_ptr(), dst_ptrs.data_ptr(), len(src_caches), mapping.data_ptr(), n,
                block_bytes, src_caches[0][0].shape[0], dst_caches[0][0].shape[0],
                _ptr(status), _stream(device),
            )
        )
    # src_ptrs / dst_ptrs / mapping are freed in stream order on the launching
    # stream, after the kernel that reads them.


def copy_blocks(caches, mapping) -> None:
    """Copy-on-write block copies inside one set of device caches."""
    copy_blocks_between(caches, caches, mapping)


def swap_in(gpu_caches, cpu_caches, mapping) -> None:
    """KVCache.swap_in: gpu[layer][dst] = cpu[layer][src] (pinned host caches)."""
    copy_blocks_between(cpu_caches, gpu_caches, mapping)


def swap_out(gpu_caches, cpu_caches, mapping) -> None:
    """KVCache.swap_out: cpu[layer][dst] = gpu[layer][src]; synchronises the
    stream so the host copy is complete on return."""
    copy_blocks_between(gpu_caches, cpu_caches, mapping)
    dev = next(t.device for pair in gpu_caches for t in pair)
    torch.cuda.current_stream(dev).synchronize()


def default_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)
