"""The minimal ctypes binding of include/litekern.h that a maintainer would add
to litevllm to call liblitekern.so without the litevllm_b200 Python layer:
the KV store (replaces litevllm/layers/attention.py:79-84) and the paged
decode (replaces attention.py:91-139), bf16 caches. The library is opened
from LITEKERN_LIB, or by name through the loader's search path."""

import ctypes
import os
from ctypes import c_float, c_int32, c_int64, c_size_t, c_void_p

import torch

_lk = ctypes.CDLL(os.environ.get("LITEKERN_LIB", "liblitekern.so"))
_lk.lk_store_kv.argtypes = [c_void_p] * 5 + [c_int32] * 3 + [c_int64] * 3 + [c_int32, c_void_p, c_void_p]
_lk.lk_paged_decode.argtypes = [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_int64,
                                c_void_p, c_int64, c_void_p] + [c_int32] * 6 + [c_float, c_int32,
                                c_void_p, c_size_t, c_int32, c_void_p]
_lk.lk_paged_decode_workspace_bytes.restype = c_size_t
_lk.lk_status_string.restype = ctypes.c_char_p


def store_kvcache(key, value, k_cache, v_cache, slot_mapping):        # attention.py:79-84
    rc = _lk.lk_store_kv(key.data_ptr(), value.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                         slot_mapping.data_ptr(), key.shape[0], key.shape[1], key.shape[2],
                         key.stride(0), value.stride(0), k_cache.shape[0] * k_cache.shape[1],
                         2, None, torch.cuda.current_stream().cuda_stream)     # 2 = bf16
    assert rc == 0, _lk.lk_status_string(rc)


_ws = {}


def decode(q, k_cache, v_cache, block_table, context_lens, scale):    # attention.py:91-139
    B, H, D = q.shape
    nb, bs, Hkv, _ = k_cache.shape
    n = _lk.lk_paged_decode_num_splits(B, Hkv, block_table.shape[1], bs)
    need = _lk.lk_paged_decode_workspace_bytes(B, H, Hkv, D, n)
    ws = _ws.get(q.device)
    if ws is None or ws.numel() < need:
        ws = _ws[q.device] = torch.zeros(need, dtype=torch.uint8, device=q.device)  # zeroed once
    out = torch.empty_like(q)
    rc = _lk.lk_paged_decode(out.data_ptr(), out.stride(0), q.data_ptr(), q.stride(0),
                             k_cache.data_ptr(), v_cache.data_ptr(), nb, block_table.data_ptr(),
                             block_table.stride(0), context_lens.data_ptr(), B, H, Hkv, D, bs,
                             block_table.shape[1], scale, n, ws.data_ptr(), ws.numel(), 2,
                             torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lk.lk_status_string(rc)
    return out
