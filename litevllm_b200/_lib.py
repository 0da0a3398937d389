"""ctypes binding of liblitekern.so.

The library is the only compute path: if it is missing, `lib()` raises
instead of falling back to PyTorch or the CPU. Argument types mirror
include/litekern.h one for one.
"""

from __future__ import annotations

import ctypes
import threading
from ctypes import c_float, c_int32, c_int64, c_size_t, c_uint64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "liblitekern.so"

LK_OK = 0
LK_DTYPE_F32, LK_DTYPE_F16, LK_DTYPE_BF16 = 0, 1, 2
LK_STATUS_SLOT_OOB = 1
LK_STATUS_BLOCK_OOB = 2
LK_STATUS_WAIT_TIMEOUT = 4
LK_STATUS_CTX_OOB = 8
LK_STATUS_TOKEN_OOB = 16

# name -> (restype, argtypes)
SIGNATURES: dict[str, tuple] = {
    "lk_version": (c_int32, []),
    "lk_status_string": (ctypes.c_char_p, [c_int32]),
    "lk_store_kv": (
        c_int32,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32,
         c_int64, c_int64, c_int64, c_int32, c_void_p, c_void_p],
    ),
    "lk_paged_decode_num_splits": (c_int32, [c_int32, c_int32, c_int32, c_int32]),
    "lk_paged_decode_workspace_bytes": (c_size_t, [c_int32, c_int32, c_int32, c_int32, c_int32]),
    "lk_paged_decode": (
        c_int32,
        [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_void_p, c_int64,
         c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_float, c_int32,
         c_void_p, c_size_t, c_int32, c_void_p],
    ),
    "lk_paged_decode_status": (c_int32, [c_void_p, c_void_p]),
    "lk_paged_decode_shared_prefix_workspace_bytes": (
        c_size_t, [c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32]),
    "lk_paged_decode_shared_prefix": (
        c_int32,
        [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_void_p, c_int64,
         c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_float, c_int32,
         c_void_p, c_size_t, c_int32, c_void_p],
    ),
    "lk_paged_prefill": (
        c_int32,
        [c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_void_p, c_int64, c_void_p,
         c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_float, c_int32,
         c_void_p, c_void_p],
    ),
    "lk_paged_prefill_workspace_bytes": (c_size_t, []),
    "lk_paged_prefill_ws": (
        c_int32,
        [c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_void_p, c_int64, c_void_p,
         c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_float, c_int32,
         c_void_p, c_size_t, c_void_p, c_void_p],
    ),
    "lk_paged_attention_generic_workspace_bytes": (
        c_size_t, [c_int32, c_int32, c_int32, c_int32, c_int32]),
    "lk_paged_attention_generic": (
        c_int32,
        [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_void_p, c_int64,
         c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32,
         c_float, c_int32, c_void_p, c_void_p],
    ),
    "lk_sample_workspace_bytes": (c_size_t, [c_int32, c_int32]),
    "lk_sample": (
        c_int32,
        [c_void_p, c_void_p, c_int32, c_int32, c_int64, c_void_p, c_void_p, c_int64, c_uint64,
         c_uint64, c_void_p, c_void_p, c_size_t, c_int32, c_void_p],
    ),
    "lk_sample_noalloc": (
        c_int32,
        [c_void_p, c_void_p, c_int32, c_int32, c_int64, c_void_p, c_void_p, c_int64, c_uint64,
         c_uint64, c_void_p, c_int32, c_void_p],
    ),
    "lk_copy_blocks": (
        c_int32,
        [c_void_p, c_void_p, c_int32, c_void_p, c_int32, c_int64, c_int64, c_int64, c_void_p,
         c_void_p],
    ),
    "lk_host_device_pointer": (c_int32, [c_void_p, c_void_p]),
    "lk_selftest_wait_timeout": (c_int32, [c_void_p, c_uint64, c_void_p]),
    "lk_selftest_sampler_div": (c_int32, [c_void_p, c_void_p, c_int32, c_void_p, c_int32, c_void_p]),
    "lk_selftest_gumbel": (c_int32, [c_void_p, c_void_p, c_int32, c_void_p]),
    "lk_selftest_mma_rate": (c_int32, [c_int32, c_int32, c_void_p, c_void_p, c_void_p]),
    "lk_sample_filtered": (
        c_int32,
        [c_void_p, c_void_p, c_int32, c_int32, c_int64, c_void_p, c_void_p, c_void_p, c_void_p,
         c_int64, c_uint64, c_uint64, c_int32, c_void_p],
    ),
    "lk_rope_store_kv": (
        c_int32,
        [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p,
         c_void_p, c_int64,
         c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_float, c_int32,
         c_int32, c_int32, c_int32, c_int32, c_void_p, c_void_p],
    ),
    "lk_repetition_penalty": (
        c_int32,
        [c_void_p, c_int32, c_int32, c_int64, c_void_p, c_int64, c_int32, c_void_p, c_void_p,
         c_int32, c_void_p],
    ),
    "lk_softmax_temp": (
        c_int32,
        [c_void_p, c_int64, c_void_p, c_int32, c_int32, c_int64, c_void_p, c_int32, c_void_p],
    ),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class LiteKernError(RuntimeError):
    """A liblitekern entry point returned a non-zero status."""


def lib() -> ctypes.CDLL:
    """Load liblitekern.so once and attach the prototypes. Raises if absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise LiteKernError(
                    f"{LIB_PATH} is missing: build it with `python -m litevllm_b200.build`; "
                    "there is no fallback implementation"
                )
            handle = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(code: int) -> None:
    if code != LK_OK:
        msg = lib().lk_status_string(code).decode()
        raise LiteKernError(f"{msg} (code {code})")
