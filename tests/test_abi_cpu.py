"""C-ABI checks that need no GPU: the library loads, exports every entry point
include/litekern.h declares, and rejects bad arguments before any launch."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

from litevllm_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "litekern.h"


def declared_symbols():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(lk_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    for s in ("lk_store_kv", "lk_paged_decode", "lk_paged_prefill", "lk_sample", "lk_softmax_temp"):
        assert s in syms


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    for s in declared_symbols():
        assert hasattr(lib, s), s
    assert set(declared_symbols()) <= set(_lib.SIGNATURES), "ctypes prototypes missing"


def test_status_strings():
    lib = _lib.lib()
    assert lib.lk_version() >= 100
    assert lib.lk_status_string(0) == b"ok"
    for code in (-1, -2, -3, -4, -5, -6, -99):
        assert lib.lk_status_string(code).startswith(b"litekern")


def test_argument_validation_without_launch():
    lib = _lib.lib()
    # zero tokens is a no-op
    assert lib.lk_store_kv(None, None, None, None, None, 0, 8, 128, 1024, 1024, 16, 2, None, None) == 0
    # bad dtype
    assert lib.lk_store_kv(1, 1, 1, 1, 1, 4, 8, 128, 1024, 1024, 16, 7, None, None) == -2
    # null pointers
    assert lib.lk_store_kv(None, 1, 1, 1, 1, 4, 8, 128, 1024, 1024, 16, 2, None, None) == -1
    # decode: H not a multiple of H_kv
    assert lib.lk_paged_decode(1, 0, 1, 0, 1, 1, 10, 1, 4, 1, 2, 12, 8, 128, 16, 4, 0.1, 1,
                               1, 1 << 20, 2, None) == -1
    # decode shapes the split kernel does not take (D = 64, G = 16, fp32, 8-slot
    # blocks) go to the generic kernel, which still wants the workspace
    P = 1 << 20  # 256-byte aligned stand-in pointer: these paths launch nothing
    for H, H_kv, D, bs, dt in ((16, 8, 64, 16, 2), (32, 2, 128, 16, 2), (16, 8, 128, 16, 0),
                               (16, 8, 128, 8, 2)):
        assert lib.lk_paged_decode(P, 0, P, 0, P, P, 10, P, 4, P, 2, H, H_kv, D, bs, 4, 0.1, 1,
                                   None, 0, dt, None) == -4
        assert lib.lk_paged_decode(P, 0, P, 0, P, P, 10, P, 4, P, 2, H, H_kv, D, bs, 4, 0.1, 1,
                                   1, 1 << 30, dt, None) == -4  # misaligned
    # decode: a head dim no kernel takes, and G above 32
    assert lib.lk_paged_decode(P, 0, P, 0, P, P, 10, P, 4, P, 2, 16, 8, 80, 16, 4, 0.1, 1,
                               P, 1 << 30, 2, None) == -2
    assert lib.lk_paged_decode(P, 0, P, 0, P, P, 10, P, 4, P, 2, 64, 1, 128, 16, 4, 0.1, 1,
                               P, 1 << 30, 2, None) == -2
    # decode: workspace missing
    assert lib.lk_paged_decode(16, 4096, 16, 4096, 256, 256, 10, 16, 4, 16, 2, 32, 8, 128, 16, 4,
                               0.1, 2, None, 0, 2, None) == -4
    # prefill: G = 3 goes to the generic kernel, which takes no D = 80
    assert lib.lk_paged_prefill(16, 16, 0, 16, 16, 10, None, 0, 16, None, 1, 8, 24, 8, 80, 16,
                                0.1, 2, None, None) == -2
    # generic kernel: bad dtype, decode form with several queries, decode form
    # without block tables, H not a multiple of H_kv, unaligned fp32 pointer
    g = lib.lk_paged_attention_generic
    gargs = [P, 2048, P, 2048, P, P, 10, P, 4, None, P, 2, 1, 16, 8, 128, 16, 4, 0.1, 0, None,
             None]
    bad = list(gargs); bad[19] = 7
    assert g(*bad) == -2
    bad = list(gargs); bad[12] = 3
    assert g(*bad) == -1
    bad = list(gargs); bad[7] = None
    assert g(*bad) == -1
    bad = list(gargs); bad[13] = 12
    assert g(*bad) == -1
    bad = list(gargs); bad[2] = P + 2
    assert g(*bad) == -3
    bad = list(gargs); bad[11] = 0                            # no sequences: nothing to do
    assert g(*bad) == 0
    # sampler: ld < V
    assert lib.lk_sample(1, 1, 2, 100, 50, None, None, 0, 0, 0, None, None, 0, 2, None) == -1
    # sampler: B = 0 no-op
    assert lib.lk_sample(None, None, 0, 100, 100, None, None, 0, 0, 0, None, None, 0, 2, None) == 0


def test_workspace_sizes_and_split_plan():
    lib = _lib.lib()
    # one split: status + counters + the launch-order list (8 bytes per unit)
    assert lib.lk_paged_decode_workspace_bytes(256, 32, 8, 128, 1) == 256 + 65536 * 4 + 256 * 8
    w4 = lib.lk_paged_decode_workspace_bytes(256, 32, 8, 128, 4)
    assert w4 >= 256 * 4 * 32 * (128 + 2) * 4
    # long contexts split; a single short sequence per SM-wave does not over-split
    assert lib.lk_paged_decode_num_splits(8, 8, 8192, 16) == 24
    assert lib.lk_paged_decode_workspace_bytes(8, 32, 8, 128, -1) > 256 + 65536 * 4
    assert lib.lk_paged_decode_num_splits(256, 8, 4, 16) == 1
    assert lib.lk_paged_decode_num_splits(256, 8, 256, 16) == 2
    assert lib.lk_sample_workspace_bytes(8, 151936) > 0


def test_ops_refuse_cpu_tensors():
    """No CPU fallback: host tensors are rejected loudly."""
    from litevllm_b200 import ops

    q = torch.zeros(2, 32, 128, dtype=torch.bfloat16)
    kc = torch.zeros(4, 16, 8, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.paged_decode(q, kc, kc, torch.zeros(2, 1, dtype=torch.int32),
                         torch.ones(2, dtype=torch.int32), 0.1)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.sample(torch.zeros(2, 10))
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.store_kvcache(torch.zeros(1, 8, 128, dtype=torch.bfloat16),
                          torch.zeros(1, 8, 128, dtype=torch.bfloat16), kc, kc,
                          torch.zeros(1, dtype=torch.int64))
    # shapes for the generic kernel (fp32, head_dim 64) are refused the same way
    q32 = torch.zeros(2, 32, 64)
    kc32 = torch.zeros(4, 16, 8, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.paged_decode(q32, kc32, kc32, torch.zeros(2, 1, dtype=torch.int32),
                         torch.ones(2, dtype=torch.int32), 0.1)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.paged_attention_generic(q32, kc32, kc32, 0.1,
                                    block_tables=torch.zeros(2, 1, dtype=torch.int32),
                                    context_lens=torch.ones(2, dtype=torch.int32))


def test_generic_shape_routing_and_workspace_sizes():
    from litevllm_b200 import ops

    assert ops.tuned_attention_shape(torch.bfloat16, 128, 16, 4)
    assert not ops.tuned_attention_shape(torch.float32, 128, 16, 4)
    assert not ops.tuned_attention_shape(torch.bfloat16, 64, 16, 4)
    assert not ops.tuned_attention_shape(torch.bfloat16, 128, 8, 4)
    assert not ops.tuned_attention_shape(torch.bfloat16, 128, 16, 3)
    # the decode workspace follows lk_paged_decode's routing: G = 3 takes the
    # split kernel there, so its default workspace is the split kernel's
    for G, split in ((1, True), (3, True), (7, True), (8, True), (16, False)):
        assert ops._decode_takes_split_kernel(torch.bfloat16, 128, 16, G) is split
    assert not ops._decode_takes_split_kernel(torch.float32, 128, 16, 4)
    assert not ops._decode_takes_split_kernel(torch.bfloat16, 64, 16, 4)
    assert not ops._decode_takes_split_kernel(torch.bfloat16, 128, 8, 4)
    f = _lib.lib().lk_paged_attention_generic_workspace_bytes
    head = 256 + 65536 * 4
    assert f(256, 32, 64, 32, 16) == 256          # 512 keys: one split, status word only
    # 4096 keys -> 8 splits of 512: head, then (max, sum) and output partials
    assert f(256, 32, 64, 256, 16) == head + 256 * 32 * 8 * 2 * 4 + 256 * 32 * 8 * 64 * 4
    assert f(1, 1, 64, 100000, 16) == head + 64 * 2 * 4 + 64 * 64 * 4   # capped at 64 splits
    assert f(0, 32, 64, 256, 16) == 256


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "absent.so")
    with pytest.raises(_lib.LiteKernError, match="no fallback"):
        _lib.lib()


def test_repetition_penalty_rejects_bad_arguments():
    lib = _lib.lib()
    # B = 0 or L = 0: nothing to do
    assert lib.lk_repetition_penalty(None, 0, 10, 10, None, 0, 0, None, None, 2, None) == 0
    assert lib.lk_repetition_penalty(1, 2, 10, 10, 1, 4, 0, 1, None, 2, None) == 0
    # row stride shorter than the row, history stride shorter than its length
    assert lib.lk_repetition_penalty(1, 2, 10, 9, 1, 4, 4, 1, None, 2, None) == -1
    assert lib.lk_repetition_penalty(1, 2, 10, 10, 1, 3, 4, 1, None, 2, None) == -1
    # missing pointers, unknown dtype
    assert lib.lk_repetition_penalty(None, 2, 10, 10, 1, 4, 4, 1, None, 2, None) == -1
    assert lib.lk_repetition_penalty(1, 2, 10, 10, 1, 4, 4, None, None, 2, None) == -1
    assert lib.lk_repetition_penalty(1, 2, 10, 10, 1, 4, 4, 1, None, 7, None) == -2


def test_integration_stub_binds_against_the_library(monkeypatch):
    """The ctypes stub include/litekern_ctypes.py (quoted in the integration
    notes) loads against the library as written (prototypes only; its
    functions need a GPU and are not called here)."""
    import importlib.util

    monkeypatch.setenv("LITEKERN_LIB", str(_lib.LIB_PATH))
    path = Path(__file__).resolve().parent.parent / "include" / "litekern_ctypes.py"
    spec = importlib.util.spec_from_file_location("litekern_ctypes", path)
    ns = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ns)
    assert callable(ns.store_kvcache) and callable(ns.decode)
    assert ns._lk.lk_status_string(0) == b"ok"
    assert ns._lk.lk_paged_decode_workspace_bytes(256, 32, 8, 128, 2) > 256 + 65536 * 4


def test_shared_prefix_decode_rejects_bad_arguments():
    lib = _lib.lib()
    ws = lib.lk_paged_decode_shared_prefix_workspace_bytes
    assert ws(128, 32, 8, 128, 144, 16, 2032) > 256 + 65536 * 4
    assert ws(128, 32, 8, 128, 144, 16, 0) == 0          # no prefix
    assert ws(128, 30, 8, 128, 144, 16, 2032) == 0       # H not a multiple of H_kv
    f = lib.lk_paged_decode_shared_prefix
    P = 1 << 20  # aligned stand-in pointers: nothing is launched on these paths
    args = [P, 4096, P, 4096, P, P, 1000, P, 144, P, 128, 32, 8, 128, 16, 144, 0.088, 2032, None,
            0, 2, None]
    assert f(*args) == -4                                    # no workspace
    bad = list(args); bad[17] = 2030                         # prefix not a multiple of bs
    assert f(*bad) == -1
    bad = list(args); bad[17] = 144 * 16 + 16                # prefix longer than the table
    assert f(*bad) == -1
    bad = list(args); bad[12] = 2                            # G = 16 unsupported
    assert f(*bad) == -2
    bad = list(args); bad[10] = 0                            # B = 0: nothing to do
    assert f(*bad) == 0
