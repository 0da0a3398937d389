"""Load the reference-generated fixtures in tests/golden/ as torch tensors."""

from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


def bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


def load(name: str) -> dict:
    d = np.load(GOLDEN / name)
    return {k: d[k] for k in d.files}


def decode_case(name: str) -> dict:
    d = load(name)
    out = {k: d[k] for k in ("H", "H_kv", "D", "bs", "scale")}
    for k in ("key_cache", "value_cache", "query", "key", "value", "stored_k", "stored_v"):
        out[k] = bf16(d[k])
    out["block_tables"] = torch.from_numpy(d["block_tables"]).to(torch.int32)
    out["context_lens"] = torch.from_numpy(d["ctx"]).to(torch.int32)
    out["slot_mapping"] = torch.from_numpy(d["slot_mapping"]).to(torch.int64)
    out["out"] = torch.from_numpy(d["out"])
    out["untouched_equal"] = bool(d["untouched_equal"])
    return out
