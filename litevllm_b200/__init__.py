"""litevllm_b200 — sm_100a kernels for litevllm's per-step hot path.

    from litevllm_b200 import install
    install()          # patch an imported litevllm to use these kernels

Modules: ops (C-ABI wrappers), attention (drop-in Attention / PagedAttention),
sampler (drop-in Sampler), workloads (seeded synthetic inputs), sharding
(request sharding across GPUs), build (nvcc build of liblitekern.so).
"""

from __future__ import annotations

import importlib

__all__ = ["install"]

# (module, attribute) pairs of litevllm that name the replaced classes. Models
# import Attention from litevllm.layers at import time, so the name is
# replaced wherever it was bound.
_ATTENTION_SITES = ("litevllm.layers.attention", "litevllm.layers", "litevllm.models.qwen3",
                    "litevllm.models.llama")
_SAMPLER_SITES = ("litevllm.layers.sampler", "litevllm.layers", "litevllm.engine.llm_engine")


def install() -> list[str]:
    """Point litevllm's Attention, PagedAttention and Sampler at this package.

    Returns the patched "module.name" sites. Modules of litevllm that are not
    importable are skipped; the reference's call sites need no other change.
    """
    from .attention import Attention, PagedAttention
    from .sampler import Sampler

    patched = []
    for mod_name in _ATTENTION_SITES:
        try:
            mod = importlib.import_module(mod_name)
        except Exception:
            continue
        for name, obj in (("Attention", Attention), ("PagedAttention", PagedAttention)):
            if hasattr(mod, name):
                setattr(mod, name, obj)
                patched.append(f"{mod_name}.{name}")
    for mod_name in _SAMPLER_SITES:
        try:
            mod = importlib.import_module(mod_name)
        except Exception:
            continue
        if hasattr(mod, "Sampler"):
            setattr(mod, "Sampler", Sampler)
            patched.append(f"{mod_name}.Sampler")
    return patched
