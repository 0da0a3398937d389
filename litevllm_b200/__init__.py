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


def install(engine_hooks: bool = False, merged_steps: bool = False,
            fused_rope: bool = False) -> list[str]:
    """Point litevllm's Attention, PagedAttention and Sampler at this package.

    Returns the patched "module.name" sites. Modules of litevllm that are not
    importable are skipped; the reference's call sites need no other change.
    With engine_hooks=True, ModelRunner.prepare_inputs and
    LLMEngine._process_outputs are also replaced by the vectorised / batched
    versions in litevllm_b200.engine_hooks (one sampler launch and one host
    sync per step instead of one per sequence); merged_steps=True (with
    engine_hooks) also replaces LLMEngine.step by one forward per step for
    the prefill chunks and the decodes together. fused_rope=True replaces
    Qwen3Attention.forward / LlamaAttention.forward by versions whose q/k
    RMSNorm, rotary embedding and KV store are one kernel
    (litevllm_b200.model_hooks).
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
    if engine_hooks:
        try:
            runner_mod = importlib.import_module("litevllm.engine.model_runner")
            engine_mod = importlib.import_module("litevllm.engine.llm_engine")
        except Exception:
            return patched
        from . import engine_hooks as hooks

        hooks.install(runner_mod.ModelRunner, engine_mod.LLMEngine, merged_steps=merged_steps)
        patched += ["litevllm.engine.model_runner.ModelRunner.prepare_inputs",
                    "litevllm.engine.llm_engine.LLMEngine._process_outputs"]
        if merged_steps:
            patched.append("litevllm.engine.llm_engine.LLMEngine.step")
    if fused_rope:
        from . import model_hooks

        patched += model_hooks.install()
    return patched
