"""Replacements for the two engine methods either side of the hot path.

* ``prepare_inputs`` — same result as ``ModelRunner.prepare_inputs``
  (litevllm/engine/model_runner.py:180-260): input ids, positions, slot
  mapping (missing blocks map to slot 0), zero-padded int32 block tables and
  int32 context lengths for decode batches, ``None`` tables for prefill. The
  per-token Python loops become numpy arithmetic, and all int64 data reaches
  the device in one pinned host-to-device copy (one more for the int32 data)
  instead of one synchronous copy per tensor.
* ``process_outputs`` — same bookkeeping as ``LLMEngine._process_outputs``
  (litevllm/engine/llm_engine.py:172-199): each sequence gets the token
  sampled from its row (the last prompt row for a prefill), prompts are marked
  computed, stop rules run in sequence order. Rows without a repetition
  penalty are sampled in one ``Sampler.sample_batch`` launch with per-row
  temperature, top-k and top-p and read
  back with one ``.tolist()``; the other rows go through ``Sampler.sample``.

* ``prepare_inputs_mixed`` / ``merged_step`` — one forward per engine step
  instead of one for the decode groups plus one per prefill group
  (litevllm/engine/llm_engine.py:127-138): the step's prefill chunks come
  first in the batch (packed by ``cu_seqlens_q``), then one token per decode
  sequence; every sequence has its block table and context length, and the
  attention layers run the chunked-prefill kernel (over the prior paged
  context plus the chunk, causal inside it) next to the decode kernel.
  Prefill rows see their prior context, which the reference's ``_prefill``
  (block tables None) does not: the two agree for chunks that start at
  position 0, the reference's own case.

``install(runner_cls, engine_cls, merged_steps=False)`` binds them onto the
reference classes.
"""

from __future__ import annotations

import sys

import numpy as np
import torch

from .attention import set_mixed_step_hint, set_shared_prefix_hint
from .sampler import Sampler


def _fast_params(params, logits_dtype) -> bool:
    return getattr(params, "repetition_penalty", 1.0) == 1.0


def shared_prefix_tokens(tables, ctx_lens, bs: int) -> int:
    """Tokens at the start of every row that live in the same physical blocks,
    whole blocks that every row has filled."""
    if len(tables) < 2:
        return 0
    n = min(min(t.shape[0] for t in tables), min(int(c) // bs for c in ctx_lens))
    first = tables[0]
    for t in tables[1:]:
        if n == 0:
            break
        diff = np.nonzero(t[:n] != first[:n])[0]
        if diff.size:
            n = int(diff[0])
    return n * bs


def prepare_inputs(self, seq_groups, block_manager):
    """Vectorised ModelRunner.prepare_inputs; returns the runner module's InputMetadata."""
    InputMetadata = sys.modules[type(self).__module__].InputMetadata
    bs = self.config.cache_config.block_size
    ids_parts, pos_parts, slot_parts = [], [], []
    tables, ctx_lens, seq_ids = [], [], []
    is_prefill = False
    for sg in seq_groups:
        for seq in sg.get_unfinished_seqs():
            seq_ids.append(seq.seq_id)
            blocks = np.asarray(block_manager.get_block_table(seq.seq_id).physical_block_ids,
                                dtype=np.int64)
            if seq.is_prefill:
                is_prefill = True
                start, end = seq.num_computed_tokens, seq.data.prompt_len
                toks = np.asarray(seq.data.prompt_token_ids[start:end], dtype=np.int64)
                pos = np.arange(start, end, dtype=np.int64)
            else:
                toks = np.asarray(seq.data.all_token_ids[-1:], dtype=np.int64)
                pos = np.asarray([seq.data.total_len - 1], dtype=np.int64)
                ctx_lens.append(seq.data.total_len)
                tables.append(blocks)
            bidx = pos // bs
            have = bidx < blocks.shape[0]
            slot = np.zeros_like(pos)
            if have.any():
                slot[have] = blocks[bidx[have]] * bs + pos[have] % bs
            ids_parts.append(toks)
            pos_parts.append(pos)
            slot_parts.append(slot)
    n = sum(p.shape[0] for p in pos_parts)
    cat = lambda parts: np.concatenate(parts) if parts else np.zeros(0, dtype=np.int64)
    packed = np.concatenate([cat(ids_parts), cat(pos_parts), cat(slot_parts)])
    device = torch.device(self.device)
    host = torch.from_numpy(packed)
    if device.type == "cuda":
        host = host.pin_memory()
    dev64 = host.to(device, non_blocking=True)
    input_ids, positions, slot_mapping = dev64[:n], dev64[n:2 * n], dev64[2 * n:]
    if is_prefill:
        block_tables = context_lens = None
        set_shared_prefix_hint(None, 0)
    else:
        max_blocks = max((t.shape[0] for t in tables), default=0)
        tab = np.zeros((len(tables), max_blocks), dtype=np.int32)
        for i, t in enumerate(tables):
            tab[i, :t.shape[0]] = t
        tab = np.concatenate([tab.reshape(-1), np.asarray(ctx_lens, dtype=np.int32)])
        h32 = torch.from_numpy(tab)
        if device.type == "cuda":
            h32 = h32.pin_memory()
        d32 = h32.to(device, non_blocking=True)
        nb = len(tables) * max_blocks
        block_tables = d32[:nb].view(len(tables), max_blocks)
        context_lens = d32[nb:]
        # Leading blocks every decode row shares (the PrefixCache hands the same
        # physical blocks to sequences with a common prefix), counted only while
        # every row has filled them: the shared-prefix decode computes that part
        # once for the batch.
        set_shared_prefix_hint(block_tables, shared_prefix_tokens(tables, ctx_lens, bs))
    return InputMetadata(input_ids=input_ids, positions=positions, slot_mapping=slot_mapping,
                         block_tables=block_tables, context_lens=context_lens,
                         is_prefill=is_prefill, seq_ids=seq_ids)


def _to_device(arr: np.ndarray, device: torch.device) -> torch.Tensor:
    host = torch.from_numpy(arr)
    if device.type == "cuda":
        host = host.pin_memory()
    return host.to(device, non_blocking=True)


def prepare_inputs_mixed(self, prefill_groups, decode_groups, block_manager):
    """InputMetadata of one merged step: the prefill chunks of prefill_groups
    (in order), then one token per sequence of decode_groups. Token data are
    what ModelRunner.prepare_inputs builds for each group
    (model_runner.py:180-260); block_tables / context_lens cover every
    sequence (a prefill row's context is its prior tokens plus its chunk).
    The step's layout is handed to the attention layers through
    set_mixed_step_hint; is_prefill is True when the step has a chunk."""
    if not prefill_groups:
        set_mixed_step_hint(None)
        return prepare_inputs(self, decode_groups, block_manager)
    InputMetadata = sys.modules[type(self).__module__].InputMetadata
    bs = self.config.cache_config.block_size
    ids_parts, pos_parts, slot_parts = [], [], []
    tables, ctx_lens, seq_ids, q_lens = [], [], [], []
    for phase, groups in ((True, prefill_groups), (False, decode_groups)):
        for sg in groups:
            for seq in sg.get_unfinished_seqs():
                blocks = np.asarray(block_manager.get_block_table(seq.seq_id).physical_block_ids,
                                    dtype=np.int64)
                if seq.is_prefill != phase:
                    raise ValueError("prefill_groups / decode_groups hold the other kind")
                if phase:
                    start, end = seq.num_computed_tokens, seq.data.prompt_len
                    toks = np.asarray(seq.data.prompt_token_ids[start:end], dtype=np.int64)
                    pos = np.arange(start, end, dtype=np.int64)
                    ctx_lens.append(end)
                    q_lens.append(end - start)
                else:
                    toks = np.asarray(seq.data.all_token_ids[-1:], dtype=np.int64)
                    pos = np.asarray([seq.data.total_len - 1], dtype=np.int64)
                    ctx_lens.append(seq.data.total_len)
                seq_ids.append(seq.seq_id)
                tables.append(blocks)
                bidx = pos // bs
                have = bidx < blocks.shape[0]
                slot = np.zeros_like(pos)
                if have.any():
                    slot[have] = blocks[bidx[have]] * bs + pos[have] % bs
                ids_parts.append(toks)
                pos_parts.append(pos)
                slot_parts.append(slot)
    n = sum(p.shape[0] for p in pos_parts)
    device = torch.device(self.device)
    dev64 = _to_device(np.concatenate([np.concatenate(ids_parts), np.concatenate(pos_parts),
                                       np.concatenate(slot_parts)]), device)
    input_ids, positions, slot_mapping = dev64[:n], dev64[n:2 * n], dev64[2 * n:]
    P = len(q_lens)
    cu = np.zeros(P + 1, dtype=np.int32)
    cu[1:] = np.cumsum(q_lens)
    max_blocks = max(t.shape[0] for t in tables)
    tab = np.zeros((len(tables), max_blocks), dtype=np.int32)
    for i, t in enumerate(tables):
        tab[i, :t.shape[0]] = t
    d32 = _to_device(np.concatenate([tab.reshape(-1), np.asarray(ctx_lens, dtype=np.int32), cu]),
                     device)
    nb = len(tables) * max_blocks
    block_tables = d32[:nb].view(len(tables), max_blocks)
    context_lens = d32[nb:nb + len(tables)]
    cu_seqlens_q = d32[nb + len(tables):]
    set_shared_prefix_hint(None, 0)
    set_mixed_step_hint(block_tables, cu_seqlens_q, P, int(cu[-1]), max(q_lens))
    return InputMetadata(input_ids=input_ids, positions=positions, slot_mapping=slot_mapping,
                         block_tables=block_tables, context_lens=context_lens,
                         is_prefill=True, seq_ids=seq_ids)


def merged_step(self):
    """LLMEngine.step with one forward for all scheduled groups (prefill
    chunks, then decodes) instead of llm_engine.py:127-138's one forward for
    the decode groups plus one per prefill group; scheduling, outputs and
    bookkeeping as in the reference step (:111-151)."""
    sched_output = self.scheduler.schedule()
    if sched_output.is_empty:
        return []
    groups = sched_output.scheduled_seq_groups
    prefill = [sg for sg in groups if any(s.is_prefill for s in sg.get_unfinished_seqs())]
    decode = [sg for sg in groups if not any(s.is_prefill for s in sg.get_unfinished_seqs())]
    metadata = prepare_inputs_mixed(self.model_runner, prefill, decode, self.block_manager)
    logits = self.model_runner.execute_model(metadata)
    set_mixed_step_hint(None)
    self._process_outputs(logits, prefill + decode)
    results = [self._build_step_output(sg) for sg in groups]
    self.scheduler.update_running(groups)
    self.scheduler.free_finished()
    return results


def process_outputs(self, logits, seq_groups) -> None:
    """Batched LLMEngine._process_outputs (one sampler launch for plain rows)."""
    entries = []
    idx = 0
    for sg in seq_groups:
        for seq in sg.get_unfinished_seqs():
            if seq.is_prefill:
                n = seq.data.prompt_len - seq.num_computed_tokens
                seq.num_computed_tokens = seq.data.prompt_len
                row = idx + n - 1
                idx += n
            else:
                row = idx
                idx += 1
            entries.append((sg, seq, row))
    if logits.dim() == 1:
        logits = logits.unsqueeze(0)
    tokens = [None] * len(entries)
    fast = [i for i, (sg, _, _) in enumerate(entries)
            if _fast_params(sg.sampling_params, logits.dtype)]
    if fast:
        dev = logits.device
        params = [entries[i][0].sampling_params for i in fast]
        rows = torch.tensor([entries[i][2] for i in fast], dtype=torch.int64, device=dev)
        temps = torch.tensor([float(sp.temperature) for sp in params], dtype=torch.float32,
                             device=dev)
        top_k = top_p = None
        if any(sp.top_k > 0 or sp.top_p < 1.0 for sp in params):
            top_k = torch.tensor([int(sp.top_k) for sp in params], dtype=torch.int32, device=dev)
            top_p = torch.tensor([float(sp.top_p) for sp in params], dtype=torch.float32,
                                 device=dev)
        row_ids = [entries[i][2] for i in fast]
        if row_ids == list(range(logits.shape[0])):
            sel = logits  # every row sampled, in order: no gather
        else:
            sel = logits.index_select(0, rows)
        picked = Sampler.sample_batch(sel, temps, top_k=top_k, top_p=top_p).tolist()
        for i, t in zip(fast, picked):
            tokens[i] = int(t)
    for i, (sg, seq, row) in enumerate(entries):
        if tokens[i] is None:
            tokens[i] = int(self.sampler.sample(logits[row:row + 1], sg.sampling_params).item())
    for (sg, seq, _), tok in zip(entries, tokens):
        seq.data.append_token(tok)
        self._should_stop(seq, sg.sampling_params, tok)


def install(runner_cls, engine_cls, merged_steps: bool = False) -> None:
    """Bind the batched methods onto the reference ModelRunner / LLMEngine;
    with merged_steps also LLMEngine.step (one forward per step)."""
    runner_cls.prepare_inputs = prepare_inputs
    engine_cls._process_outputs = process_outputs
    if merged_steps:
        engine_cls.step = merged_step
