"""KV-store oracle (numpy). Test infrastructure only.

Restates litevllm/layers/attention.py:79-84 (Attention.forward) ==
PagedAttention.write_to_cache (:18-33):
    b_idx = slot // block_size; b_off = slot % block_size
    key_cache[b_idx, b_off] = key;  value_cache[b_idx, b_off] = value
"""

from __future__ import annotations

import numpy as np


def store_kv(key: np.ndarray, value: np.ndarray, key_cache: np.ndarray,
             value_cache: np.ndarray, slot_mapping: np.ndarray) -> None:
    """In place. key/value [T, H_kv, D]; caches [num_blocks, bs, H_kv, D]."""
    bs = key_cache.shape[1]
    slot = np.asarray(slot_mapping, dtype=np.int64)
    b_idx = slot // bs  # attention.py:81
    b_off = slot % bs   # attention.py:82
    key_cache[b_idx, b_off] = key      # attention.py:83
    value_cache[b_idx, b_off] = value  # attention.py:84
