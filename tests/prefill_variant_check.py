"""Child-process check used by test_gpu_prefill.test_prefill_kernel_options:
runs ragged paged prefill cases with whichever kernel the environment selects
and compares them with the fp32 oracle."""

import torch

from litevllm_b200 import ops, workloads
from oracle import paged_attention as pa
from tests.tolerance import assert_attn_close


def main() -> None:
    dev = torch.device("cuda", 0)
    for q_lens, prior, seed in (([1, 33, 128, 7], [0, 15, 2000, 3], 1),
                                ([512] * 4, [workloads.prefill_prior(0, i) for i in range(4)], 2)):
        b = workloads.make_prefill_batch(q_lens, prior, seed=seed, device=dev)
        ops.store_kvcache(b.key, b.value, b.key_cache, b.value_cache, b.slot_mapping)
        out = ops.paged_prefill(b.query, b.key_cache, b.value_cache, b.cu_seqlens_q, max(q_lens),
                                b.scale, block_tables=b.block_tables, context_lens=b.context_lens)
        ref = pa.prefill(b.query.float(), b.key_cache.float(), b.value_cache.float(),
                         b.block_tables, b.context_lens, b.cu_seqlens_q, b.scale)
        assert_attn_close(out, ref)
    print("ok")


if __name__ == "__main__":
    main()
