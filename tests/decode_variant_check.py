"""Child-process check used by test_gpu_decode.test_decode_kernel_options:
ragged decode batches (split and unsplit, several GQA ratios) and a
shared-prefix batch with whichever decode options the environment selects,
against the fp32 oracle."""

import torch

from litevllm_b200 import ops, workloads
from oracle import paged_attention as pa
from tests.tolerance import assert_attn_close


def main() -> None:
    dev = torch.device("cuda", 0)
    for H, H_kv, ctx, splits in ((32, 8, [4096, 1, 2000, 17, 1023, 300], 0),
                                 (32, 8, [4096, 1, 2000, 17, 1023, 300], 3),
                                 (16, 4, [5, 700, 64, 129], 0), (8, 8, [33, 2048], 2)):
        b = workloads.make_decode_batch(2, len(ctx), seed=H + len(ctx), H=H, H_kv=H_kv, ctx=ctx,
                                        device=dev)
        out = ops.paged_decode(b.query, b.key_cache, b.value_cache, b.block_tables,
                               b.context_lens, b.scale, num_splits=splits)
        ref = pa.decode(b.query.float(), b.key_cache.float(), b.value_cache.float(),
                        b.block_tables, b.context_lens, b.scale)
        assert_attn_close(out, ref)
    # shared-prefix decode (config 4 shape, fewer rows)
    b = workloads.make_prefix_batch(24, seed=2, device=dev)
    out = ops.paged_decode_shared_prefix(b.query, b.key_cache, b.value_cache, b.block_tables,
                                         b.context_lens, b.scale, 127 * 16)
    ref = pa.decode(b.query.float(), b.key_cache.float(), b.value_cache.float(), b.block_tables,
                    b.context_lens, b.scale, rows=[0, 5, 23])
    assert_attn_close(out[[0, 5, 23]], ref)
    print("ok")


if __name__ == "__main__":
    main()
