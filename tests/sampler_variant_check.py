"""Child-process check used by test_gpu_sampler.test_sampler_kernel_options:
greedy ids (with planted ties and a NaN row) from whichever greedy kernel the
environment selects, against the oracle."""

import numpy as np
import torch

from litevllm_b200 import ops
from oracle import sampler as osamp


def main() -> None:
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(5)
    for B, V in ((256, 128256), (8, 151936), (3, 1000), (64, 50000)):
        x = torch.randn((B, V), generator=g).bfloat16()
        for b in range(B):
            i, j = sorted(torch.randint(0, V, (2,), generator=g).tolist())
            x[b, j] = 40.0
            x[b, i] = 40.0
        x[B - 1, V // 3] = float("nan")
        got = ops.sample(x.to(dev)).cpu().numpy()
        assert np.array_equal(got, osamp.greedy(x.float().numpy())), (B, V)
    print("ok")


if __name__ == "__main__":
    main()
