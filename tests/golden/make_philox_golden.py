"""Generates tests/golden/philox_golden.pt: uniforms of Triton's own tl.rand (the random source
of the reference's dropout kernel, kernels/dropout.py:10) for several seeds and offsets,
computed by Triton's CPU interpreter (TRITON_INTERPRET=1; Triton 3.6 in this image), so the
oracle's Philox restatement (oracle/ops.py philox_rand) is pinned to Triton's implementation.

Run from the repository root: python tests/golden/make_philox_golden.py
"""

import os

os.environ["TRITON_INTERPRET"] = "1"

import torch  # noqa: E402
import triton  # noqa: E402
import triton.language as tl  # noqa: E402


@triton.jit
def _rand_kernel(out_ptr, off_ptr, seed, n, BLOCK: tl.constexpr):
    i = tl.program_id(0) * BLOCK + tl.arange(0, BLOCK)
    m = i < n
    off = tl.load(off_ptr + i, mask=m, other=0)
    tl.store(out_ptr + i, tl.rand(seed, off), mask=m)


def main():
    g = torch.Generator().manual_seed(0)
    offsets = torch.cat([
        torch.arange(0, 512, dtype=torch.int64),
        torch.randint(0, 2**31, (256,), generator=g, dtype=torch.int64),
        torch.randint(2**32, 2**44, (256,), generator=g, dtype=torch.int64),
    ])
    cases = []
    for seed in (0, 1, 12345, 2**31 - 1, 987654321):
        out = torch.empty(offsets.shape, dtype=torch.float32)
        block = 1024
        _rand_kernel[(triton.cdiv(offsets.numel(), block),)](out, offsets, seed, offsets.numel(), BLOCK=block)
        cases.append({"seed": seed, "offsets": offsets.clone(), "rand": out})
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "philox_golden.pt")
    torch.save({"triton": triton.__version__, "cases": cases}, path)
    print("wrote", path, "triton", triton.__version__)


if __name__ == "__main__":
    main()
