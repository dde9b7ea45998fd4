"""ntops.torch.mul drop-in: src/ntops/torch/mul.py:7-15 (kernel src/ntops/kernels/mul.py:8-9)."""

from ntops_b200.torch.utils import binary


def mul(input, other, *, out=None):
    return binary("mul", input, other, out=out)
