"""ntops.torch.bitwise_and drop-in: src/ntops/torch/bitwise_and.py:7-15 (kernel src/ntops/kernels/bitwise_and.py:8-9)."""

from ntops_b200.torch.utils import binary


def bitwise_and(input, other, *, out=None):
    return binary("bitwise_and", input, other, out=out)
