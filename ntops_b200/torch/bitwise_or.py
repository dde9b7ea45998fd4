"""ntops.torch.bitwise_or drop-in: src/ntops/torch/bitwise_or.py:7-15 (kernel src/ntops/kernels/bitwise_or.py:8-9)."""

from ntops_b200.torch.utils import binary


def bitwise_or(input, other, *, out=None):
    return binary("bitwise_or", input, other, out=out)
