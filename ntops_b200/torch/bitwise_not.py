"""ntops.torch.bitwise_not drop-in: src/ntops/torch/bitwise_not.py:7-17 (kernel src/ntops/kernels/bitwise_not.py:9-24; logical not for bool)."""

from ntops_b200.torch.utils import unary


def bitwise_not(input, *, out=None):
    return unary("bitwise_not", input, out=out)
