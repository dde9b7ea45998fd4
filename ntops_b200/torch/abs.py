"""ntops.torch.abs drop-in: src/ntops/torch/abs.py:7-15 (kernel src/ntops/kernels/abs.py:9-10)."""

from ntops_b200.torch.utils import unary


def abs(input, *, out=None):
    return unary("abs", input, out=out)
