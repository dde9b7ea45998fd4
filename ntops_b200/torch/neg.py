"""ntops.torch.neg drop-in: src/ntops/torch/neg.py:7-15 (kernel src/ntops/kernels/neg.py:8)."""

from ntops_b200.torch.utils import unary


def neg(input, *, out=None):
    return unary("neg", input, out=out)
