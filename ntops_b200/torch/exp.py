"""ntops.torch.exp drop-in: src/ntops/torch/exp.py:7-15 (kernel src/ntops/kernels/exp.py:9-10)."""

from ntops_b200.torch.utils import unary


def exp(input, *, out=None):
    return unary("exp", input, out=out, float_op=True)
