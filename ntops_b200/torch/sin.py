"""ntops.torch.sin drop-in: src/ntops/torch/sin.py:7-15 (kernel src/ntops/kernels/sin.py:9)."""

from ntops_b200.torch.utils import unary


def sin(input, *, out=None):
    return unary("sin", input, out=out, float_op=True)
