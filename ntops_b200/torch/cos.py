"""ntops.torch.cos drop-in: src/ntops/torch/cos.py:7-15 (kernel src/ntops/kernels/cos.py:9)."""

from ntops_b200.torch.utils import unary


def cos(input, *, out=None):
    return unary("cos", input, out=out, float_op=True)
