"""ntops.torch.tanh drop-in: src/ntops/torch/tanh.py:7-15 (kernel src/ntops/kernels/tanh.py:9-12)."""

from ntops_b200.torch.utils import unary


def tanh(input, *, out=None):
    return unary("tanh", input, out=out, float_op=True)
