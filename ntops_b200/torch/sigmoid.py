"""ntops.torch.sigmoid drop-in: src/ntops/torch/sigmoid.py:7-15 (kernel src/ntops/kernels/sigmoid.py:9-10)."""

from ntops_b200.torch.utils import unary


def sigmoid(input, *, out=None):
    return unary("sigmoid", input, out=out, float_op=True)
