"""ntops.torch.rsqrt drop-in: src/ntops/torch/rsqrt.py:7-15 (kernel src/ntops/kernels/rsqrt.py:9-10)."""

from ntops_b200.torch.utils import unary


def rsqrt(input, *, out=None):
    return unary("rsqrt", input, out=out, float_op=True)
