"""ntops.torch.pow drop-in: src/ntops/torch/pow.py:7-15 (kernel src/ntops/kernels/pow.py:9-10)."""

from ntops_b200.torch.utils import binary


def pow(input, exponent, *, out=None):
    return binary("pow", input, exponent, out=out)
