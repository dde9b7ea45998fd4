"""ntops.torch.lt drop-in: src/ntops/torch/lt.py:7-15 (kernel src/ntops/kernels/lt.py:8-9); returns bool like torch."""

from ntops_b200.torch.utils import binary


def lt(input, other, *, out=None):
    return binary("lt", input, other, out=out, bool_out=True)
