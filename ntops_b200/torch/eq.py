"""ntops.torch.eq drop-in: src/ntops/torch/eq.py:7-15 (kernel src/ntops/kernels/eq.py:8-9); returns bool like torch."""

from ntops_b200.torch.utils import binary


def eq(input, other, *, out=None):
    return binary("eq", input, other, out=out, bool_out=True)
