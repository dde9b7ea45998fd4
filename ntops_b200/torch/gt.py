"""ntops.torch.gt drop-in: src/ntops/torch/gt.py:7-15 (kernel src/ntops/kernels/gt.py:8-9); returns bool like torch."""

from ntops_b200.torch.utils import binary


def gt(input, other, *, out=None):
    return binary("gt", input, other, out=out, bool_out=True)
