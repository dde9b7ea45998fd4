"""ntops.torch.ne drop-in: src/ntops/torch/ne.py:7-15 (kernel src/ntops/kernels/ne.py:8-9); returns bool like torch."""

from ntops_b200.torch.utils import binary


def ne(input, other, *, out=None):
    return binary("ne", input, other, out=out, bool_out=True)
