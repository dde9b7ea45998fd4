"""ntops.torch.le drop-in: src/ntops/torch/le.py:7-15 (kernel src/ntops/kernels/le.py:8-9); returns bool like torch."""

from ntops_b200.torch.utils import binary


def le(input, other, *, out=None):
    return binary("le", input, other, out=out, bool_out=True)
