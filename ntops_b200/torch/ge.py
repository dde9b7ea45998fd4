"""ntops.torch.ge drop-in: src/ntops/torch/ge.py:7-15 (kernel src/ntops/kernels/ge.py:8-9); returns bool like torch."""

from ntops_b200.torch.utils import binary


def ge(input, other, *, out=None):
    return binary("ge", input, other, out=out, bool_out=True)
