"""ntops.torch.nextafter drop-in: src/ntops/torch/nextafter.py:36-72 (kernel src/ntops/kernels/nextafter.py:13-123).

The next representable value after input toward other, in the operands' floating dtype.
"""

from ntops_b200.torch.utils import binary


def nextafter(input, other, *, out=None):
    return binary("nextafter", input, other, out=out)
