"""ntops.torch.rad2deg drop-in: src/ntops/torch/rad2deg.py:37-65 (kernel src/ntops/kernels/rad2deg.py:13-19).

x * 180 / pi; integer inputs promote to the default float dtype (torch).
"""

from ntops_b200.torch.utils import unary


def rad2deg(input, *, out=None):
    return unary("rad2deg", input, out=out, float_op=True)
