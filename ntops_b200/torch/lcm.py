"""ntops.torch.lcm drop-in: src/ntops/torch/lcm.py:4-92 (kernel src/ntops/kernels/lcm.py:14-128).

Least common multiple of integer tensors (non-negative; 0 when either operand is 0).
"""

from ntops_b200.torch.utils import binary


def lcm(input, other, *, out=None):
    return binary("lcm", input, other, out=out)
