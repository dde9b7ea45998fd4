"""ntops.torch.frac drop-in: src/ntops/torch/frac.py (kernel src/ntops/kernels/frac.py:12-27).

x - trunc(x) for floating tensors.
"""

from ntops_b200.torch.utils import unary


def frac(input, *, out=None):
    if not input.is_floating_point():
        raise RuntimeError(f"frac is not implemented for {input.dtype}")
    return unary("frac", input, out=out)
