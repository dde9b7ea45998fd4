"""ntops.torch.lgamma drop-in: src/ntops/torch/lgamma.py:11-44 (kernel src/ntops/kernels/lgamma.py:14-29).

log|gamma(x)| (CUDA's lgamma); integer inputs promote to the default float dtype.
"""

from ntops_b200.torch.utils import unary


def lgamma(input, *, out=None):
    return unary("lgamma", input, out=out, float_op=True)
