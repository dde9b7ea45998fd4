"""ntops.torch.silu drop-in: src/ntops/torch/silu.py:7-17 (kernel src/ntops/kernels/silu.py:9-10)."""

from ntops_b200.torch.utils import unary, unary_inplace


def silu(input, inplace=False):
    if inplace:
        return unary_inplace("silu", input)
    return unary("silu", input, float_op=True)
