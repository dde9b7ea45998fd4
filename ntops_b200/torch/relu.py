"""ntops.torch.relu drop-in: src/ntops/torch/relu.py:7-17 (kernel src/ntops/kernels/relu.py:8-9)."""

from ntops_b200.torch.utils import unary, unary_inplace


def relu(input, inplace=False):
    if inplace:
        return unary_inplace("relu", input)
    return unary("relu", input, float_op=False)
