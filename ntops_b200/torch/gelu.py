"""ntops.torch.gelu drop-in: src/ntops/torch/gelu.py:7-14 (kernel src/ntops/kernels/gelu.py:10-39)."""

from ntops_b200.torch.utils import unary


def gelu(input, approximate="none"):
    if approximate == "tanh":
        return unary("gelu_tanh", input, float_op=True)
    if approximate == "none":
        return unary("gelu", input, float_op=True)
    raise RuntimeError(f"approximate argument must be either none or tanh, got {approximate!r}")
