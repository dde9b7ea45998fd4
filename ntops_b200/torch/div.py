"""ntops.torch.div drop-in: src/ntops/torch/div.py:7-15 (kernel src/ntops/kernels/div.py:9-37)."""

import torch

from ntops_b200.torch.utils import _as_tensor, binary


def div(input, other, *, rounding_mode=None, out=None):
    if rounding_mode is None:
        # True division promotes integer operands to the default floating dtype (torch rule).
        a = input if isinstance(input, torch.Tensor) else _as_tensor(input, other)
        dtype = torch.result_type(a, other)
        if not dtype.is_floating_point:
            dtype = torch.get_default_dtype()
        return binary("div", input, other, out=out, compute_dtype=dtype)
    if rounding_mode == "trunc":
        return binary("div_trunc", input, other, out=out)
    if rounding_mode == "floor":
        return binary("div_floor", input, other, out=out)
    raise ValueError(
        f"div expected rounding_mode to be one of None, 'trunc', or 'floor' but found '{rounding_mode}'"
    )
