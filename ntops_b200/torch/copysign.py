"""ntops.torch.copysign drop-in: src/ntops/torch/copysign.py:33-68 (kernel src/ntops/kernels/copysign.py:13-53).

|input| with the sign of other; integer operands promote to the default float dtype (torch).
"""

import torch

from ntops_b200.torch.utils import _as_tensor, binary


def copysign(input, other, *, out=None):
    a = input if isinstance(input, torch.Tensor) else _as_tensor(input, other)
    dtype = torch.result_type(a, other)
    if not dtype.is_floating_point:
        dtype = torch.get_default_dtype()
    return binary("copysign", input, other, out=out, compute_dtype=dtype)
