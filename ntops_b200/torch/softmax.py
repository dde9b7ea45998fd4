"""ntops.torch.softmax drop-in: src/ntops/torch/softmax.py:7-16 (kernel src/ntops/kernels/softmax.py:14-42).

The output dtype is ``dtype`` when given, else the input's (:8-10).  Statistics accumulate in
fp32 (fp64 when input or output is fp64) for every dtype.
"""

import ctypes

import torch

from ntops_b200 import _lib
from ntops_b200.torch.utils import _check_cuda, contiguous, launch, lib


def softmax(input, dim, dtype=None):
    _check_cuda(input)
    out_dtype = dtype if dtype is not None else input.dtype
    y = torch.empty(input.shape, dtype=out_dtype, device=input.device)
    if input.numel() == 0:
        return y
    nd = input.ndim
    d = dim + nd if (nd > 0 and dim < 0) else dim
    if nd > 0 and not (0 <= d < nd):
        raise IndexError(f"Dimension out of range (expected to be in range of [{-nd}, {nd - 1}], but got {dim})")
    x = input
    inner_is_last = nd == 0 or all(s == 1 for s in x.shape[d + 1:])
    if not inner_is_last or not x.is_contiguous():
        x = contiguous(x)
    xd, yd = _lib.describe(x), _lib.describe(y)
    launch("softmax", lib().ntb_softmax, ctypes.byref(xd), ctypes.byref(yd), int(d if nd else 0),
           device_tensor=y)
    return y
