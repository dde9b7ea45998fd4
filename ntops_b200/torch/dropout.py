"""ntops.torch.dropout drop-in: src/ntops/torch/dropout.py:9-29 (kernel src/ntops/kernels/dropout.py:10-11).

As in the reference, each call draws its seed with Python's ``random.randrange(0, 2**31)``, so
seeding Python's ``random`` reproduces a call, and the keep mask for a seed is the reference's
(Philox-4x32-10 uniform of the element index, kept where it exceeds ``p``); kept elements are
divided by ``1 - p``.  Non-contiguous inputs are processed in their logical (row-major) order.
"""

import ctypes
import random

import torch

from ntops_b200 import _lib
from ntops_b200.torch.utils import _check_cuda, contiguous, copy_into, launch, lib


def dropout(input, p=0.5, training=True, inplace=False):
    _check_cuda(input)
    if not training or p == 0:
        return input if inplace else _copy(input)

    seed = random.randrange(0, 2**31)

    x = contiguous(input)
    if inplace and input.is_contiguous():
        output = input
    else:
        output = torch.empty(input.shape, dtype=input.dtype, device=input.device)
    xd, yd = _lib.describe(x), _lib.describe(output)
    launch("dropout", lib().ntb_dropout, ctypes.byref(xd), ctypes.byref(yd), float(p), int(seed),
           device_tensor=output)
    if inplace and output is not input:
        copy_into(input, output)
        return input
    return output


def _copy(t):
    """A fresh tensor with t's values (the reference's ``input.clone()``), via the library's copy."""
    out = torch.empty_like(t)
    copy_into(out, t)
    return out
