"""ntops.torch.rms_norm drop-in: src/ntops/torch/rms_norm.py:9-31 (kernel src/ntops/kernels/rms_norm.py:10-43).

Same defaults as the reference: ``eps`` defaults to ``torch.finfo(input.dtype).eps`` (:20-21),
the output has the input's dtype and shape (:23).  The statistics run in fp32 on the device.
"""

import ctypes
import math

import torch

from ntops_b200 import _lib
from ntops_b200.torch.utils import _check_cuda, launch, lib
from ntops_b200.torch._rows import row_operands


def rms_norm(input, normalized_shape, weight=None, eps=None):
    if isinstance(normalized_shape, int):
        normalized_shape = (normalized_shape,)
    normalized_shape = tuple(normalized_shape)
    _check_cuda(input, weight)
    if eps is None:
        eps = torch.finfo(input.dtype).eps
    n = math.prod(normalized_shape)
    x2, y, y2, (w,) = row_operands(input, normalized_shape, n, (weight,))
    if x2 is None:
        return y
    xd, yd = _lib.describe(x2), _lib.describe(y2)
    wd = _lib.describe(w) if w is not None else None
    launch("rms_norm", lib().ntb_rms_norm, ctypes.byref(xd), _lib.ref(wd), ctypes.byref(yd),
           float(eps), device_tensor=y)
    return y
