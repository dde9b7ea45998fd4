"""ntops.torch.layer_norm drop-in: src/ntops/torch/layer_norm.py:9-33 (kernel src/ntops/kernels/layer_norm.py:11-48).

Biased variance, fp32 statistics, ``eps=1e-5`` default (:9).  A missing weight or bias is not
materialised as a full-size ones/zeros tensor as in the reference (:15-23); the kernel skips it.
"""

import ctypes
import math

from ntops_b200 import _lib
from ntops_b200.torch.utils import _check_cuda, launch, lib
from ntops_b200.torch._rows import row_operands


def layer_norm(input, normalized_shape, weight=None, bias=None, eps=1e-5):
    if isinstance(normalized_shape, int):
        normalized_shape = (normalized_shape,)
    normalized_shape = tuple(normalized_shape)
    _check_cuda(input, weight, bias)
    n = math.prod(normalized_shape)
    x2, y, y2, (w, b) = row_operands(input, normalized_shape, n, (weight, bias))
    if x2 is None:
        return y
    xd, yd = _lib.describe(x2), _lib.describe(y2)
    wd = _lib.describe(w) if w is not None else None
    bd = _lib.describe(b) if b is not None else None
    launch("layer_norm", lib().ntb_layer_norm, ctypes.byref(xd), _lib.ref(wd), _lib.ref(bd),
           ctypes.byref(yd), float(eps), device_tensor=y)
    return y
