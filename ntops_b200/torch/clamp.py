"""ntops.torch.clamp drop-in: src/ntops/torch/clamp.py:7-15 (kernel src/ntops/kernels/clamp.py:9-10); scalar bounds accepted as in torch."""

import ctypes

import torch

from ntops_b200 import _lib
from ntops_b200.torch.utils import _check_cuda, _finish, _prepare_out, cast, launch, lib, unary


def clamp(input, min=None, max=None, *, out=None):
    if min is None and max is None:
        raise RuntimeError("torch.clamp: At least one of 'min' or 'max' must not be None")
    _check_cuda(input, min, max)
    if not isinstance(min, torch.Tensor) and not isinstance(max, torch.Tensor):
        x = input
        if not x.is_floating_point() and any(isinstance(v, float) for v in (min, max)):
            x = cast(x, torch.get_default_dtype())
        scalars = [
            float(min) if min is not None else 0.0,
            float(max) if max is not None else 0.0,
            1.0 if min is not None else 0.0,
            1.0 if max is not None else 0.0,
        ]
        return unary("clamp", x, out=out, scalars=scalars)
    bounds = [b if (b is None or isinstance(b, torch.Tensor)) else torch.full((), b, device=input.device)
              for b in (min, max)]
    present = [input] + [b for b in bounds if b is not None]
    dtype = torch.result_type(*present) if len(present) == 2 else torch.promote_types(
        torch.result_type(present[0], present[1]), present[2].dtype)
    shape = torch.broadcast_shapes(*(t.shape for t in present))
    x = cast(input, dtype).expand(shape)
    lo = cast(bounds[0], dtype).expand(shape) if bounds[0] is not None else None
    hi = cast(bounds[1], dtype).expand(shape) if bounds[1] is not None else None
    y, out_user = _prepare_out(out, shape, dtype, input.device)
    xd, yd = _lib.describe(x), _lib.describe(y)
    lod = _lib.describe(lo) if lo is not None else None
    hid = _lib.describe(hi) if hi is not None else None
    launch("clamp", lib().ntb_clamp_tensor, ctypes.byref(xd), _lib.ref(lod), _lib.ref(hid),
           ctypes.byref(yd), device_tensor=y)
    return _finish(y, out_user)
