"""Shared launcher of mm / bmm / addmm / matmul over ntb_gemm."""

import ctypes

import torch

from ntops_b200 import _lib
from ntops_b200.torch.utils import _check_cuda, _get_matmul_input_precision, contiguous, copy_into, launch, lib


def _k_major(t):
    """A view of t ([..., rows, K]) whose K dimension has unit stride (copy if needed)."""
    if t.stride(-1) == 1:
        return t
    return contiguous(t)


def _k_major_b(t):
    """A view of t ([..., K, N]) whose K dimension has unit stride (copy of the transpose if needed)."""
    if t.stride(-2) == 1:
        return t
    return contiguous(t.transpose(-1, -2)).transpose(-1, -2)


def gemm(a, b, c, out, alpha, beta, out_shape, what):
    """out = alpha * a @ b + beta * c with a [.., M, K], b [.., K, N], c expanded to out_shape."""
    _check_cuda(a, b, c, out)
    if a.dtype != b.dtype:
        raise RuntimeError(f"{what}: expected mat1 and mat2 to have the same dtype, but got {a.dtype} != {b.dtype}")
    dtype = c.dtype if c is not None else a.dtype
    if dtype != a.dtype:
        raise RuntimeError(f"{what}: expected the input and the matrices to have the same dtype, but got {dtype} and {a.dtype}")
    precision = int(_get_matmul_input_precision()) if a.dtype == torch.float32 else _lib.PRECISION_IEEE
    if precision == _lib.PRECISION_TF32:
        # TF32 tensor-core kernels take K-major operands.
        a, b = _k_major(a), _k_major_b(b)
    user_out = None
    if out is not None:
        if tuple(out.shape) != tuple(out_shape):
            out.resize_(out_shape)
        if out.dtype == dtype and out.stride(-1) == 1:
            d = out
        else:
            user_out, d = out, torch.empty(out_shape, dtype=dtype, device=a.device)
    else:
        d = torch.empty(out_shape, dtype=dtype, device=a.device)
    ad, bd, dd = _lib.describe(a), _lib.describe(b), _lib.describe(d)
    cd = None
    if c is not None:
        cd = _lib.describe(c.expand(out_shape))
    launch(what, lib().ntb_gemm, ctypes.byref(ad), ctypes.byref(bd), _lib.ref(cd), ctypes.byref(dd),
           float(alpha), float(beta), precision, device_tensor=d)
    if user_out is not None:
        copy_into(user_out, d)
        return user_out
    return d
