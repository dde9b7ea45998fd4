"""ntops.torch.conv2d drop-in: src/ntops/torch/conv2d.py:8-52 (kernel src/ntops/kernels/conv2d.py).

Same arguments and rules as the reference: int or pair stride / padding / dilation, padding
"valid" means 0, groups must be 1, NCHW output of the input's dtype, bias optional.  The output
size follows src/ntops/torch/pooling.py:4-16 (floor mode).  The library runs im2col into a
workspace allocated here plus one GEMM per image on the tensor cores (fp16 / bf16)."""

import ctypes

import torch

from ntops_b200 import _lib
from ntops_b200.torch.utils import _check_cuda, _get_matmul_input_precision, launch, lib


def _pair(v):
    return (v, v) if isinstance(v, int) else tuple(v)


def conv2d(input, weight, bias=None, stride=1, padding=0, dilation=1, groups=1):
    _check_cuda(input, weight, bias)
    stride = _pair(stride)
    if isinstance(padding, str):
        if padding == "valid":
            padding = 0
        else:
            raise RuntimeError(f"conv2d: padding '{padding}' is not supported")
    padding = _pair(padding)
    dilation = _pair(dilation)
    assert groups == 1, "`groups` is not supported yet."

    n, _, h, w = input.shape
    k, _, r, s = weight.shape
    p = (h + 2 * padding[0] - dilation[0] * (r - 1) - 1) // stride[0] + 1
    q = (w + 2 * padding[1] - dilation[1] * (s - 1) - 1) // stride[1] + 1
    output = torch.empty((n, k, p, q), dtype=input.dtype, device=input.device)

    L = lib()
    params = (ctypes.c_int * 6)(stride[0], stride[1], padding[0], padding[1], dilation[0], dilation[1])
    xd, wd, yd = _lib.describe(input), _lib.describe(weight), _lib.describe(output)
    bd = _lib.describe(bias) if bias is not None else None
    nbytes = ctypes.c_int64(0)
    _lib.check(L.ntb_conv2d_workspace(ctypes.byref(xd), ctypes.byref(wd), params, ctypes.byref(nbytes)), "conv2d")
    ws = torch.empty(max(nbytes.value, 256), dtype=torch.uint8, device=input.device)
    precision = int(_get_matmul_input_precision()) if input.dtype == torch.float32 else _lib.PRECISION_IEEE
    launch("conv2d", L.ntb_conv2d, ctypes.byref(xd), ctypes.byref(wd), _lib.ref(bd), ctypes.byref(yd), params,
           precision, ctypes.c_void_p(ws.data_ptr()), nbytes.value, device_tensor=output)
    return output
