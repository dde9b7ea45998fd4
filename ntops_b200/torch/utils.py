"""Host-side helpers shared by the ``ntops_b200.torch`` operators.

Mirrors ``ntops.torch.utils`` (src/ntops/torch/utils.py): the launch-config knobs
(``set_default_num_warps`` and friends, :22-43) are kept so callers of the reference keep
working, but hand-written kernels choose their own launch shapes, so the values are only
stored.  ``_get_matmul_input_precision`` (:218-222) keeps the reference's TF32-vs-IEEE rule.

The elementwise helpers implement torch's broadcasting and type promotion on the host and
hand the kernels stride-0 views; dtype conversion for promotion runs in the library's own copy
kernel.  Nothing here computes on the CPU.
"""

import ctypes
import warnings

import torch

from ntops_b200 import _lib


class _CachedMakeDefaultConfig:
    def __init__(self, num_warps=None, num_stages=None, max_num_configs=None):
        self.num_warps = num_warps
        self.num_stages = num_stages
        self.max_num_configs = max_num_configs


_cached_make_default_config = _CachedMakeDefaultConfig()


def get_default_num_warps():
    return _cached_make_default_config.num_warps


def set_default_num_warps(num_warps):
    _cached_make_default_config.num_warps = num_warps


def get_default_num_stages():
    return _cached_make_default_config.num_stages


def set_default_num_stages(num_stages):
    _cached_make_default_config.num_stages = num_stages


def get_default_max_num_configs():
    return _cached_make_default_config.max_num_configs


def set_default_max_num_configs(max_num_configs):
    _cached_make_default_config.max_num_configs = max_num_configs


def _get_matmul_input_precision():
    """IEEE fp32 when torch's float32 matmul precision is "highest", else TF32."""
    from ntops_b200.kernels.mm import InputPrecisionVariant

    if torch.get_float32_matmul_precision() == "highest":
        return InputPrecisionVariant.IEEE
    return InputPrecisionVariant.TF32


# --------------------------------------------------------------------------- launching ------
def lib():
    return _lib.load()


# Number of C-ABI launch calls made so far in this process (each issues at most one kernel).
launch_count = 0


def launch(what, fn, *args, device_tensor):
    """Calls ``fn(*args, stream)`` with the tensor's device current; raises on failure."""
    global launch_count
    with _lib.device_of(device_tensor):
        status = fn(*args, _lib.stream_of(device_tensor))
    _lib.check(status, what)
    launch_count += 1


def _check_cuda(*tensors):
    for t in tensors:
        if isinstance(t, torch.Tensor) and t.device.type != "cuda":
            raise RuntimeError(
                f"ntops_b200 operators run on CUDA tensors only (got {t.device}); "
                "there is no CPU fallback"
            )


def _as_tensor(value, like):
    """A 0-d device tensor for a Python scalar operand (torch.result_type keeps scalar rules)."""
    if isinstance(value, torch.Tensor):
        return value
    return torch.full((), value, device=like.device, dtype=torch.result_type(like, value))


def cast(t, dtype):
    """t converted to dtype by the library's copy kernel (t itself when already dtype)."""
    if t.dtype == dtype:
        return t
    out = torch.empty(t.shape, dtype=dtype, device=t.device)
    copy_into(out, t)
    return out


def copy_into(dst, src):
    """dst[...] = src (broadcast to dst's shape, any dtypes) on the device."""
    src = src.expand(dst.shape) if tuple(src.shape) != tuple(dst.shape) else src
    L = lib()
    xd, yd = _lib.describe(src), _lib.describe(dst)
    launch("copy", L.ntb_unary, _lib.UNARY["copy"], ctypes.byref(xd), ctypes.byref(yd), None, 0,
           device_tensor=dst)
    return dst


def contiguous(t):
    """A contiguous version of t made by the library's copy kernel."""
    if t.is_contiguous():
        return t
    out = torch.empty(t.shape, dtype=t.dtype, device=t.device)
    return copy_into(out, t)


def _prepare_out(out, shape, dtype, device):
    """Output tensor following ntops.torch.utils._prepare_out (:158-189): resize with a warning."""
    shape = tuple(shape)
    if out is None:
        return torch.empty(shape, dtype=dtype, device=device), None
    if not torch.can_cast(dtype, out.dtype):
        raise RuntimeError(f"result type {dtype} can't be cast to the desired output type {out.dtype}")
    if tuple(out.shape) != shape:
        warnings.warn(
            f"An output with one or more elements was resized since it had shape "
            f"{tuple(out.shape)}, which does not match the required output shape {shape}.",
            UserWarning,
            stacklevel=3,
        )
        out.resize_(shape)
    if out.dtype != dtype:
        return torch.empty(shape, dtype=dtype, device=device), out
    return out, None


def _finish(result, out_user):
    if out_user is None:
        return result
    copy_into(out_user, result)
    return out_user


def unary(name, input, *, out=None, out_dtype=None, scalars=None, float_op=False):
    """Runs unary op `name`; integer inputs of floating ops are promoted like torch does."""
    _check_cuda(input)
    x = input
    if float_op and not (x.is_floating_point()):
        x = cast(x, torch.get_default_dtype())
    dtype = out_dtype if out_dtype is not None else x.dtype
    y, out_user = _prepare_out(out, x.shape, dtype, x.device)
    L = lib()
    xd, yd = _lib.describe(x), _lib.describe(y)
    if scalars is not None:
        arr = (ctypes.c_double * len(scalars))(*scalars)
        sp, ns = arr, len(scalars)
    else:
        sp, ns = None, 0
    launch(name, L.ntb_unary, _lib.UNARY[name], ctypes.byref(xd), ctypes.byref(yd), sp, ns,
           device_tensor=y)
    return _finish(y, out_user)


def unary_inplace(name, input):
    """Writes op(input) back into input (ntops' ``inplace=True`` path)."""
    _check_cuda(input)
    L = lib()
    xd = _lib.describe(input)
    launch(name, L.ntb_unary, _lib.UNARY[name], ctypes.byref(xd), ctypes.byref(xd), None, 0,
           device_tensor=input)
    return input


def binary(name, input, other, *, out=None, alpha=1.0, compute_dtype=None, bool_out=False):
    """Runs binary op `name` with torch broadcasting and type promotion."""
    if not isinstance(input, torch.Tensor):
        input = _as_tensor(input, other)
    other = _as_tensor(other, input)
    _check_cuda(input, other)
    dtype = compute_dtype if compute_dtype is not None else torch.result_type(input, other)
    shape = torch.broadcast_shapes(input.shape, other.shape)
    a = cast(input, dtype).expand(shape)
    b = cast(other, dtype).expand(shape)
    y, out_user = _prepare_out(out, shape, torch.bool if bool_out else dtype, a.device)
    L = lib()
    ad, bd, yd = _lib.describe(a), _lib.describe(b), _lib.describe(y)
    launch(name, L.ntb_binary, _lib.BINARY[name], ctypes.byref(ad), ctypes.byref(bd),
           ctypes.byref(yd), float(alpha), device_tensor=y)
    return _finish(y, out_user)
