"""ctypes binding of libntops_b200.so (the C ABI in include/ntops_b200.h).

Loading fails loudly: there is no CPU or PyTorch fallback for any operator.  Every call goes
to the sm_100a kernels of the shared library on the caller's current CUDA stream.
"""

import ctypes
import os

import torch

MAX_DIMS = 8
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libntops_b200.so")

# Status codes (include/ntops_b200.h).
OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_TIMEOUT = 0, 1, 2, 3, 4

# Element type codes (include/ntops_b200.h, NtbDtype).
DTYPE_CODES = {
    torch.bool: 0,
    torch.uint8: 1,
    torch.int8: 2,
    torch.int16: 3,
    torch.int32: 4,
    torch.int64: 5,
    torch.float16: 6,
    torch.bfloat16: 7,
    torch.float32: 8,
    torch.float64: 9,
}

UNARY = {
    "copy": 0, "neg": 1, "abs": 2, "relu": 3, "exp": 4, "sigmoid": 5, "silu": 6, "gelu": 7,
    "gelu_tanh": 8, "tanh": 9, "rsqrt": 10, "sin": 11, "cos": 12, "isnan": 13, "isinf": 14,
    "bitwise_not": 15, "clamp": 16, "rad2deg": 17, "frac": 18, "lgamma": 19,
}
BINARY = {
    "add": 0, "sub": 1, "mul": 2, "div": 3, "div_trunc": 4, "div_floor": 5, "pow": 6,
    "eq": 7, "ne": 8, "lt": 9, "le": 10, "gt": 11, "ge": 12, "bitwise_and": 13, "bitwise_or": 14,
    "copysign": 15, "nextafter": 16, "lcm": 17,
}

PRECISION_TF32, PRECISION_IEEE = 1, 2
CAUSAL_NONE, CAUSAL_UPPER_LEFT, CAUSAL_LOWER_RIGHT = 0, 1, 2

# Exported symbols (every entry point declared in include/ntops_b200.h).
EXPORTS = (
    "ntb_version",
    "ntb_last_error",
    "ntb_check_device_error",
    "ntb_unary",
    "ntb_binary",
    "ntb_clamp_tensor",
    "ntb_rms_norm",
    "ntb_layer_norm",
    "ntb_softmax",
    "ntb_rotary_position_embedding",
    "ntb_gemm",
    "ntb_gemm_swiglu",
    "ntb_gemm_rope",
    "ntb_add_rms_norm",
    "ntb_dropout",
    "ntb_conv2d_workspace",
    "ntb_conv2d",
    "ntb_sdpa",
    "ntb_sdpa_workspace",
    "ntb_sdpa_ws",
    "ntb_sdpa_decode_workspace",
    "ntb_sdpa_decode",
    "ntb_sdpa_decode_static",
)


class NtbTensor(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("ndim", ctypes.c_int32),
        ("shape", ctypes.c_int64 * MAX_DIMS),
        ("stride", ctypes.c_int64 * MAX_DIMS),
    ]


_P = ctypes.POINTER(NtbTensor)
_VP = ctypes.c_void_p
_SIGNATURES = {
    "ntb_version": ([], ctypes.c_int),
    "ntb_last_error": ([], ctypes.c_char_p),
    "ntb_check_device_error": ([_VP], ctypes.c_int),
    "ntb_unary": (
        [ctypes.c_int, _P, _P, ctypes.POINTER(ctypes.c_double), ctypes.c_int, _VP],
        ctypes.c_int,
    ),
    "ntb_binary": ([ctypes.c_int, _P, _P, _P, ctypes.c_double, _VP], ctypes.c_int),
    "ntb_clamp_tensor": ([_P, _P, _P, _P, _VP], ctypes.c_int),
    "ntb_rms_norm": ([_P, _P, _P, ctypes.c_double, _VP], ctypes.c_int),
    "ntb_layer_norm": ([_P, _P, _P, _P, ctypes.c_double, _VP], ctypes.c_int),
    "ntb_softmax": ([_P, _P, ctypes.c_int, _VP], ctypes.c_int),
    "ntb_rotary_position_embedding": ([_P, _P, _P, _P, ctypes.c_int, _VP], ctypes.c_int),
    "ntb_gemm": (
        [_P, _P, _P, _P, ctypes.c_double, ctypes.c_double, ctypes.c_int, _VP],
        ctypes.c_int,
    ),
    "ntb_gemm_swiglu": ([_P, _P, _P, _VP], ctypes.c_int),
    "ntb_gemm_rope": ([_P, _P, _P, _P, _P, ctypes.c_int64, _VP], ctypes.c_int),
    "ntb_add_rms_norm": ([_P, _P, _P, _P, _P, ctypes.c_double, _VP], ctypes.c_int),
    "ntb_dropout": ([_P, _P, ctypes.c_double, ctypes.c_int64, _VP], ctypes.c_int),
    "ntb_conv2d_workspace": ([_P, _P, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int64)], ctypes.c_int),
    "ntb_conv2d": ([_P, _P, _P, _P, ctypes.POINTER(ctypes.c_int), ctypes.c_int, _VP, ctypes.c_int64, _VP],
                   ctypes.c_int),
    "ntb_sdpa": ([_P, _P, _P, _P, _P, ctypes.c_double, ctypes.c_int, _VP], ctypes.c_int),
    "ntb_sdpa_workspace": ([_P, _P, _P, _P, _P, ctypes.c_double, ctypes.POINTER(ctypes.c_int64)], ctypes.c_int),
    "ntb_sdpa_ws": ([_P, _P, _P, _P, _P, ctypes.c_double, ctypes.c_int, _VP, ctypes.c_int64, _VP], ctypes.c_int),
    "ntb_sdpa_decode_workspace": ([_P, _P, _P, ctypes.POINTER(ctypes.c_int64)], ctypes.c_int),
    "ntb_sdpa_decode": (
        [_P, _P, _P, _P, _P, ctypes.c_double, ctypes.c_int, _VP, ctypes.c_int64, _VP],
        ctypes.c_int,
    ),
    "ntb_sdpa_decode_static": ([_P, _P, _P, _P, _P, ctypes.c_double, ctypes.c_int, _VP], ctypes.c_int),
}

_lib = None


def load(path=None):
    """Loads the shared library (once) and declares every entry point's signature."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    path = path or os.environ.get("NTOPS_B200_LIB", LIB_PATH)
    if not os.path.exists(path):
        raise ImportError(
            f"ntops_b200: kernel library {path} is missing; build it with "
            "`python ntops_b200/build.py` (there is no CPU fallback)"
        )
    lib = ctypes.CDLL(path)
    for name, (argtypes, restype) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = restype
    _lib = lib
    return lib


def describe(t, shape=None, stride=None):
    """NtbTensor for a CUDA tensor (optionally reinterpreted with another shape/stride)."""
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"expected a torch.Tensor, got {type(t).__name__}")
    if t.device.type != "cuda":
        raise RuntimeError(
            f"ntops_b200 operators run on CUDA tensors only (got a tensor on {t.device}); "
            "there is no CPU fallback"
        )
    code = DTYPE_CODES.get(t.dtype)
    if code is None:
        raise RuntimeError(f"ntops_b200: unsupported dtype {t.dtype}")
    shape = tuple(t.shape) if shape is None else tuple(shape)
    stride = tuple(t.stride()) if stride is None else tuple(stride)
    if len(shape) > MAX_DIMS:
        raise RuntimeError(f"ntops_b200: at most {MAX_DIMS} dimensions are supported")
    d = NtbTensor()
    d.data = t.data_ptr()
    d.dtype = code
    d.ndim = len(shape)
    for i, (s, st) in enumerate(zip(shape, stride)):
        d.shape[i] = s
        d.stride[i] = st
    return d


def ref(desc):
    """Pointer argument for an optional descriptor (None -> NULL)."""
    return None if desc is None else ctypes.byref(desc)


def stream_of(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def check(status, what):
    if status != OK:
        msg = load().ntb_last_error().decode(errors="replace")
        raise RuntimeError(f"ntops_b200.{what}: {msg} (status {status})")


class device_of:
    """Makes the tensor's device current for the duration of a launch."""

    __slots__ = ("idx", "prev")

    def __init__(self, t):
        self.idx = t.device.index if t.device.index is not None else torch.cuda.current_device()
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.idx:
            self.prev = cur
            torch.cuda.set_device(self.idx)
        return self

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)
        return False
