"""CPU tests of the C ABI boundary: the shared library loads, exports exactly the entry points
include/ntops_b200.h declares, and rejects bad arguments with status codes and messages before
touching a GPU.  No kernel is launched here."""

import ctypes
import os
import re
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "ntops_b200.h")


def _declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"NTB_API\s+(?:const\s+)?\w+\**\s*\**\s*(ntb_\w+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    from ntops_b200 import _lib

    lib = _lib.load()
    declared = _declared()
    assert len(declared) >= 12
    for name in declared:
        assert hasattr(lib, name), name
    assert sorted(_lib.EXPORTS) == declared
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = sorted(l.split()[-1] for l in out.splitlines() if re.search(r" T ntb_", l))
    assert exported == declared


def test_version_and_empty_error():
    from ntops_b200 import _lib

    lib = _lib.load()
    assert lib.ntb_version() == 1
    assert isinstance(lib.ntb_last_error(), bytes)


def test_null_descriptor_is_rejected_without_a_gpu():
    from ntops_b200 import _lib

    lib = _lib.load()
    d = _lib.NtbTensor()
    rc = lib.ntb_unary(_lib.UNARY["exp"], None, ctypes.byref(d), None, 0, None)
    assert rc == _lib.ERR_INVALID
    assert b"NULL" in lib.ntb_last_error()
    rc = lib.ntb_rms_norm(None, None, None, 1e-6, None)
    assert rc == _lib.ERR_INVALID


def test_bad_ndim_and_dtype_codes_are_rejected():
    from ntops_b200 import _lib

    lib = _lib.load()
    d = _lib.NtbTensor()
    d.ndim = 9
    rc = lib.ntb_softmax(ctypes.byref(d), ctypes.byref(d), 0, None)
    assert rc == _lib.ERR_INVALID and b"ndim" in lib.ntb_last_error()
    d.ndim = 1
    d.dtype = 42
    rc = lib.ntb_softmax(ctypes.byref(d), ctypes.byref(d), 0, None)
    assert rc == _lib.ERR_UNSUPPORTED


def test_cpu_tensors_are_refused_by_the_shim():
    import torch

    import ntops_b200.torch as nt

    for fn, args in [(nt.add, (torch.ones(2), torch.ones(2))), (nt.rms_norm, (torch.ones(2, 4), 4)),
                     (nt.mm, (torch.ones(2, 2), torch.ones(2, 2)))]:
        with pytest.raises(RuntimeError, match="CUDA"):
            fn(*args)


def test_public_api_matches_reference_names():
    import ntops_b200.torch as nt
    from ntops_b200.kernels.mm import InputPrecisionVariant
    from ntops_b200.kernels.scaled_dot_product_attention import CausalVariant

    for name in ["rms_norm", "layer_norm", "softmax", "rotary_position_embedding", "add", "sub", "mul", "div",
                 "silu", "gelu", "sigmoid", "exp", "clamp", "pow", "eq", "ne", "lt", "le", "gt", "ge",
                 "bitwise_and", "bitwise_or", "bitwise_not", "neg", "abs", "relu", "tanh", "rsqrt", "sin", "cos",
                 "isnan", "isinf", "mm", "bmm", "addmm", "matmul", "scaled_dot_product_attention"]:
        assert name in nt.__all__ and callable(getattr(nt, name))
    assert int(CausalVariant.UPPER_LEFT) == 1 and int(CausalVariant.LOWER_RIGHT) == 2
    assert int(InputPrecisionVariant.TF32) == 1 and int(InputPrecisionVariant.IEEE) == 2
    import inspect

    sig = inspect.signature(nt.scaled_dot_product_attention)
    assert list(sig.parameters)[:13] == ["query", "key", "value", "attn_mask", "dropout_p", "is_causal", "scale",
                                         "enable_gqa", "causal_variant", "present_key", "present_value",
                                         "present_key_slot", "present_value_slot"]
    assert str(inspect.signature(nt.add)) == "(input, other, *, alpha=1, out=None)"
    assert str(inspect.signature(nt.rms_norm)) == "(input, normalized_shape, weight=None, eps=None)"


def test_launch_knobs_are_kept():
    from ntops_b200.torch import utils

    utils.set_default_num_warps(4)
    utils.set_default_num_stages(2)
    utils.set_default_max_num_configs(3)
    assert (utils.get_default_num_warps(), utils.get_default_num_stages(), utils.get_default_max_num_configs()) == (4, 2, 3)
