"""Fused operators for the Llama layer chain (beyond the reference's operator list).

``swiglu_linear(x, w_packed)`` computes ``silu(x @ Wg) * (x @ Wu)`` — the chain's gate / up
projections, silu and mul — in one tcgen05 GEMM whose epilogue applies SwiGLU, so the two
[tokens, 14336] products never reach HBM.  ``pack_swiglu_weight(wg, wu)`` lays the two weights
out once, interleaved in column blocks of 128, as the kernel expects.
"""

import ctypes

import torch

from ntops_b200 import _lib
from ntops_b200.torch.utils import _check_cuda, copy_into, launch, lib

BLOCK = 128


def pack_swiglu_weight(w_gate, w_up):
    """[K, N] gate and up weights -> [K, 2N] with 128-column blocks alternating gate / up."""
    _check_cuda(w_gate, w_up)
    if w_gate.shape != w_up.shape or w_gate.ndim != 2:
        raise RuntimeError("gate and up weights must be 2-D with the same shape")
    K, N = w_gate.shape
    if N % BLOCK:
        raise RuntimeError(f"weight width {N} must be a multiple of {BLOCK}")
    packed = torch.empty((K, 2 * N), dtype=w_gate.dtype, device=w_gate.device)
    view = packed.view(K, N // BLOCK, 2, BLOCK)
    copy_into(view[:, :, 0, :], w_gate.view(K, N // BLOCK, BLOCK))
    copy_into(view[:, :, 1, :], w_up.view(K, N // BLOCK, BLOCK))
    return packed


def swiglu_linear(x, w_packed, out=None):
    """silu(x @ Wg) * (x @ Wu) for x [M, K] and a packed weight [K, 2N]; returns [M, N]."""
    _check_cuda(x, w_packed)
    M, N = x.shape[0], w_packed.shape[1] // 2
    d = out if out is not None else torch.empty((M, N), dtype=x.dtype, device=x.device)
    xd, wd, dd = _lib.describe(x), _lib.describe(w_packed), _lib.describe(d)
    launch("swiglu_linear", lib().ntb_gemm_swiglu, ctypes.byref(xd), ctypes.byref(wd), ctypes.byref(dd),
           device_tensor=d)
    return d
