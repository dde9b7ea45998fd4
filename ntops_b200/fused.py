"""Fused operators for the Llama layer chain (beyond the reference's operator list).

``swiglu_linear(x, w_packed)`` computes ``silu(x @ Wg) * (x @ Wu)`` — the chain's gate / up
projections, silu and mul — in one tcgen05 GEMM whose epilogue applies SwiGLU, so the two
[tokens, 14336] products never reach HBM.  ``pack_swiglu_weight(wg, wu)`` lays the two weights
out once, interleaved in column blocks of 128, as the kernel expects.

``add_rms_norm(x, residual, weight, eps)`` returns ``(s, rms_norm(s))`` with ``s = x + residual``
in one pass over the rows (the chain's residual add and the following norm).

``qkv_rope_linear(x, w_qkv, sin, cos, rope_cols)`` computes the Q, K and V projections as one
GEMM over the side-by-side weight and rotates the Q and K heads (the first ``rope_cols``
columns, heads of 128, non-interleaved RoPE) in its epilogue, so RoPE costs no pass over HBM.
"""

import ctypes

import torch

from ntops_b200 import _lib
from ntops_b200.torch.utils import _check_cuda, contiguous, copy_into, launch, lib

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


def qkv_rope_linear(x, w_qkv, sin_table, cos_table, rope_cols, out=None):
    """x [M, K] @ w_qkv [K, N], with every 128-column head below ``rope_cols`` rotated by RoPE
    (non-interleaved; position = row % seq_len of the [seq_len, 64] tables); returns [M, N]."""
    _check_cuda(x, w_qkv, sin_table, cos_table)
    M, N = x.shape[0], w_qkv.shape[1]
    d = out if out is not None else torch.empty((M, N), dtype=x.dtype, device=x.device)
    xd, wd, dd = _lib.describe(x), _lib.describe(w_qkv), _lib.describe(d)
    sd, cd = _lib.describe(contiguous(sin_table)), _lib.describe(contiguous(cos_table))
    launch("qkv_rope_linear", lib().ntb_gemm_rope, ctypes.byref(xd), ctypes.byref(wd), ctypes.byref(sd),
           ctypes.byref(cd), ctypes.byref(dd), int(rope_cols), device_tensor=d)
    return d


def pack_qkv_weight(w_q, w_k, w_v):
    """[K, Nq], [K, Nk], [K, Nv] -> [K, Nq + Nk + Nv] side by side (Q columns first)."""
    _check_cuda(w_q, w_k, w_v)
    K = w_q.shape[0]
    if not (w_k.shape[0] == K and w_v.shape[0] == K):
        raise RuntimeError("Q, K and V weights must share their input dimension")
    nq, nk, nv = w_q.shape[1], w_k.shape[1], w_v.shape[1]
    packed = torch.empty((K, nq + nk + nv), dtype=w_q.dtype, device=w_q.device)
    copy_into(packed[:, :nq], w_q)
    copy_into(packed[:, nq:nq + nk], w_k)
    copy_into(packed[:, nq + nk:], w_v)
    return packed


def add_rms_norm(x, residual, weight, eps, out=None):
    """s = x + residual (rounded to x's dtype) and rms_norm(s) over the last dim with ``weight``;
    returns ``(s, y)``.  ``out`` may be ``x`` or ``residual`` to update the stream in place."""
    _check_cuda(x, residual, weight)
    n = x.shape[-1]
    x2, r2 = contiguous(x).view(-1, n), contiguous(residual).view(-1, n)
    s = out if out is not None else torch.empty_like(x2)
    s2 = s.view(-1, n)
    y = torch.empty_like(x2)
    xd, rd, sd, yd = _lib.describe(x2), _lib.describe(r2), _lib.describe(s2), _lib.describe(y)
    wd = _lib.describe(contiguous(weight).view(n)) if weight is not None else None
    launch("add_rms_norm", lib().ntb_add_rms_norm, ctypes.byref(xd), ctypes.byref(rd), _lib.ref(wd), ctypes.byref(sd),
           ctypes.byref(yd), float(eps), device_tensor=y)
    return s.view(x.shape), y.view(x.shape)
