"""ntops.torch.rotary_position_embedding drop-in: src/ntops/torch/rotary_position_embedding.py:7-29
(kernel src/ntops/kernels/rotary_position_embedding.py:6-66).

input is [batch, seq, heads, emb_dim] (any strides with a unit inner stride, e.g. a view of a
fused QKV projection); sin/cos tables are [seq, emb_dim/2] broadcast over batch and heads
(:17-18).  ``inplace=True`` writes back into ``input`` (:10-11).
"""

import ctypes

import torch

from ntops_b200 import _lib
from ntops_b200.torch.utils import _check_cuda, cast, contiguous, launch, lib


def rotary_position_embedding(input, sin_table, cos_table, interleaved=True, inplace=False):
    _check_cuda(input, sin_table, cos_table)
    if input.ndim != 4:
        raise RuntimeError("rotary_position_embedding expects input of shape [batch, seq, heads, emb_dim]")
    x = input
    if x.stride(-1) != 1 and x.shape[-1] > 1:
        if inplace:
            raise RuntimeError("inplace rotary_position_embedding needs a unit inner stride")
        x = contiguous(x)
    output = input if inplace else torch.empty(input.shape, dtype=input.dtype, device=input.device)
    sn = cast(sin_table, input.dtype)
    cs = cast(cos_table, input.dtype)
    if sn.stride(-1) != 1:
        sn = contiguous(sn)
    if cs.stride(-1) != 1:
        cs = contiguous(cs)
    xd, yd = _lib.describe(x), _lib.describe(output)
    sd, cd = _lib.describe(sn), _lib.describe(cs)
    launch("rotary_position_embedding", lib().ntb_rotary_position_embedding, ctypes.byref(xd),
           ctypes.byref(sd), ctypes.byref(cd), ctypes.byref(yd), 1 if interleaved else 0,
           device_tensor=output)
    return output
