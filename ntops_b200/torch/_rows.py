"""Row view shared by rms_norm and layer_norm: [rows, prod(normalized_shape)] with unit inner
stride, per-row parameters as contiguous vectors of the input's dtype."""

import torch

from ntops_b200.torch.utils import cast, contiguous


def row_operands(input, normalized_shape, n, params):
    k = len(normalized_shape)
    if k > input.ndim or tuple(input.shape[input.ndim - k:]) != normalized_shape:
        raise RuntimeError(
            f"Given normalized_shape={list(normalized_shape)}, expected input with shape "
            f"[*, {', '.join(str(s) for s in normalized_shape)}], but got input of size {list(input.shape)}"
        )
    y = torch.empty(input.shape, dtype=input.dtype, device=input.device)
    rows = input.numel() // n if n else 0
    if input.numel() == 0:
        return None, y, None, tuple(None for _ in params)
    try:
        x2 = input.view(rows, n)
    except RuntimeError:
        x2 = None
    if x2 is None or (n > 1 and x2.stride(1) != 1):
        x2 = contiguous(input).view(rows, n)
    y2 = y.view(rows, n)
    out = []
    for p in params:
        if p is None:
            out.append(None)
            continue
        if p.device != input.device:
            raise RuntimeError("weight/bias must be on the input's device")
        p = p.expand(normalized_shape) if tuple(p.shape) != tuple(normalized_shape) else p
        out.append(contiguous(cast(p, input.dtype)).view(n))
    return x2, y, y2, tuple(out)
