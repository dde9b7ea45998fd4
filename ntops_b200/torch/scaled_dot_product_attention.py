"""ntops.torch.scaled_dot_product_attention drop-in: src/ntops/torch/scaled_dot_product_attention.py:10-108
(kernel src/ntops/kernels/scaled_dot_product_attention.py:12-262).

Same argument checks as the reference (:26-46, kept as ``assert`` for fidelity), bool masks turned
into additive 0 / -inf masks (:53-54), default scale 1/sqrt(D) (:62-63), causal variant
UPPER_LEFT by default (:65-66), output dtype = value's dtype (:73).  With ``present_key`` /
``present_value`` the new key/value rows are first stored into the cache slots
(``present_*_slot``, views into key / value; :138-139) and attention then runs over the
updated key / value.  An additive float mask is applied in natural-log units as in torch.
"""

import ctypes
import math

import torch

from ntops_b200 import _lib
from ntops_b200.kernels.scaled_dot_product_attention import CausalVariant
from ntops_b200.torch.utils import _check_cuda, cast, copy_into, launch, lib


def scaled_dot_product_attention(
    query,
    key,
    value,
    attn_mask=None,
    dropout_p=0,
    is_causal=False,
    scale=None,
    enable_gqa=False,
    causal_variant=None,
    present_key=None,
    present_value=None,
    present_key_slot=None,
    present_value_slot=None,
):
    assert dropout_p == 0, "`dropout_p` is not supported yet."

    assert attn_mask is None or not is_causal, "Cannot use `attn_mask` and `is_causal` together."

    num_heads_q = query.shape[-3]
    num_heads_kv = key.shape[-3]

    assert num_heads_kv == value.shape[-3], "Number of heads in `key` and `value` must be the same."

    if not enable_gqa:
        assert num_heads_q == num_heads_kv, (
            "Number of heads in `query`, `key`, and `value` must be the same when GQA is not enabled."
        )
    else:
        assert num_heads_q % num_heads_kv == 0, (
            "Number of heads in `query` must be divisible by number of heads in `key` and `value` when GQA is enabled."
        )

    _check_cuda(query, key, value, attn_mask)
    if query.ndim != 4 or key.ndim != 4 or value.ndim != 4:
        raise RuntimeError("scaled_dot_product_attention expects 4-D [batch, heads, seq, head_dim] tensors")

    if present_key is not None:
        # Store the new key / value rows into their cache slots before attending.
        copy_into(present_key_slot, present_key)
        copy_into(present_value_slot, present_value)

    mask = None
    if attn_mask is not None:
        if attn_mask.dtype == torch.bool:
            attn_mask = torch.where(attn_mask, 0.0, float("-inf")).to(query.dtype)
        mask_shape = query.shape[:-1] + (key.shape[-2],)
        mask = cast(attn_mask, query.dtype).expand(mask_shape)

    if scale is None:
        scale = 1 / math.sqrt(query.shape[-1])

    if causal_variant is None:
        causal_variant = CausalVariant.UPPER_LEFT
    causal = int(causal_variant) if is_causal else _lib.CAUSAL_NONE

    if value.shape[-1] == query.shape[-1]:
        # Same rule as the reference (:73): the output takes the query's memory layout, so a
        # [B, S, H, D] query viewed as [B, H, S, D] yields an output readable as [B*S, H*D].
        output = torch.empty_like(query, dtype=value.dtype)
    else:
        output = torch.empty(query.shape[:-1] + (value.shape[-1],), dtype=value.dtype, device=query.device)
    if output.numel() == 0:
        return output
    q, k, v = query, key, value
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise RuntimeError("scaled_dot_product_attention: query, key and value must share one dtype")
    qd, kd, vd, od = (_lib.describe(t) for t in (q, k, v, output))
    md = _lib.describe(mask) if mask is not None else None
    sq, group = q.shape[-2], q.shape[-3] // k.shape[-3]
    if sq <= _DECODE_MAX_Q and sq * group <= _DECODE_MAX_ROWS and q.dtype != torch.float64 \
            and all(t.stride(-1) == 1 for t in (q, k, v)):
        # Short query blocks (decoding against a KV cache): key-split kernel with a workspace
        # for the per-chunk partial results, allocated here by the caller side.
        nbytes = ctypes.c_int64(0)
        launch_ok = lib().ntb_sdpa_decode_workspace(ctypes.byref(qd), ctypes.byref(kd), ctypes.byref(vd),
                                                   ctypes.byref(nbytes))
        _lib.check(launch_ok, "scaled_dot_product_attention")
        ws = torch.empty(max(nbytes.value, 16), dtype=torch.uint8, device=q.device)
        launch("scaled_dot_product_attention", lib().ntb_sdpa_decode, ctypes.byref(qd), ctypes.byref(kd),
               ctypes.byref(vd), _lib.ref(md), ctypes.byref(od), float(scale), causal,
               ctypes.c_void_p(ws.data_ptr()), nbytes.value, device_tensor=output)
        return output
    if q.dtype == torch.float32:
        # fp32 runs on the tensor cores through fp16 copies in a workspace (TF32-equivalent
        # precision, as the reference's tl.dot on fp32); 0 bytes when the call takes another path.
        nbytes = ctypes.c_int64(0)
        _lib.check(lib().ntb_sdpa_workspace(ctypes.byref(qd), ctypes.byref(kd), ctypes.byref(vd), _lib.ref(md),
                                            ctypes.byref(od), float(scale), ctypes.byref(nbytes)),
                   "scaled_dot_product_attention")
        if nbytes.value > 0:
            ws = torch.empty(nbytes.value, dtype=torch.uint8, device=q.device)
            launch("scaled_dot_product_attention", lib().ntb_sdpa_ws, ctypes.byref(qd), ctypes.byref(kd),
                   ctypes.byref(vd), _lib.ref(md), ctypes.byref(od), float(scale), causal,
                   ctypes.c_void_p(ws.data_ptr()), nbytes.value, device_tensor=output)
            return output
    launch("scaled_dot_product_attention", lib().ntb_sdpa, ctypes.byref(qd), ctypes.byref(kd),
           ctypes.byref(vd), _lib.ref(md), ctypes.byref(od), float(scale), causal, device_tensor=output)
    return output


# Query blocks up to this many rows (and GQA group x rows) take the key-split decode kernel.
_DECODE_MAX_Q = 16
_DECODE_MAX_ROWS = 64
