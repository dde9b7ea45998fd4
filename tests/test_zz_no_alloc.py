"""GPU test of ntb_sdpa_decode_static, the decode-attention entry point that allocates nothing.

It exists for callers that cannot allocate device memory when they run attention: a serving
runtime that reserved all of HBM for its own pools at start-up, a host whose only device memory
is what another framework's allocator hands it, or a foreign-language binding that can pass the
tensors it owns but has no way to obtain a workspace.  Those callers get the per-chunk partial
results kept in a fixed 4 MiB device array inside the library.

The cases here take the path that really uses that array (the key-split partials plus the merge
kernel): an additive mask, fp32 inputs, and more than 16 query rows per kv head.  They run one
after another through the C ABI with a large shape first and smaller ones after it, so later
calls find the earlier calls' partials still in the array, then the first shape once more.  Each
result is checked against the fp64 oracle (attention tolerance: 2.5e-2 for bf16, 1e-4 for fp32)
and against ntb_sdpa_decode given a caller-allocated workspace (the same kernels, so the results
are bit-identical).  Shapes whose partials exceed 4 MiB are refused, while the cluster-merged
path, which needs no scratch, takes large shapes.  This file is collected last so a run that
stops at the first failure has already run every other test.
"""

import ctypes
import math

import pytest
import torch

import oracle.ops as O
from tests.utils import assert_close

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 4 << 20


def _lib():
    from ntops_b200 import _lib as L

    return L, L.load()


def _need(L, lib, q, k, v):
    """Bytes of partials the key-split path needs for these shapes (the workspace query)."""
    nbytes = ctypes.c_int64(0)
    qd, kd, vd = L.describe(q), L.describe(k), L.describe(v)
    assert lib.ntb_sdpa_decode_workspace(ctypes.byref(qd), ctypes.byref(kd), ctypes.byref(vd),
                                         ctypes.byref(nbytes)) == 0
    return nbytes.value


def _inputs(b, hq, hkv, sq, skv, d, dtype, masked, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn((b, hq, sq, d), generator=g, device="cuda").to(dtype)
    k = torch.randn((b, hkv, skv, d), generator=g, device="cuda").to(dtype)
    v = torch.randn((b, hkv, skv, d), generator=g, device="cuda").to(dtype)
    mask = None
    if masked:
        keep = torch.rand((sq, skv), generator=g, device="cuda") > 0.3
        keep[:, 0] = True  # no fully masked row
        mask = torch.where(keep, 0.0, float("-inf")).to(dtype).expand(b, hq, sq, skv)
    return q, k, v, mask


def _run(L, lib, q, k, v, mask, causal):
    """(static-entry output, workspace-entry output, partial bytes) for one call of each."""
    scale = 1.0 / math.sqrt(q.shape[-1])
    o_static = torch.full_like(q, float("nan"))
    o_ws = torch.empty_like(q)
    qd, kd, vd, od_s, od_w = (L.describe(t) for t in (q, k, v, o_static, o_ws))
    md = L.describe(mask) if mask is not None else None
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    need = _need(L, lib, q, k, v)
    rc = lib.ntb_sdpa_decode_static(ctypes.byref(qd), ctypes.byref(kd), ctypes.byref(vd), L.ref(md),
                                    ctypes.byref(od_s), scale, causal, stream)
    assert rc == 0, lib.ntb_last_error()
    ws = torch.empty(max(need, 16), dtype=torch.uint8, device="cuda")
    rc = lib.ntb_sdpa_decode(ctypes.byref(qd), ctypes.byref(kd), ctypes.byref(vd), L.ref(md), ctypes.byref(od_w),
                             scale, causal, ctypes.c_void_p(ws.data_ptr()), need, stream)
    assert rc == 0, lib.ntb_last_error()
    torch.cuda.synchronize()
    return o_static, o_ws, need


# (b, hq, hkv, sq, skv, d, dtype, masked, causal): every case needs partials (the scratch path)
CASES = [
    (2, 32, 8, 1, 4096, 128, torch.bfloat16, True, 0),   # additive mask: ~0.5 MiB of partials
    (1, 8, 2, 4, 777, 64, torch.float32, False, 2),      # fp32, lower-right causal: ~33 KiB
    (1, 32, 1, 1, 2048, 128, torch.bfloat16, False, 0),  # 32 query rows per kv head: ~130 KiB
]


def test_static_scratch_entry_on_the_scratch_path():
    L, lib = _lib()
    first = None
    for i, (b, hq, hkv, sq, skv, d, dtype, masked, causal) in enumerate(CASES + CASES[:1]):
        q, k, v, mask = _inputs(b, hq, hkv, sq, skv, d, dtype, masked, seed=10 + (i % len(CASES)))
        o_static, o_ws, need = _run(L, lib, q, k, v, mask, causal)
        assert 0 < need <= SCRATCH_BYTES, need
        assert torch.isfinite(o_static.float()).all()
        assert torch.equal(o_static, o_ws), "static scratch and caller workspace give different results"
        want = O.scaled_dot_product_attention(q.cpu(), k.cpu(), v.cpu(), None if mask is None else mask.cpu(),
                                              causal != 0, None, causal or 1)
        tol = (1e-4, 1e-4) if dtype == torch.float32 else (2.5e-2, 2.5e-2)
        assert_close(o_static, want, tol=tol)
        if i == 0:
            first = o_static.clone()
        elif i == len(CASES):
            # the first shape again, after smaller calls left their partials in the array
            assert torch.equal(o_static, first)


def test_static_scratch_entry_refuses_oversized_shapes():
    L, lib = _lib()
    # batch 16 x 64 query heads over 32 kv heads x 16 query rows (32 rows per kv head, which
    # takes the key-split path) x head_dim 128: more partials than the array holds
    q = torch.zeros((16, 64, 16, 128), dtype=torch.bfloat16, device="cuda")
    k = torch.zeros((16, 32, 256, 128), dtype=torch.bfloat16, device="cuda")
    assert _need(L, lib, q, k, k) > SCRATCH_BYTES
    o = torch.empty_like(q)
    qd, kd, od = L.describe(q), L.describe(k), L.describe(o)
    rc = lib.ntb_sdpa_decode_static(ctypes.byref(qd), ctypes.byref(kd), ctypes.byref(kd), None, ctypes.byref(od),
                                    0.1, 0, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == L.ERR_UNSUPPORTED
    assert b"static scratch" in lib.ntb_last_error()


def test_static_scratch_refusal_depends_on_the_path():
    L, lib = _lib()
    # 16 rows per kv head, bf16, head_dim 128: without a mask the key chunks merge on chip and
    # need no scratch, so the shape runs although its partials would exceed the array; the same
    # shape with an additive mask takes the key-split path and is refused
    b, hq, hkv, sq, skv, d = 16, 64, 64, 16, 256, 128
    q, k, v, mask = _inputs(b, hq, hkv, sq, skv, d, torch.bfloat16, True, seed=3)
    assert _need(L, lib, q, k, v) > SCRATCH_BYTES
    o_static, o_ws, _ = _run(L, lib, q, k, v, None, 0)
    assert torch.equal(o_static, o_ws)
    want = O.scaled_dot_product_attention(q[:2].cpu(), k[:2].cpu(), v[:2].cpu())
    assert_close(o_static[:2], want, tol=(2.5e-2, 2.5e-2))
    o = torch.empty_like(q)
    qd, kd, vd, md, od = (L.describe(t) for t in (q, k, v, mask, o))
    rc = lib.ntb_sdpa_decode_static(ctypes.byref(qd), ctypes.byref(kd), ctypes.byref(vd), ctypes.byref(md),
                                    ctypes.byref(od), 1.0 / math.sqrt(d), 0,
                                    ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == L.ERR_UNSUPPORTED
    assert b"static scratch" in lib.ntb_last_error()
