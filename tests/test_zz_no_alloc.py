"""GPU test of ntb_sdpa_decode_static, the decode-attention entry point that allocates nothing.

It exists for callers that cannot allocate device memory when they run attention (their memory
is fully reserved by their own pools or handed out by another allocator, or they reach the
library through a binding that can only pass the tensors it owns).  The test calls it through
the C ABI twice in a row, with different shapes, and checks each result against the regular
entry point ntb_sdpa_decode given a caller-allocated workspace, within the attention tolerance
the other tests use (2.5e-2 for bf16).  It also checks that shapes needing more than the fixed
scratch are refused, and that shapes whose key chunks merge on chip (no scratch) are not.  This file is collected last so a run that stops at the first failure has
already run every other test.
"""

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from ntops_b200 import _lib as L

    return L, L.load()


def _run_both(L, lib, b, hq, hkv, sq, skv, d, causal, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn((b, hq, sq, d), generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn((b, hkv, skv, d), generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn((b, hkv, skv, d), generator=g, device="cuda").to(torch.bfloat16)
    o_ref = torch.empty_like(q)
    o_static = torch.full_like(q, float("nan"))
    qd, kd, vd = L.describe(q), L.describe(k), L.describe(v)
    od_ref, od_static = L.describe(o_ref), L.describe(o_static)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    scale = 1.0 / math.sqrt(d)
    nbytes = ctypes.c_int64(0)
    assert lib.ntb_sdpa_decode_workspace(ctypes.byref(qd), ctypes.byref(kd), ctypes.byref(vd), ctypes.byref(nbytes)) == 0
    ws = torch.empty(max(nbytes.value, 16), dtype=torch.uint8, device="cuda")
    rc = lib.ntb_sdpa_decode(ctypes.byref(qd), ctypes.byref(kd), ctypes.byref(vd), None, ctypes.byref(od_ref), scale,
                             causal, ctypes.c_void_p(ws.data_ptr()), nbytes.value, stream)
    assert rc == 0, lib.ntb_last_error()
    rc = lib.ntb_sdpa_decode_static(ctypes.byref(qd), ctypes.byref(kd), ctypes.byref(vd), None,
                                    ctypes.byref(od_static), scale, causal, stream)
    assert rc == 0, lib.ntb_last_error()
    torch.cuda.synchronize()
    return o_static, o_ref


def test_static_scratch_entry_matches_workspace_entry_twice():
    L, lib = _lib()
    # two calls in a row with different shapes: the second must not see the first one's partials
    for args in [(2, 32, 8, 1, 4096, 128, 0, 1), (1, 8, 2, 4, 777, 64, 2, 2)]:
        o_static, o_ref = _run_both(L, lib, *args)
        assert torch.isfinite(o_static.float()).all()
        torch.testing.assert_close(o_static.float(), o_ref.float(), rtol=2.5e-2, atol=2.5e-2)


def test_static_scratch_entry_refuses_oversized_shapes():
    L, lib = _lib()
    # batch 16 x 64 query heads over 32 kv heads x 16 query rows (32 rows per kv head, which
    # takes the workspace path) x head_dim 128: ~8.5 MB of partials > 4 MiB
    q = torch.zeros((16, 64, 16, 128), dtype=torch.bfloat16, device="cuda")
    k = torch.zeros((16, 32, 256, 128), dtype=torch.bfloat16, device="cuda")
    o = torch.empty_like(q)
    qd, kd, od = L.describe(q), L.describe(k), L.describe(o)
    rc = lib.ntb_sdpa_decode_static(ctypes.byref(qd), ctypes.byref(kd), ctypes.byref(kd), None, ctypes.byref(od),
                                    0.1, 0, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == L.ERR_UNSUPPORTED
    assert b"static scratch" in lib.ntb_last_error()


def test_static_scratch_entry_takes_large_cluster_merged_shapes():
    L, lib = _lib()
    # 16 rows per kv head, bf16, head_dim 128: the chunks merge on chip and need no scratch, so
    # a shape whose partials would not fit the 4 MiB array still runs
    o_static, o_ref = _run_both(L, lib, 16, 64, 64, 16, 256, 128, 0, 3)
    assert torch.isfinite(o_static.float()).all()
    torch.testing.assert_close(o_static.float(), o_ref.float(), rtol=2.5e-2, atol=2.5e-2)
