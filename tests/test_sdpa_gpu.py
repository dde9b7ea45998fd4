"""Parity of scaled_dot_product_attention against the oracle.

The reference grid (tests/test_scaled_dot_product_attention.py:15-92: mask None / bool /
float(0 or -inf), causal, scale, fp32 / fp16, KV cache, causal variant; seq 1-512, head_dim
32 / 64, GQA always on; tolerances fp32 1e-2, fp16 2.5e-2) runs mostly on the CUDA-core kernel;
the bf16 / fp16 head_dim 64 / 128 cases without a mask run on the tcgen05 kernel, including
ragged sequence lengths, Sq != Skv, lower-right causal, GQA and strided [B, S, H, D] views.
"""

import itertools
import math
import random

import pytest
import torch

import oracle.ops as O
from ntops_b200.kernels.scaled_dot_product_attention import CausalVariant
from tests.utils import assert_close

pytestmark = pytest.mark.gpu

nt = pytest.importorskip("ntops_b200.torch") if torch.cuda.is_available() else None
DEV = "cuda"


def _reference_grid():
    r = random.Random(99)
    out = []
    for mask_t, causal, scale, dtype, kv, variant in itertools.product(
        (None, torch.bool, torch.float32), (False, True), (None, r.uniform(0.05, 0.5)),
        (torch.float32, torch.float16), (False, True), (None, CausalVariant.LOWER_RIGHT, CausalVariant.UPPER_LEFT)):
        if mask_t is not None and causal:
            continue
        b, hq = r.randint(1, 4), 2 ** r.randint(1, 5)
        sq, d = r.randint(1, 512), r.choice([32, 64])
        hkv = 2 ** r.randint(1, int(math.log2(hq)))
        skv = r.randint(1, 512)
        if variant == CausalVariant.LOWER_RIGHT and sq > skv:
            continue
        out.append((b, hq, sq, d, hkv, skv, mask_t, causal, scale, variant, kv, dtype))
    return out


def _tol(dtype):
    return {torch.float32: (1e-2, 1e-2), torch.float16: (2.5e-2, 2.5e-2), torch.bfloat16: (2.5e-2, 2.5e-2)}[dtype]


@pytest.mark.parametrize("b,hq,sq,d,hkv,skv,mask_t,causal,scale,variant,with_kv,dtype", _reference_grid())
def test_reference_grid(b, hq, sq, d, hkv, skv, mask_t, causal, scale, variant, with_kv, dtype):
    q = torch.randn((b, hq, sq, d)).to(dtype)
    k = torch.randn((b, hkv, skv, d)).to(dtype)
    v = torch.randn((b, hkv, skv, d)).to(dtype)
    mask = None
    if mask_t is not None:
        mask = torch.rand((sq, skv)) > 0.5
        if mask_t is not torch.bool:
            mask = torch.where(mask, 0.0, float("-inf")).to(dtype)
    kd, vd = k.to(DEV), v.to(DEV)
    pk = pv = pks = pvs = None
    if with_kv:
        pk, pv = kd[:, :, -1:, :].clone(), vd[:, :, -1:, :].clone()
        pks, pvs = kd[:, :, -1:, :], vd[:, :, -1:, :]
        pks[...] = 0
        pvs[...] = 0
    got = nt.scaled_dot_product_attention(q.to(DEV), kd, vd, attn_mask=None if mask is None else mask.to(DEV),
                                          is_causal=causal, scale=scale, enable_gqa=True, causal_variant=variant,
                                          present_key=pk, present_value=pv, present_key_slot=pks,
                                          present_value_slot=pvs)
    cv = 2 if variant == CausalVariant.LOWER_RIGHT else 1
    want = O.scaled_dot_product_attention(q, k, v, mask, causal, scale, cv)
    assert_close(got, want, tol=_tol(dtype), equal_nan=True)


TC_CASES = [
    # b, hq, hkv, sq, skv, d, causal_variant (0 none)
    (1, 2, 2, 128, 128, 128, 0),
    (2, 4, 2, 256, 256, 128, 1),
    (1, 8, 2, 300, 300, 128, 1),
    (2, 4, 4, 200, 333, 64, 0),
    (1, 4, 1, 129, 520, 128, 2),
    (1, 2, 2, 1000, 1000, 64, 1),
    (1, 4, 2, 64, 700, 128, 2),
    (2, 2, 1, 512, 384, 128, 0),
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("b,hq,hkv,sq,skv,d,cv", TC_CASES)
def test_tensor_core_path(b, hq, hkv, sq, skv, d, cv, dtype):
    q = torch.randn((b, hq, sq, d)).to(dtype)
    k = torch.randn((b, hkv, skv, d)).to(dtype)
    v = torch.randn((b, hkv, skv, d)).to(dtype)
    got = nt.scaled_dot_product_attention(q.to(DEV), k.to(DEV), v.to(DEV), is_causal=cv != 0, enable_gqa=True,
                                          causal_variant=CausalVariant(cv) if cv else None)
    want = O.scaled_dot_product_attention(q, k, v, None, cv != 0, None, cv if cv else 1)
    assert_close(got, want, tol=(2e-2, 2e-2), equal_nan=True)


def test_strided_bshd_views():
    # Llama layout: q/k/v come from [B, S, H, D] projections and are attended as [B, H, S, D] views.
    B, S, Hq, Hkv, D = 2, 256, 8, 2, 128
    q = torch.randn((B, S, Hq, D)).to(torch.bfloat16)
    k = torch.randn((B, S, Hkv, D)).to(torch.bfloat16)
    v = torch.randn((B, S, Hkv, D)).to(torch.bfloat16)
    got = nt.scaled_dot_product_attention(q.to(DEV).transpose(1, 2), k.to(DEV).transpose(1, 2),
                                          v.to(DEV).transpose(1, 2), is_causal=True, enable_gqa=True)
    want = O.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), None, True)
    assert_close(got, want, tol=(2e-2, 2e-2))


def test_large_logits_rescale():
    # Rows whose max grows across KV blocks exercise the O rescale of the tcgen05 kernel.
    B, H, S, D = 1, 2, 640, 128
    q = torch.randn((B, H, S, D)) * 3
    k = torch.randn((B, H, S, D)) * 3
    k[:, :, 500:] *= 2.0
    v = torch.randn((B, H, S, D))
    qb, kb, vb = (t.to(torch.bfloat16) for t in (q, k, v))
    got = nt.scaled_dot_product_attention(qb.to(DEV), kb.to(DEV), vb.to(DEV))
    want = O.scaled_dot_product_attention(qb, kb, vb)
    assert_close(got, want, tol=(2e-2, 2e-2))


def test_asserts_like_reference():
    q = torch.randn((1, 4, 8, 32), device=DEV)
    k = torch.randn((1, 2, 8, 32), device=DEV)
    with pytest.raises(AssertionError):
        nt.scaled_dot_product_attention(q, k, k)  # GQA shapes without enable_gqa
    with pytest.raises(AssertionError):
        nt.scaled_dot_product_attention(q, q, q, dropout_p=0.1)


# Additive / bool masks on the tensor-core kernel (bf16 / fp16, head_dim 64 / 128, more than 16
# query rows so the decode kernel is not taken): broadcast and per-head masks, ragged lengths,
# GQA, rows whose every key is masked (NaN, as torch), and negative scales.
MASK_TC_CASES = [
    # b, hq, hkv, sq, skv, d, dtype, mask_kind, scale
    (1, 4, 4, 256, 256, 128, torch.bfloat16, "bool_2d", None),
    (2, 8, 2, 300, 517, 128, torch.bfloat16, "float_per_head", None),
    (1, 2, 1, 129, 1000, 64, torch.float16, "float_2d", None),
    (2, 4, 4, 384, 384, 64, torch.bfloat16, "bool_per_batch", 0.3),
    (1, 4, 2, 200, 333, 128, torch.float16, "float_per_head", -0.08),
    (1, 2, 2, 256, 256, 128, torch.bfloat16, "rows_fully_masked", None),
    # fp32: the staged tensor-core path (mask copied to fp16 in its broadcast shape)
    (1, 4, 4, 256, 256, 128, torch.float32, "bool_2d", None),
    (2, 8, 2, 300, 517, 128, torch.float32, "float_per_head", None),
    (1, 2, 1, 129, 1000, 64, torch.float32, "float_2d", None),
    (2, 4, 4, 384, 384, 64, torch.float32, "bool_per_batch", 0.3),
    (1, 4, 2, 200, 333, 128, torch.float32, "float_per_head", -0.08),
    (1, 2, 2, 256, 256, 128, torch.float32, "rows_fully_masked", None),
]


@pytest.mark.parametrize("b,hq,hkv,sq,skv,d,dtype,mask_kind,scale", MASK_TC_CASES)
def test_masked_attention_tensor_core(b, hq, hkv, sq, skv, d, dtype, mask_kind, scale):
    g = torch.Generator().manual_seed(sq * 7 + skv)
    q = torch.randn((b, hq, sq, d), generator=g).to(dtype)
    k = torch.randn((b, hkv, skv, d), generator=g).to(dtype)
    v = torch.randn((b, hkv, skv, d), generator=g).to(dtype)
    keep = None
    if mask_kind == "bool_2d":
        mask = torch.rand((sq, skv), generator=g) > 0.3
    elif mask_kind == "bool_per_batch":
        mask = torch.rand((b, 1, sq, skv), generator=g) > 0.5
    elif mask_kind == "float_2d":
        mask = torch.where(torch.rand((sq, skv), generator=g) > 0.4, 0.0, float("-inf")).to(dtype)
    elif mask_kind == "float_per_head":
        mask = (torch.randn((b, hq, sq, skv), generator=g) * 2).to(dtype)
        mask[..., ::7] = float("-inf")
    else:  # every key of some rows masked
        keep = torch.rand((sq, skv), generator=g) > 0.3
        keep[::5] = False
        mask = keep
    got = nt.scaled_dot_product_attention(q.to(DEV), k.to(DEV), v.to(DEV), attn_mask=mask.to(DEV), scale=scale,
                                          enable_gqa=True)
    want = O.scaled_dot_product_attention(q, k, v, mask, False, scale)
    tol = (1e-2, 1e-2) if dtype == torch.float32 else (2.5e-2, 2.5e-2)
    assert_close(got, want, tol=tol, equal_nan=True)
    if keep is not None:
        assert torch.isnan(got[:, :, ::5].float()).all()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_negative_scale_without_mask(dtype):
    # the unmasked tensor-core kernel needs a positive scale; a negative one runs elsewhere
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn((1, 2, 256, 128), generator=g).to(dtype) for _ in range(3))
    got = nt.scaled_dot_product_attention(q.to(DEV), k.to(DEV), v.to(DEV), scale=-0.05)
    assert_close(got, O.scaled_dot_product_attention(q, k, v, None, False, -0.05), tol=(2.5e-2, 2.5e-2))


# fp32 attention on the tensor cores (fp16 copies with an exact power-of-two scale per tensor,
# TF32-equivalent precision like the reference's tl.dot on fp32): magnitudes far from 1 in both
# directions, head_dim 64 / 128, causal variants, GQA, Sq != Skv, strided [B, S, H, D] views.
FP32_TC_CASES = [
    # b, hq, hkv, sq, skv, d, magnitude, causal, layout
    (1, 4, 2, 1024, 1024, 128, 1.0, None, "bhsd"),
    (2, 8, 2, 300, 517, 64, 1e3, None, "bhsd"),
    (1, 4, 4, 777, 777, 128, 1e-3, CausalVariant.UPPER_LEFT, "bhsd"),
    (2, 4, 1, 200, 640, 64, 37.0, CausalVariant.LOWER_RIGHT, "bshd"),
    (1, 2, 2, 2048, 2048, 128, 0.05, CausalVariant.UPPER_LEFT, "bshd"),
    (2, 4, 2, 333, 400, 64, 3.0, None, "offset"),  # rows not 16-byte aligned: element-wise staging
]


@pytest.mark.parametrize("case", FP32_TC_CASES)
def test_fp32_tensor_core_staged(case):
    b, hq, hkv, sq, skv, d, mag, causal, layout = case
    g = torch.Generator().manual_seed(11)
    q = torch.randn((b, hq, sq, d), generator=g) * mag
    k = torch.randn((b, hkv, skv, d), generator=g) * mag
    v = torch.randn((b, hkv, skv, d), generator=g) * mag
    scale = 1.0 / (math.sqrt(d) * mag * mag) if mag != 1.0 else None
    if layout == "bshd":
        qd, kd, vd = (t.transpose(1, 2).contiguous().to(DEV).transpose(1, 2) for t in (q, k, v))
    elif layout == "offset":  # views one element into wider rows
        qd, kd, vd = (torch.cat((torch.zeros(t.shape[:-1] + (1,)), t), -1).to(DEV)[..., 1:] for t in (q, k, v))
    else:
        qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    kw = {}
    if causal is None:
        want = O.scaled_dot_product_attention(q, k, v, None, False, scale)
    else:
        kw = {"is_causal": True, "causal_variant": causal}
        want = O.scaled_dot_product_attention(q, k, v, None, True, scale, causal_variant=int(causal))
    got = nt.scaled_dot_product_attention(qd, kd, vd, scale=scale, enable_gqa=True, **kw)
    assert got.dtype == torch.float32
    assert_close(got, want, tol=(1e-2, 1e-2 * mag))


def test_fp32_workspace_query():
    """The staged path asks for a workspace only for fp32 without a mask and with a positive
    scale; ntb_sdpa (no workspace) still runs fp32 on the CUDA-core kernel, within the same
    tolerance of the oracle."""
    import ctypes

    from ntops_b200 import _lib as L

    lib = L.load()
    g = torch.Generator().manual_seed(12)
    q, k, v = (torch.randn((1, 2, 256, 64), generator=g) for _ in range(3))
    o = torch.empty((1, 2, 256, 64), device=DEV)
    qg, kg, vg = q.to(DEV), k.to(DEV), v.to(DEV)  # kept alive while their descriptors are used
    qd, kd, vd, od = (L.describe(t) for t in (qg, kg, vg, o))
    nbytes = ctypes.c_int64(-1)
    assert lib.ntb_sdpa_workspace(ctypes.byref(qd), ctypes.byref(kd), ctypes.byref(vd), None, ctypes.byref(od),
                                  0.125, ctypes.byref(nbytes)) == L.OK
    assert nbytes.value >= 256 + 3 * 256 * 64 * 2 * 2
    assert lib.ntb_sdpa_workspace(ctypes.byref(qd), ctypes.byref(kd), ctypes.byref(vd), None, ctypes.byref(od),
                                  -0.125, ctypes.byref(nbytes)) == L.OK
    assert nbytes.value == 0
    qb, kb, vb, ob = (t.to(DEV, torch.bfloat16) for t in (q, k, v, o))
    qbd, kbd, vbd, obd = (L.describe(t) for t in (qb, kb, vb, ob))
    assert lib.ntb_sdpa_workspace(ctypes.byref(qbd), ctypes.byref(kbd), ctypes.byref(vbd), None,
                                  ctypes.byref(obd), 0.125, ctypes.byref(nbytes)) == L.OK
    assert nbytes.value == 0
    assert lib.ntb_sdpa(ctypes.byref(qd), ctypes.byref(kd), ctypes.byref(vd), None, ctypes.byref(od), 0.125, 0,
                        None) == L.OK
    torch.cuda.synchronize()
    assert_close(o.cpu(), O.scaled_dot_product_attention(q, k, v, None, False, 0.125), tol=(1e-2, 1e-2))
