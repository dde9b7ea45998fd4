"""Parity of the key-split decode attention (short query blocks against a long KV range) with
the oracle: GQA groups, ragged key counts, causal variants, additive / bool masks, head dims
and dtypes, and the KV-cache slot store of the reference API (present_key / present_value)."""

import pytest
import torch

import oracle.ops as O
from ntops_b200.kernels.scaled_dot_product_attention import CausalVariant
from tests.utils import assert_close

pytestmark = pytest.mark.gpu

nt = pytest.importorskip("ntops_b200.torch") if torch.cuda.is_available() else None
DEV = "cuda"

CASES = [
    # b, hq, hkv, sq, skv, d
    (1, 32, 8, 1, 8192, 128),
    (2, 8, 8, 1, 1000, 64),
    (2, 16, 4, 4, 777, 128),
    (1, 4, 1, 16, 300, 64),
    (3, 4, 2, 2, 33, 128),
    (1, 8, 2, 1, 1, 128),
    (1, 2, 2, 8, 5000, 96),
]


def _tol(dtype):
    return {torch.float32: (1e-4, 1e-4), torch.float16: (2.5e-2, 2.5e-2), torch.bfloat16: (2.5e-2, 2.5e-2)}[dtype]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("b,hq,hkv,sq,skv,d", CASES)
@pytest.mark.parametrize("causal", [0, 2])
def test_decode(b, hq, hkv, sq, skv, d, causal, dtype):
    if causal == 2 and sq > skv:
        pytest.skip("lower-right causal needs Skv >= Sq")
    q = torch.randn((b, hq, sq, d)).to(dtype)
    k = torch.randn((b, hkv, skv, d)).to(dtype)
    v = torch.randn((b, hkv, skv, d)).to(dtype)
    got = nt.scaled_dot_product_attention(q.to(DEV), k.to(DEV), v.to(DEV), is_causal=causal != 0, enable_gqa=True,
                                          causal_variant=CausalVariant.LOWER_RIGHT if causal else None)
    want = O.scaled_dot_product_attention(q, k, v, None, causal != 0, None, causal or 1)
    assert_close(got, want, tol=_tol(dtype))


@pytest.mark.parametrize("mask_kind", ["bool", "float"])
def test_decode_masks(mask_kind):
    b, hq, hkv, sq, skv, d = 2, 8, 2, 2, 900, 128
    q, k, v = (torch.randn(s).to(torch.bfloat16) for s in ((b, hq, sq, d), (b, hkv, skv, d), (b, hkv, skv, d)))
    m = torch.rand(sq, skv) > 0.3
    if mask_kind == "float":
        m = torch.where(m, 0.0, float("-inf")).to(torch.bfloat16)
    got = nt.scaled_dot_product_attention(q.to(DEV), k.to(DEV), v.to(DEV), attn_mask=m.to(DEV), enable_gqa=True)
    assert_close(got, O.scaled_dot_product_attention(q, k, v, m), tol=(2.5e-2, 2.5e-2))


def test_decode_with_kv_cache_slot_store():
    b, hq, hkv, sq, skv, d = 1, 8, 2, 1, 2048, 128
    q = torch.randn((b, hq, sq, d)).to(torch.bfloat16)
    k = torch.randn((b, hkv, skv, d)).to(torch.bfloat16)
    v = torch.randn((b, hkv, skv, d)).to(torch.bfloat16)
    kd, vd = k.to(DEV), v.to(DEV)
    pk, pv = kd[:, :, -1:, :].clone(), vd[:, :, -1:, :].clone()
    kd[:, :, -1:, :] = 0
    vd[:, :, -1:, :] = 0
    got = nt.scaled_dot_product_attention(q.to(DEV), kd, vd, enable_gqa=True, present_key=pk, present_value=pv,
                                          present_key_slot=kd[:, :, -1:, :], present_value_slot=vd[:, :, -1:, :])
    assert torch.equal(kd.cpu(), k) and torch.equal(vd.cpu(), v)
    assert_close(got, O.scaled_dot_product_attention(q, k, v), tol=(2.5e-2, 2.5e-2))
