"""Parity of rms_norm, layer_norm, softmax and rotary_position_embedding against the oracle.

Grids follow the reference tests (tests/test_rms_norm.py, test_layer_norm.py:11-37,
test_softmax.py:11-21, test_rotary_position_embedding.py:48-89) plus bf16, rows that stay
resident in the shared-memory ring, rows too long for it (re-read path), many rows per CTA (the
ring wraps), odd lengths (strided fallback), strided layouts and data far from zero.
"""

import random

import pytest
import torch

import oracle.ops as O
from tests.utils import assert_close, case_id, float_cases

pytestmark = pytest.mark.gpu

nt = pytest.importorskip("ntops_b200.torch") if torch.cuda.is_available() else None
DEV = "cuda"
CASES = float_cases()


def _randn(shape, dtype, scale=1.0):
    return (torch.randn(shape) * scale).to(dtype)


@pytest.mark.parametrize("eps", [None, 0.0, 1e-5, 1e-3])
@pytest.mark.parametrize("weight_is_none", [False, True])
@pytest.mark.parametrize("case", CASES, ids=case_id)
def test_rms_norm(case, weight_is_none, eps):
    shape, dtype = case
    x = _randn(shape, dtype)
    ns = tuple(shape[-random.randint(1, len(shape)):])
    w = None if weight_is_none else _randn(ns, dtype)
    got = nt.rms_norm(x.to(DEV), ns, None if w is None else w.to(DEV), eps)
    assert_close(got, O.rms_norm(x, ns, w, eps))


@pytest.mark.parametrize("eps", [1e-8, 1e-5, 1e-3])
@pytest.mark.parametrize("bias_is_none", [False, True])
@pytest.mark.parametrize("weight_is_none", [False, True])
@pytest.mark.parametrize("case", CASES, ids=case_id)
def test_layer_norm(case, weight_is_none, bias_is_none, eps):
    shape, dtype = case
    x = _randn(shape, dtype)
    ns = tuple(shape[-random.randint(1, len(shape)):])
    w = None if weight_is_none else _randn(ns, dtype)
    b = None if bias_is_none else _randn(ns, dtype)
    got = nt.layer_norm(x.to(DEV), ns, None if w is None else w.to(DEV), None if b is None else b.to(DEV), eps)
    assert_close(got, O.layer_norm(x, ns, w, b, eps))


@pytest.mark.parametrize("out_dtype", [None, torch.float16, torch.float32, torch.float64])
@pytest.mark.parametrize("case", CASES, ids=case_id)
def test_softmax(case, out_dtype):
    shape, dtype = case
    x = _randn(shape, dtype)
    dim = random.randint(0, len(shape) - 1)
    got = nt.softmax(x.to(DEV), dim, out_dtype)
    want = O.softmax(x, dim, out_dtype)
    assert_close(got, want, dtype=want.dtype if want.dtype != torch.float64 else torch.float32)


@pytest.mark.parametrize("cols", [1, 7, 31, 33, 255, 1000, 4096, 8192, 16384, 32768, 65536, 70001, 300000])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_long_rows(cols, dtype):
    rows = 3
    x = _randn((rows, cols), dtype, 2.0)
    w = _randn((cols,), dtype)
    b = _randn((cols,), dtype)
    assert_close(nt.rms_norm(x.to(DEV), cols, w.to(DEV), 1e-6), O.rms_norm(x, cols, w, 1e-6))
    assert_close(nt.layer_norm(x.to(DEV), cols, w.to(DEV), b.to(DEV), 1e-5), O.layer_norm(x, cols, w, b, 1e-5))
    assert_close(nt.softmax(x.to(DEV), -1), O.softmax(x, -1))


@pytest.mark.parametrize(
    "rows,cols,dtype",
    [(5000, 4096, torch.float32), (1200, 8192, torch.bfloat16), (600, 32768, torch.float32),
     (300, 65536, torch.float32), (3000, 96, torch.float16), (700, 24576, torch.bfloat16)],
)
def test_many_rows(rows, cols, dtype):
    # more rows than CTAs: each CTA walks several rows and its ring of slots wraps around
    x = _randn((rows, cols), dtype, 2.0)
    w = _randn((cols,), dtype)
    b = _randn((cols,), dtype)
    xd = x.to(DEV)
    assert_close(nt.rms_norm(xd, cols, w.to(DEV), 1e-6), O.rms_norm(x, cols, w, 1e-6))
    assert_close(nt.layer_norm(xd, cols, w.to(DEV), b.to(DEV), 1e-5), O.layer_norm(x, cols, w, b, 1e-5))
    assert_close(nt.softmax(xd, -1), O.softmax(x, -1))


@pytest.mark.parametrize(
    "rows,cols,dtype",
    [(4096, 4096, torch.bfloat16), (777, 4096, torch.float16), (300, 2048, torch.float32), (64, 8192, torch.bfloat16),
     (50, 33, torch.float32), (1, 16384, torch.bfloat16)],
)
@pytest.mark.parametrize("weight_is_none", [False, True])
def test_add_rms_norm(rows, cols, dtype, weight_is_none):
    from ntops_b200.fused import add_rms_norm

    x = _randn((rows, cols), dtype)
    r = _randn((rows, cols), dtype)
    w = None if weight_is_none else _randn((cols,), dtype)
    s_want = (x.double() + r.double()).to(dtype)
    y_want = O.rms_norm(s_want, cols, w, 1e-6)
    s, y = add_rms_norm(x.to(DEV), r.to(DEV), None if w is None else w.to(DEV), 1e-6)
    assert torch.equal(s.cpu(), s_want)
    assert_close(y, y_want)
    # in place: the sum overwrites x
    xd = x.to(DEV)
    s2, y2 = add_rms_norm(xd, r.to(DEV), None if w is None else w.to(DEV), 1e-6, out=xd)
    assert s2.data_ptr() == xd.data_ptr() and torch.equal(xd.cpu(), s_want)
    assert_close(y2, y_want)


@pytest.mark.parametrize("cols", [4096, 65536])
def test_layer_norm_offset_data(cols):
    # mean far from zero relative to the spread: the statistics must not cancel
    x = torch.randn(64, cols) * 0.01 + 1000.0
    assert_close(nt.layer_norm(x.to(DEV), cols, None, None, 1e-5), O.layer_norm(x, cols, None, None, 1e-5))


def test_strided_rows():
    base = _randn((64, 3000), torch.float32)
    x = base[:, 100:2148]  # row stride 3000, inner stride 1
    w = _randn((2048,), torch.float32)
    assert_close(nt.rms_norm(x.to(DEV), 2048, w.to(DEV), 1e-6), O.rms_norm(x, 2048, w, 1e-6))
    assert_close(nt.softmax(base.to(DEV)[:, 100:2148], 1), O.softmax(x, 1))
    xt = _randn((512, 40), torch.float32).t()  # inner stride 40 -> copied first
    assert_close(nt.layer_norm(xt.to(DEV), 512), O.layer_norm(xt, 512))


def test_softmax_special_values():
    x = torch.randn(4, 300)
    x[0, :] = float("-inf")  # fully masked row -> NaN, as torch
    x[1, 5] = float("inf")
    x[2, 7] = float("nan")
    got = nt.softmax(x.to(DEV), -1).cpu()
    want = torch.softmax(x.double(), -1).float()
    torch.testing.assert_close(got, want, equal_nan=True, rtol=1e-5, atol=1e-5)


# ---------------------------------------------------------------------------- RoPE --------
def _ref_rope(x, s, c, interleaved):
    return O.rotary_position_embedding(x, s, c, interleaved)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("inplace", [False, True])
@pytest.mark.parametrize("interleaved", [False, True])
@pytest.mark.parametrize("emb_dim", [32, 64, 128])
@pytest.mark.parametrize("num_heads", [1, 8])
@pytest.mark.parametrize("seq_len", [1, 128])
@pytest.mark.parametrize("batch_size", [1, 4])
def test_rope(batch_size, seq_len, num_heads, emb_dim, interleaved, inplace, dtype):
    x = _randn((batch_size, seq_len, num_heads, emb_dim), dtype)
    s, c = O.rope_tables(seq_len, emb_dim, dtype=dtype)
    xd = x.to(DEV)
    got = nt.rotary_position_embedding(xd.clone() if inplace else xd, s.to(DEV), c.to(DEV),
                                       interleaved=interleaved, inplace=inplace)
    tol = {torch.float32: (1e-5, 1e-5), torch.float16: (1e-3, 1e-3), torch.bfloat16: (1.6e-2, 1e-5)}[dtype]
    assert_close(got, _ref_rope(x, s, c, interleaved), tol=tol)


def test_rope_strided_llama():
    # q viewed out of a fused [T, 3*H*D] projection: strides (S*3HD, 3HD, D, 1)
    B, S, H, D = 2, 64, 4, 128
    fused = _randn((B, S, 3 * H * D), torch.bfloat16)
    q = fused[..., : H * D].view(B, S, H, D)
    s, c = O.rope_tables(S, D, base=500000.0, dtype=torch.bfloat16)
    got = nt.rotary_position_embedding(fused.to(DEV)[..., : H * D].view(B, S, H, D), s.to(DEV), c.to(DEV),
                                       interleaved=False)
    assert_close(got, _ref_rope(q, s, c, False))


def test_rope_inplace_aliases():
    x = _randn((2, 16, 2, 64), torch.float32).to(DEV)
    s, c = O.rope_tables(16, 64)
    r = nt.rotary_position_embedding(x, s.to(DEV), c.to(DEV), inplace=True)
    assert r is x
