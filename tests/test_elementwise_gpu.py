"""Parity of the elementwise operators (CUDA path through the C ABI) against the oracle.

Cases follow the reference tests (tests/test_<op>.py: random shapes from tests/utils.py,
randn inputs, fp32/fp16) plus bf16, integer / bool dtypes, broadcasting, type promotion,
non-contiguous and empty inputs, NaN / inf values, ``out=`` and ``inplace``.
"""

import pytest
import torch

import oracle.ops as O
from tests.utils import TOL, assert_close, case_id, float_cases, int_cases, randint_full

pytestmark = pytest.mark.gpu

nt = pytest.importorskip("ntops_b200.torch") if torch.cuda.is_available() else None
FLOAT_CASES = float_cases()
INT_CASES = int_cases()
DEV = "cuda"


def _randn(shape, dtype):
    return torch.randn(shape, dtype=torch.float32).to(dtype)


UNARY_FLOAT = ["exp", "sigmoid", "silu", "tanh", "sin", "cos", "neg", "abs", "relu"]


@pytest.mark.parametrize("op", UNARY_FLOAT)
@pytest.mark.parametrize("case", FLOAT_CASES, ids=case_id)
def test_unary_float(op, case):
    shape, dtype = case
    x = _randn(shape, dtype)
    got = getattr(nt, op)(x.to(DEV))
    assert_close(got, getattr(O, op)(x))


@pytest.mark.parametrize("approximate", ["none", "tanh"])
@pytest.mark.parametrize("case", FLOAT_CASES, ids=case_id)
def test_gelu(approximate, case):
    shape, dtype = case
    x = _randn(shape, dtype) * 3
    assert_close(nt.gelu(x.to(DEV), approximate=approximate), O.gelu(x, approximate=approximate))


@pytest.mark.parametrize("case", FLOAT_CASES, ids=case_id)
def test_rsqrt(case):
    shape, dtype = case
    x = torch.rand(shape).to(dtype) + 0.05
    assert_close(nt.rsqrt(x.to(DEV)), O.rsqrt(x))


@pytest.mark.parametrize("case", FLOAT_CASES, ids=case_id)
def test_isnan_isinf(case):
    shape, dtype = case
    x = _randn(shape, dtype)
    flat = x.view(-1)
    flat[::7] = float("nan")
    flat[1::11] = float("inf")
    flat[2::13] = float("-inf")
    assert_close(nt.isnan(x.to(DEV)), O.isnan(x))
    assert_close(nt.isinf(x.to(DEV)), O.isinf(x))


@pytest.mark.parametrize("case", FLOAT_CASES, ids=case_id)
def test_add_sub(case):
    shape, dtype = case
    a, b = _randn(shape, dtype), _randn(shape, dtype)
    alpha = 0.7312
    assert_close(nt.add(a.to(DEV), b.to(DEV), alpha=alpha), O.add(a, b, alpha))
    assert_close(nt.sub(a.to(DEV), b.to(DEV), alpha=alpha), O.sub(a, b, alpha))
    assert_close(nt.add(a.to(DEV), b.to(DEV)), O.add(a, b))


@pytest.mark.parametrize("case", FLOAT_CASES, ids=case_id)
def test_mul(case):
    shape, dtype = case
    a, b = _randn(shape, dtype), _randn(shape, dtype)
    assert_close(nt.mul(a.to(DEV), b.to(DEV)), O.mul(a, b))


@pytest.mark.parametrize("rounding_mode", [None, "trunc", "floor"])
@pytest.mark.parametrize("case", FLOAT_CASES, ids=case_id)
def test_div(rounding_mode, case):
    shape, dtype = case
    a, b = _randn(shape, dtype) * 4, _randn(shape, dtype)
    got = nt.div(a.to(DEV), b.to(DEV), rounding_mode=rounding_mode)
    want = O.div(a, b, rounding_mode)
    if rounding_mode is None:
        assert_close(got, want)
    else:
        # integer-valued results: bit-exact against the oracle's exact restatement
        torch.testing.assert_close(got.cpu(), want, rtol=0, atol=0, equal_nan=True)


@pytest.mark.parametrize("rounding_mode", ["trunc", "floor"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16, torch.float64])
def test_div_rounding_edges(rounding_mode, dtype):
    # quotients at and next to integers, signed zeros, mixed signs, zero / inf / nan divisors
    g = torch.Generator().manual_seed(17)
    q = torch.randint(-50, 50, (4000,), generator=g).to(torch.float64)
    b = (torch.rand(4000, generator=g, dtype=torch.float64) * 8 - 4)
    a = q * b
    a[::3] = torch.nextafter(a[::3], torch.full_like(a[::3], float("inf")))
    a[1::3] = torch.nextafter(a[1::3], torch.full_like(a[1::3], float("-inf")))
    special = torch.tensor([0.0, -0.0, 1.0, -1.0, 7.0, -7.0, float("inf"), float("-inf"), float("nan")],
                           dtype=torch.float64)
    a = torch.cat((a, special.repeat_interleave(len(special))))
    b = torch.cat((b, special.repeat(len(special))))
    a, b = a.to(dtype), b.to(dtype)
    got = nt.div(a.to(DEV), b.to(DEV), rounding_mode=rounding_mode).cpu()
    torch.testing.assert_close(got, O.div(a, b, rounding_mode), rtol=0, atol=0, equal_nan=True)


@pytest.mark.parametrize("case", FLOAT_CASES, ids=case_id)
def test_pow(case):
    shape, dtype = case
    a = (torch.rand(shape) * 8 - 4).to(dtype)
    e = (torch.rand(shape) * 1.5 + 0.5).to(dtype)
    assert_close(nt.pow(a.to(DEV), e.to(DEV)), O.pow(a, e), equal_nan=True)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16, torch.float64])
def test_pow_special_values(dtype):
    # every pairing of signed zeros, infinities, NaN, +-1, integer / odd / fractional exponents
    vals = [float("-inf"), -3.0, -2.0, -1.0, -0.5, -0.0, 0.0, 0.5, 1.0, 2.0, 3.0, float("inf"), float("nan")]
    a = torch.tensor(vals, dtype=dtype).repeat_interleave(len(vals))
    e = torch.tensor(vals, dtype=dtype).repeat(len(vals))
    got = nt.pow(a.to(DEV), e.to(DEV)).cpu()
    want = torch.pow(a.double(), e.double()).to(dtype)
    torch.testing.assert_close(got, want, equal_nan=True, rtol=TOL[dtype][0], atol=TOL[dtype][1])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_pow_wide_range(dtype):
    # bases over many octaves and exponents beyond the fast path's |b|, |b log2 a| <= 8 window
    g = torch.Generator().manual_seed(7)
    a = torch.exp2(torch.rand(20000, generator=g) * 40 - 20) * torch.where(torch.rand(20000, generator=g) < 0.3, -1.0, 1.0)
    e = torch.rand(20000, generator=g) * 24 - 12
    e[::4] = torch.round(e[::4])  # integer exponents, with negative bases
    a, e = a.to(dtype), e.to(dtype)
    got = nt.pow(a.to(DEV), e.to(DEV)).cpu()
    want = torch.pow(a.double(), e.double())
    finite = torch.isfinite(want) & (want.abs() < torch.finfo(dtype).max) & (want.abs() > torch.finfo(dtype).tiny)
    torch.testing.assert_close(got[finite].double(), want[finite], rtol=TOL[dtype][0], atol=0)
    assert torch.equal(torch.isnan(got), torch.isnan(want.to(dtype)))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16, torch.int32])
def test_clamp_scalar_edges(dtype):
    if dtype.is_floating_point:
        x = torch.tensor([float("nan"), float("-inf"), float("inf"), -2.0, -1.0, 0.0, 1.0, 2.0], dtype=dtype)
    else:
        x = torch.tensor([-2**31, -5, -1, 0, 1, 5, 2**31 - 1], dtype=dtype)
    for lo, hi in ((-1, 1), (None, 1), (-1, None), (2, 1)):
        got = nt.clamp(x.to(DEV), lo, hi).cpu()
        want = torch.clamp(x, lo, hi)
        torch.testing.assert_close(got, want, equal_nan=True, rtol=0, atol=0)


@pytest.mark.parametrize("op", ["eq", "ne", "lt", "le", "gt", "ge"])
@pytest.mark.parametrize("case", FLOAT_CASES, ids=case_id)
def test_compare_float(op, case):
    shape, dtype = case
    a, b = _randn(shape, dtype), _randn(shape, dtype)
    b.view(-1)[::3] = a.view(-1)[::3]  # exercise equality
    assert_close(getattr(nt, op)(a.to(DEV), b.to(DEV)), getattr(O, op)(a, b))


@pytest.mark.parametrize("case", FLOAT_CASES, ids=case_id)
def test_clamp_tensor(case):
    shape, dtype = case
    x, lo, hi = _randn(shape, dtype), _randn(shape, dtype), _randn(shape, dtype)
    assert_close(nt.clamp(x.to(DEV), lo.to(DEV), hi.to(DEV)), O.clamp(x, lo, hi))
    assert_close(nt.clamp(x.to(DEV), lo.to(DEV)), O.clamp(x, lo, None))
    assert_close(nt.clamp(x.to(DEV), None, hi.to(DEV)), O.clamp(x, None, hi))


@pytest.mark.parametrize("case", FLOAT_CASES, ids=case_id)
def test_clamp_scalar(case):
    shape, dtype = case
    x = _randn(shape, dtype) * 2
    assert_close(nt.clamp(x.to(DEV), -1, 1), O.clamp(x, -1, 1))
    assert_close(nt.clamp(x.to(DEV), min=-0.5), O.clamp(x, -0.5, None))
    assert_close(nt.clamp(x.to(DEV), max=0.25), O.clamp(x, None, 0.25))


# ------------------------------------------------------------------- integer / bool -------
@pytest.mark.parametrize("op", ["bitwise_and", "bitwise_or"])
@pytest.mark.parametrize("case", INT_CASES, ids=case_id)
def test_bitwise_binary(op, case):
    shape, dtype = case
    a, b = randint_full(shape, dtype), randint_full(shape, dtype)
    assert_close(getattr(nt, op)(a.to(DEV), b.to(DEV)), getattr(O, op)(a, b))


@pytest.mark.parametrize("case", INT_CASES, ids=case_id)
def test_bitwise_not(case):
    shape, dtype = case
    a = randint_full(shape, dtype)
    assert_close(nt.bitwise_not(a.to(DEV)), O.bitwise_not(a))


@pytest.mark.parametrize("op", ["eq", "ne", "lt", "le", "gt", "ge"])
@pytest.mark.parametrize("case", INT_CASES, ids=case_id)
def test_compare_int(op, case):
    shape, dtype = case
    a, b = randint_full(shape, dtype), randint_full(shape, dtype)
    b.view(-1)[::3] = a.view(-1)[::3]
    assert_close(getattr(nt, op)(a.to(DEV), b.to(DEV)), getattr(O, op)(a, b))


@pytest.mark.parametrize("dtype", [torch.int8, torch.int16, torch.int32, torch.int64])
def test_int_arith(dtype):
    a = torch.randint(-50, 50, (1000,), dtype=dtype)
    b = torch.randint(1, 20, (1000,), dtype=dtype) * torch.where(torch.rand(1000) > 0.5, 1, -1).to(dtype)
    for op in ("mul",):
        assert_close(getattr(nt, op)(a.to(DEV), b.to(DEV)), getattr(O, op)(a, b))
    assert_close(nt.add(a.to(DEV), b.to(DEV), alpha=2), O.add(a, b, 2))
    assert_close(nt.sub(a.to(DEV), b.to(DEV)), O.sub(a, b))
    assert_close(nt.div(a.to(DEV), b.to(DEV), rounding_mode="floor"), O.div(a, b, "floor"))
    assert_close(nt.div(a.to(DEV), b.to(DEV), rounding_mode="trunc"), O.div(a, b, "trunc"))
    assert_close(nt.neg(a.to(DEV)), O.neg(a))
    assert_close(nt.abs(a.to(DEV)), O.abs(a))
    e = torch.randint(0, 5, (1000,), dtype=dtype)
    base = torch.randint(-3, 4, (1000,), dtype=dtype)
    assert_close(nt.pow(base.to(DEV), e.to(DEV)), O.pow(base, e))


# ----------------------------------------------------------------- layouts / semantics ----
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_broadcast_row_column(dtype):
    a = _randn((256, 1), dtype)
    b = _randn((1, 1024), dtype)
    assert_close(nt.add(a.to(DEV), b.to(DEV)), O.add(a, b))
    c = _randn((3, 1, 40), dtype)
    d = _randn((5, 1), dtype)
    assert_close(nt.mul(c.to(DEV), d.to(DEV)), O.mul(c, d))


def test_scalar_operands_and_promotion():
    a = _randn((33, 17), torch.float16)
    b = _randn((33, 17), torch.float32)
    assert_close(nt.add(a.to(DEV), b.to(DEV)), O.add(a, b))  # fp16 + fp32 -> fp32
    assert_close(nt.mul(a.to(DEV), 2.5), O.mul(a, 2.5))
    assert_close(nt.sub(a.to(DEV), 1), O.sub(a, 1))
    i = torch.randint(-5, 5, (100,), dtype=torch.int32)
    assert_close(nt.div(i.to(DEV), 3), O.div(i, 3))  # true division promotes to float
    assert_close(nt.pow(a.to(DEV), 2.0), O.pow(a, 2.0), equal_nan=True)
    assert_close(nt.exp(i.to(DEV)), O.exp(i))  # integer input of a float op -> float32


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_non_contiguous(dtype):
    a = _randn((64, 96), dtype)
    b = _randn((96, 64), dtype)
    assert_close(nt.add(a.to(DEV), b.to(DEV).t()), O.add(a, b.t()))
    assert_close(nt.silu(a.to(DEV)[:, ::3]), O.silu(a[:, ::3]))
    assert_close(nt.eq(a.to(DEV).t(), b.to(DEV)), O.eq(a.t(), b))


def test_empty_and_zero_dim():
    e = torch.empty((0, 5), device=DEV)
    assert nt.add(e, e).shape == (0, 5)
    assert nt.exp(e).shape == (0, 5)
    s = torch.tensor(1.5)
    assert_close(nt.exp(s.to(DEV)), O.exp(s))
    assert_close(nt.add(s.to(DEV), s.to(DEV)), O.add(s, s))


def test_ragged_sizes():
    # sizes around the vector width and the unroll factor
    for n in [1, 3, 7, 8, 9, 15, 17, 127, 129, 1023, 1025, 4097, 65537]:
        for dtype in (torch.float32, torch.bfloat16, torch.float16):
            a, b = _randn((n,), dtype), _randn((n,), dtype)
            assert_close(nt.mul(a.to(DEV), b.to(DEV)), O.mul(a, b))
            assert_close(nt.silu(a.to(DEV)), O.silu(a))
        ia = randint_full((n,), torch.int32)
        assert_close(nt.bitwise_not(ia.to(DEV)), O.bitwise_not(ia))


def test_misaligned_views():
    a = _randn((1001,), torch.bfloat16)
    b = _randn((1001,), torch.bfloat16)
    got = nt.add(a.to(DEV)[1:], b.to(DEV)[:-1])
    assert_close(got, O.add(a[1:], b[:-1]))


def test_out_and_inplace():
    a, b = _randn((50, 20), torch.float32), _randn((50, 20), torch.float32)
    out = torch.empty((50, 20), device=DEV)
    r = nt.add(a.to(DEV), b.to(DEV), out=out)
    assert r is out
    assert_close(out, O.add(a, b))
    x = a.to(DEV).clone()
    r = nt.relu(x, inplace=True)
    assert r is x
    assert_close(x, O.relu(a))
    x = a.to(DEV).clone()
    nt.silu(x, inplace=True)
    assert_close(x, O.silu(a))
    with pytest.warns(UserWarning):
        out2 = torch.empty((3,), device=DEV)
        nt.mul(a.to(DEV), b.to(DEV), out=out2)
    assert_close(out2, O.mul(a, b))


def test_cpu_tensor_rejected():
    with pytest.raises(RuntimeError, match="CUDA"):
        nt.add(torch.ones(3), torch.ones(3))
