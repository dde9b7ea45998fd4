"""Parity of the special-math elementwise operators (copysign, nextafter, lcm, rad2deg, frac,
lgamma) against the oracle; nextafter and copysign are bit-exact, lcm is exact."""

import pytest
import torch

import oracle.ops as O
from tests.utils import assert_close, case_id, float_cases

pytestmark = pytest.mark.gpu

nt = pytest.importorskip("ntops_b200.torch") if torch.cuda.is_available() else None
DEV = "cuda"
CASES = float_cases((torch.float32, torch.float16, torch.bfloat16, torch.float64))


@pytest.mark.parametrize("case", CASES, ids=case_id)
def test_copysign_bit_exact(case):
    shape, dtype = case
    a, b = torch.randn(shape).to(dtype), torch.randn(shape).to(dtype)
    b.view(-1)[::5] = -0.0
    assert torch.equal(nt.copysign(a.to(DEV), b.to(DEV)).cpu(), O.copysign(a, b))


@pytest.mark.parametrize("case", CASES, ids=case_id)
def test_nextafter_bit_exact(case):
    shape, dtype = case
    a, b = torch.randn(shape).to(dtype), torch.randn(shape).to(dtype)
    fa = a.view(-1)
    fa[::7] = 0.0
    b.view(-1)[::11] = a.view(-1)[::11]
    got = nt.nextafter(a.to(DEV), b.to(DEV)).cpu()
    want = O.nextafter(a, b)
    assert torch.equal(got, want)


@pytest.mark.parametrize("dtype", [torch.int8, torch.int16, torch.int32, torch.int64])
def test_lcm_exact(dtype):
    a = torch.randint(-60, 60, (3000,), dtype=dtype)
    b = torch.randint(-60, 60, (3000,), dtype=dtype)
    assert torch.equal(nt.lcm(a.to(DEV), b.to(DEV)).cpu(), O.lcm(a, b))


@pytest.mark.parametrize("dtype", [torch.int32, torch.int64])
def test_lcm_wide_values(dtype):
    # magnitudes up to 2^15 / 2^31, shared powers of two, equal operands, +-1 and the type's
    # extremes (whose products wrap as the promoted type's arithmetic does)
    g = torch.Generator().manual_seed(5)
    hi = 1 << 15 if dtype == torch.int32 else 1 << 31
    a = torch.randint(-hi, hi, (20000,), generator=g, dtype=dtype)
    b = torch.randint(-hi, hi, (20000,), generator=g, dtype=dtype)
    b[::5] = a[::5] * 6
    b[1::5] = a[1::5]
    a[2::7] = 1
    b[3::7] = -1
    info = torch.iinfo(dtype)
    a[:4] = torch.tensor([info.max, info.min, info.min, 1 << 20], dtype=dtype)
    b[:4] = torch.tensor([info.max, 2, info.min, 3 << 12], dtype=dtype)
    assert torch.equal(nt.lcm(a.to(DEV), b.to(DEV)).cpu(), O.lcm(a, b))


@pytest.mark.parametrize("case", CASES, ids=case_id)
def test_rad2deg_frac_lgamma(case):
    shape, dtype = case
    x = (torch.randn(shape) * 5).to(dtype)
    assert_close(nt.rad2deg(x.to(DEV)), O.rad2deg(x))
    assert_close(nt.frac(x.to(DEV)), O.frac(x))
    xp = (torch.rand(shape) * 10 + 0.1).to(dtype)
    got = nt.lgamma(xp.to(DEV))
    want = O.lgamma(xp)
    tol = {torch.float32: (1e-5, 1e-5), torch.float64: (1e-10, 1e-10)}.get(dtype)
    assert_close(got, want, tol=tol)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_lgamma_wide_range(dtype):
    # negative non-integers (reflection), points next to the poles and to the zeros at 1 and 2,
    # tiny and huge magnitudes, and the special values
    g = torch.Generator().manual_seed(8)
    parts = [torch.randn(20000, generator=g) * 6,
             torch.exp2(torch.rand(5000, generator=g) * 200 - 100),
             torch.exp2(torch.rand(5000, generator=g) * 120),
             -torch.arange(1, 40).float() + torch.tensor(1e-3).expand(39),
             -torch.arange(1, 40).float() - torch.tensor(1e-3).expand(39),
             1 + torch.linspace(-1e-3, 1e-3, 101), 2 + torch.linspace(-1e-3, 1e-3, 101),
             torch.tensor([0.0, -0.0, -1.0, -7.0, 1.0, 2.0, float("inf"), float("-inf"), float("nan"), 1e-38, 3e36])]
    x = torch.cat(parts).to(dtype)
    got = nt.lgamma(x.to(DEV)).cpu()
    want = O.lgamma(x)
    tol = (1e-5, 1e-5) if dtype == torch.float32 else None
    assert_close(got, want, tol=tol, equal_nan=True)


def test_rad2deg_int_promotes():
    i = torch.arange(-10, 10, dtype=torch.int32)
    assert_close(nt.rad2deg(i.to(DEV)), O.rad2deg(i))
