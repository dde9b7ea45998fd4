"""Parity of mm / bmm / addmm / matmul against the oracle (float64 products).

Reference grid: tests/test_mm.py:10-44 (m, n, k in [1, 1024], fp32 / fp16), test_bmm.py,
test_addmm.py (random alpha / beta, full [m, n] input), test_matmul.py.  Added: bf16, sizes
that take the tcgen05 tensor-core path with edge tiles in M, N and K, K-major and MN-major
operands (transposed views), a [n] bias, TF32 mode, and sizes that fall back to the CUDA-core
kernel (rows TMA cannot address).
"""

import random

import pytest
import torch

import oracle.ops as O
from tests.utils import GEMM_TOL, assert_close

pytestmark = pytest.mark.gpu

nt = pytest.importorskip("ntops_b200.torch") if torch.cuda.is_available() else None
DEV = "cuda"


def _randn(shape, dtype):
    return torch.randn(shape).to(dtype)


def _check(got, want, dtype, k):
    rtol, atol = GEMM_TOL[dtype]
    # accumulated error grows with sqrt(k) for 16-bit outputs; scale atol like the values
    if dtype in (torch.float16, torch.bfloat16):
        atol = atol * max(1.0, (k / 64) ** 0.5)
    assert_close(got, want, tol=(rtol, atol))


def _sizes(seed):
    r = random.Random(seed)
    return [(r.randint(1, 1024), r.randint(1, 1024), r.randint(1, 1024)) for _ in range(3)]


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("mnk", _sizes(7))
def test_mm_random(mnk, dtype):
    m, n, k = mnk
    a, b = _randn((m, k), dtype), _randn((k, n), dtype)
    _check(nt.mm(a.to(DEV), b.to(DEV)), O.mm(a, b), dtype, k)


# 128-row problems run on single-SM tiles, larger ones on CTA pairs (256 x 256 tiles over two
# SMs): edge tiles where the second CTA of a pair holds only padding rows (129, 300) or padding
# columns (136), and a problem with more tiles than resident pairs (4096 x 2560).
TC_SHAPES = [(128, 256, 64), (256, 512, 1024), (300, 712, 520), (1000, 136, 2056), (8, 8, 8), (129, 264, 72),
             (4096, 2560, 512)]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", TC_SHAPES)
@pytest.mark.parametrize("majors", ["kk", "kn", "mk", "mn"])
def test_mm_tensor_core(shape, majors, dtype):
    m, n, k = shape
    a = _randn((m, k), dtype) if majors[0] == "k" else _randn((k, m), dtype).t()
    b = _randn((n, k), dtype).t() if majors[1] == "k" else _randn((k, n), dtype)
    ad = a.to(DEV) if majors[0] == "k" else a.t().contiguous().to(DEV).t()
    bd = b.t().contiguous().to(DEV).t() if majors[1] == "k" else b.to(DEV)
    _check(nt.mm(ad, bd), O.mm(a, b), dtype, k)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_bmm(dtype):
    for b_, m, n, k in [(3, 65, 130, 70), (2, 128, 256, 128), (4, 200, 48, 264), (2, 384, 520, 320)]:
        a, bb = _randn((b_, m, k), dtype), _randn((b_, k, n), dtype)
        _check(nt.bmm(a.to(DEV), bb.to(DEV)), O.bmm(a, bb), dtype, k)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("mnk", [(77, 99, 55), (256, 384, 192), (130, 264, 520)])
def test_addmm(mnk, dtype):
    m, n, k = mnk
    inp, x, y = _randn((m, n), dtype), _randn((m, k), dtype), _randn((k, n), dtype)
    beta, alpha = 0.61, -1.37
    _check(nt.addmm(inp.to(DEV), x.to(DEV), y.to(DEV), beta=beta, alpha=alpha),
           O.addmm(inp, x, y, beta, alpha), dtype, k)
    bias = _randn((n,), dtype)
    _check(nt.addmm(bias.to(DEV), x.to(DEV), y.to(DEV)), O.addmm(bias, x, y), dtype, k)


def test_addmm_beta_zero_ignores_nan():
    x, y = _randn((64, 64), torch.bfloat16), _randn((64, 64), torch.bfloat16)
    inp = torch.full((64, 64), float("nan")).to(torch.bfloat16)
    got = nt.addmm(inp.to(DEV), x.to(DEV), y.to(DEV), beta=0)
    assert not torch.isnan(got).any()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_matmul(dtype):
    for sa, sb in [((40, 30), (30, 20)), ((3, 40, 30), (3, 30, 20)), ((40, 32), (2, 32, 24)), ((2, 40, 32), (32, 24))]:
        a, b = _randn(sa, dtype), _randn(sb, dtype)
        _check(nt.matmul(a.to(DEV), b.to(DEV)), O.matmul(a, b), dtype, sa[-1])


def test_tf32_mode():
    m, n, k = 256, 384, 512
    a, b = _randn((m, k), torch.float32), _randn((k, n), torch.float32)
    prev = torch.get_float32_matmul_precision()
    try:
        torch.set_float32_matmul_precision("high")
        got = nt.mm(a.to(DEV), b.to(DEV))
    finally:
        torch.set_float32_matmul_precision(prev)
    # TF32 keeps 10 mantissa bits: relative error ~1e-3 per product, averaged over k terms
    assert_close(got, O.mm(a, b), tol=(2e-2, 5e-2))


def test_k_zero_and_empty():
    a = torch.empty((5, 0), device=DEV)
    b = torch.empty((0, 7), device=DEV)
    assert torch.equal(nt.mm(a, b).cpu(), torch.zeros(5, 7))
    c = torch.randn(5, 7)
    assert_close(nt.addmm(c.to(DEV), a, b, beta=2.0), 2.0 * c)
    assert nt.mm(torch.empty((0, 4), device=DEV), torch.empty((4, 3), device=DEV)).shape == (0, 3)


def test_out_param():
    a, b = _randn((64, 32), torch.bfloat16), _randn((32, 48), torch.bfloat16)
    out = torch.empty((64, 48), dtype=torch.bfloat16, device=DEV)
    r = nt.mm(a.to(DEV), b.to(DEV), out=out)
    assert r is out
    _check(out, O.mm(a, b), torch.bfloat16, 32)
