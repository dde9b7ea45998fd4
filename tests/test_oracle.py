"""CPU tests: the oracle (oracle/ops.py) against PyTorch's own operators — the oracle the
reference's tests use — on the reference tests' case generators, and against the committed
golden fixtures (tests/golden/golden.pt).  Also checks that a planted mistake in an oracle
function is caught, so these comparisons have teeth."""

import math
import os
import random

import pytest
import torch
import torch.nn.functional as F

import oracle.ops as O
from tests.utils import assert_close, case_id, float_cases, int_cases, randint_full

CASES = float_cases()
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden.pt")


def _randn(shape, dtype):
    return torch.randn(shape).to(dtype)


@pytest.mark.parametrize("case", CASES, ids=case_id)
def test_unary_vs_torch(case):
    shape, dtype = case
    x = _randn(shape, dtype)
    pairs = {
        "exp": torch.exp, "sigmoid": torch.sigmoid, "silu": F.silu, "tanh": torch.tanh, "sin": torch.sin,
        "cos": torch.cos, "neg": torch.neg, "abs": torch.abs, "relu": torch.relu,
    }
    for name, ref in pairs.items():
        assert_close(getattr(O, name)(x), ref(x.double()).to(dtype))
    assert_close(O.gelu(x), F.gelu(x.double()).to(dtype))
    assert_close(O.gelu(x, "tanh"), F.gelu(x.double(), approximate="tanh").to(dtype))


@pytest.mark.parametrize("case", CASES, ids=case_id)
def test_binary_vs_torch(case):
    shape, dtype = case
    a, b = _randn(shape, dtype), _randn(shape, dtype)
    assert_close(O.add(a, b, 0.3), torch.add(a.double(), b.double(), alpha=0.3).to(dtype))
    assert_close(O.mul(a, b), (a.double() * b.double()).to(dtype))
    assert_close(O.div(a, b), (a.double() / b.double()).to(dtype))
    for op in ("eq", "lt", "ge"):
        assert torch.equal(getattr(O, op)(a, b), getattr(torch, op)(a, b))


@pytest.mark.parametrize("case", int_cases(), ids=case_id)
def test_int_vs_torch(case):
    shape, dtype = case
    a, b = randint_full(shape, dtype), randint_full(shape, dtype)
    assert torch.equal(O.bitwise_and(a, b), torch.bitwise_and(a, b))
    assert torch.equal(O.bitwise_or(a, b), torch.bitwise_or(a, b))
    assert torch.equal(O.bitwise_not(a), torch.bitwise_not(a))


@pytest.mark.parametrize("case", CASES, ids=case_id)
def test_rows_vs_torch(case):
    shape, dtype = case
    x = _randn(shape, dtype)
    ns = tuple(shape[-random.randint(1, len(shape)):])
    w, b = _randn(ns, dtype), _randn(ns, dtype)
    assert_close(O.rms_norm(x, ns, w, 1e-5), F.rms_norm(x.double(), ns, w.double(), 1e-5).to(dtype))
    assert_close(O.layer_norm(x, ns, w, b, 1e-5), F.layer_norm(x.double(), ns, w.double(), b.double(), 1e-5).to(dtype))
    dim = random.randint(0, len(shape) - 1)
    assert_close(O.softmax(x, dim), torch.softmax(x.double(), dim).to(dtype))


def test_rms_norm_default_eps_is_finfo():
    x = torch.zeros(3, 8)
    # x = 0 -> y = 0 / sqrt(0 + eps) = 0; with eps=0 it is NaN (0/0)
    assert torch.equal(O.rms_norm(x, 8), torch.zeros(3, 8))
    assert torch.isnan(O.rms_norm(x, 8, eps=0.0)).all()


def test_rope_vs_reference_test_restatement():
    B, S, H, D = 2, 8, 3, 32
    x = torch.randn(B, S, H, D)
    s, c = O.rope_tables(S, D)
    # the reference test's own torch restatement (tests/test_rotary_position_embedding.py:8-29)
    x0, x1 = x[..., : D // 2], x[..., D // 2 :]
    sc, cc = s[None, :, None, :], c[None, :, None, :]
    want = torch.cat((x0 * cc - x1 * sc, x0 * sc + x1 * cc), -1)
    assert_close(O.rotary_position_embedding(x, s, c, interleaved=False), want)
    pw = x.view(B, S, H, D // 2, 2)
    want_i = torch.stack((pw[..., 0] * cc - pw[..., 1] * sc, pw[..., 0] * sc + pw[..., 1] * cc), -1).view(x.shape)
    assert_close(O.rotary_position_embedding(x, s, c, interleaved=True), want_i)


@pytest.mark.parametrize("variant", [0, 1, 2])
@pytest.mark.parametrize("mask", [None, "bool", "float"])
def test_sdpa_vs_torch(variant, mask):
    if mask is not None and variant:
        pytest.skip("mask and causal are exclusive")
    B, Hq, Hkv, Sq, Skv, D = 2, 4, 2, 37, 53, 32
    q, k, v = torch.randn(B, Hq, Sq, D), torch.randn(B, Hkv, Skv, D), torch.randn(B, Hkv, Skv, D)
    m = None
    if mask == "bool":
        m = torch.rand(Sq, Skv) > 0.3
    elif mask == "float":
        m = torch.randn(Sq, Skv)  # finite additive mask: natural-log units, as torch
    got = O.scaled_dot_product_attention(q, k, v, m, variant != 0, 0.2, variant if variant else 1, block=16)
    kk, vv = k.repeat_interleave(2, 1).double(), v.repeat_interleave(2, 1).double()
    if variant == 2:
        tm = torch.ones(Sq, Skv, dtype=torch.bool).tril(diagonal=Skv - Sq)
        want = F.scaled_dot_product_attention(q.double(), kk, vv, attn_mask=tm, scale=0.2)
    else:
        mm = m.double() if (m is not None and m.dtype != torch.bool) else m
        want = F.scaled_dot_product_attention(q.double(), kk, vv, attn_mask=mm, is_causal=variant == 1, scale=0.2)
    assert_close(got, want.float(), tol=(1e-5, 1e-5))


def test_gemm_vs_torch():
    a, b, c = torch.randn(30, 50), torch.randn(50, 20), torch.randn(30, 20)
    assert_close(O.mm(a, b), (a.double() @ b.double()).float())
    assert_close(O.addmm(c, a, b, 0.5, 2.0), torch.addmm(c.double(), a.double(), b.double(), beta=0.5, alpha=2.0).float())


def _run_golden(case, fn_map):
    op = case["op"]
    inp, kw = case["inputs"], case["kwargs"]
    return fn_map[op](*inp, **kw)


ORACLE_FNS = {
    "add": lambda a, b, alpha: O.add(a, b, alpha),
    "mul": O.mul,
    "div": O.div,
    "silu": O.silu,
    "gelu": O.gelu,
    "gelu_tanh": lambda a: O.gelu(a, "tanh"),
    "sigmoid": O.sigmoid,
    "exp": O.exp,
    "clamp": lambda a: O.clamp(a, -1, 1),
    "pow": O.pow,
    "rms_norm": lambda a, w: O.rms_norm(a, (a.shape[-1],), w, 1e-6),
    "layer_norm": lambda a, w, b: O.layer_norm(a, (a.shape[-1],), w, b, 1e-5),
    "softmax": lambda a: O.softmax(a, -1),
    "bitwise_and": O.bitwise_and,
    "bitwise_or": O.bitwise_or,
    "bitwise_not": O.bitwise_not,
    "eq": O.eq,
    "lt": O.lt,
    "rope": lambda x, s, c, interleaved: O.rotary_position_embedding(x, s, c, interleaved),
    "mm": O.mm,
    "addmm": lambda i, x, y: O.addmm(i, x, y, 0.5, 2.0),
    "bmm": O.bmm,
    "sdpa": lambda q, k, v: O.scaled_dot_product_attention(q, k, v),
    "sdpa_causal": lambda q, k, v: O.scaled_dot_product_attention(q, k, v, None, True),
}


def test_golden_fixtures_pin_oracle():
    cases = torch.load(GOLDEN)
    assert len(cases) >= 50
    for case in cases:
        got = _run_golden(case, ORACLE_FNS)
        exp = case["expected"]
        if exp.is_floating_point():
            # both sides are float64 computations rounded once: equal up to one output ulp
            tol = {torch.float32: (2e-6, 2e-6), torch.float16: (1e-3, 1e-3), torch.bfloat16: (8e-3, 1e-5)}[exp.dtype]
            assert_close(got, exp, tol=tol, equal_nan=True)
        else:
            assert torch.equal(got, exp), case["op"]


def test_planted_oracle_mistake_is_caught():
    """A wrong oracle (eps added outside the square root) must fail the golden comparison."""
    cases = [c for c in torch.load(GOLDEN) if c["op"] == "rms_norm" and c["expected"].dtype == torch.float32]

    def wrong_rms(a, w):
        x = a.double()
        return (x / (torch.sqrt((x * x).mean(-1, keepdim=True)) + 0.05) * w.double()).float()

    for case in cases:
        with pytest.raises(AssertionError):
            assert_close(wrong_rms(*case["inputs"]), case["expected"], tol=(2e-6, 2e-6))


def test_philox_oracle_matches_triton_golden():
    # uniforms of Triton's own tl.rand (the reference dropout's random source), produced by
    # tests/golden/make_philox_golden.py with Triton's interpreter: the restatement is bit-exact
    g = torch.load(os.path.join(os.path.dirname(__file__), "golden", "philox_golden.pt"))
    assert len(g["cases"]) >= 5
    for c in g["cases"]:
        got = O.philox_rand(c["seed"], c["offsets"].numpy())
        assert torch.equal(got, c["rand"]), c["seed"]


def test_dropout_oracle_semantics():
    x = torch.randn(1000, dtype=torch.float64)
    y = O.dropout(x, 0.3, 42)
    kept = y != 0
    assert torch.allclose(y[kept], x[kept] / 0.7)
    assert 0.6 < kept.double().mean().item() < 0.8
    r = O.philox_rand(42, range(1000)).double()
    assert torch.equal(kept, (r > 0.3) & (x != 0))
