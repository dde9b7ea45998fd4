"""GPU test: the CUDA path against the committed golden fixtures (tests/golden/golden.pt).

The fixtures hold seeded inputs and the outputs PyTorch's CPU operators give for them in
float64 (the oracle the reference's tests compare ntops against; made by
tests/golden/make_golden.py).  tests/test_oracle.py pins oracle/ops.py to the same numbers on
the CPU, so the kernels and the oracle are checked against one fixed set of values.
Tolerances are the ones the other GPU tests use: elementwise / row ops per dtype
(tests/utils.py:TOL), contractions 1e-2 relative for 16-bit and 1e-5 for IEEE fp32, attention
2.5e-2 for 16-bit and 1e-2 for fp32 (the reference's bounds), integer / bool bit-exact.
"""

import os

import pytest
import torch

from tests.utils import GEMM_TOL, TOL, assert_close

pytestmark = pytest.mark.gpu

nt = pytest.importorskip("ntops_b200.torch") if torch.cuda.is_available() else None
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden.pt")
DEV = "cuda"


def _fns():
    return {
        "add": lambda a, b, alpha: nt.add(a, b, alpha=alpha),
        "mul": nt.mul,
        "div": nt.div,
        "silu": nt.silu,
        "gelu": nt.gelu,
        "gelu_tanh": lambda a: nt.gelu(a, approximate="tanh"),
        "sigmoid": nt.sigmoid,
        "exp": nt.exp,
        "clamp": lambda a: nt.clamp(a, -1, 1),
        "pow": nt.pow,
        "rms_norm": lambda a, w: nt.rms_norm(a, (a.shape[-1],), w, 1e-6),
        "layer_norm": lambda a, w, b: nt.layer_norm(a, (a.shape[-1],), w, b, 1e-5),
        "softmax": lambda a: nt.softmax(a, -1),
        "bitwise_and": nt.bitwise_and,
        "bitwise_or": nt.bitwise_or,
        "bitwise_not": nt.bitwise_not,
        "eq": nt.eq,
        "lt": nt.lt,
        "rope": lambda x, s, c, interleaved: nt.rotary_position_embedding(x, s, c, interleaved=interleaved),
        "mm": nt.mm,
        "addmm": lambda i, x, y: nt.addmm(i, x, y, beta=0.5, alpha=2.0),
        "bmm": nt.bmm,
        "sdpa": lambda q, k, v: nt.scaled_dot_product_attention(q, k, v, enable_gqa=True),
        "sdpa_causal": lambda q, k, v: nt.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True),
    }


def _tol(op, dtype):
    if op in ("mm", "addmm", "bmm"):
        return GEMM_TOL[dtype]
    if op.startswith("sdpa"):
        return (1e-2, 1e-2) if dtype == torch.float32 else (2.5e-2, 2.5e-2)
    return TOL[dtype]


def _cases():
    if not os.path.exists(GOLDEN):
        return []
    return torch.load(GOLDEN)


CASES = _cases()


@pytest.mark.parametrize("idx", range(len(CASES)), ids=[f"{c['op']}-{i}" for i, c in enumerate(CASES)])
def test_golden_case_on_gpu(idx):
    case = CASES[idx]
    fns = _fns()
    inputs = [t.to(DEV) if isinstance(t, torch.Tensor) else t for t in case["inputs"]]
    got = fns[case["op"]](*inputs, **case["kwargs"]).cpu()
    exp = case["expected"]
    if exp.is_floating_point():
        assert_close(got, exp, tol=_tol(case["op"], exp.dtype), equal_nan=True)
    else:
        assert got.dtype == exp.dtype and torch.equal(got, exp), case["op"]


def test_golden_fixture_count():
    assert len(CASES) >= 50
