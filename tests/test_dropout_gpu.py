"""Parity of dropout (torch/dropout.py:9-29, kernels/dropout.py:10-11) against the oracle: the
seed is drawn from Python's `random` as the reference does, so seeding `random` reproduces a call
and the keep mask must equal the oracle's Philox mask bit for bit."""

import random

import pytest
import torch

import oracle.ops as O

pytestmark = pytest.mark.gpu

nt = pytest.importorskip("ntops_b200.torch") if torch.cuda.is_available() else None
DEV = "cuda"


def _expected(x, p, py_seed):
    random.seed(py_seed)
    seed = random.randrange(0, 2**31)
    return O.dropout(x, p, seed)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16, torch.float64])
@pytest.mark.parametrize("shape", [(1000,), (37, 129), (4, 3, 256), (1 << 20,)])
@pytest.mark.parametrize("p", [0.1, 0.5, 0.9])
def test_dropout_matches_oracle(shape, dtype, p):
    x = torch.randn(shape, generator=torch.Generator().manual_seed(3)).to(dtype)
    random.seed(1234)
    got = nt.dropout(x.to(DEV), p).cpu()
    want = _expected(x, p, 1234)
    assert torch.equal(got, want)


def test_dropout_keep_rate_and_scale():
    x = torch.ones(1 << 22, device=DEV)
    y = nt.dropout(x, 0.25).cpu()
    keep = (y != 0).double().mean().item()
    assert abs(keep - 0.75) < 2e-3
    assert torch.allclose(y[y != 0], torch.full((1,), 1 / 0.75))


def test_dropout_eval_inplace_and_views():
    x = torch.randn(64, 80, device=DEV)
    y = nt.dropout(x, 0.5, training=False)
    assert torch.equal(y, x) and y.data_ptr() != x.data_ptr()
    assert nt.dropout(x, 0.0) is not x
    z = x.clone()
    random.seed(7)
    r = nt.dropout(z, 0.5, inplace=True)
    assert r is z and torch.equal(z.cpu(), _expected(x.cpu(), 0.5, 7))
    t = x.t()  # non-contiguous: row-major logical order, in place through a copy
    tc = t.clone()
    random.seed(9)
    r = nt.dropout(t, 0.5, inplace=True)
    assert r is t and torch.equal(t.cpu(), _expected(tc.cpu(), 0.5, 9))
