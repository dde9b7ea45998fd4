"""GPU parity at the BASELINE configurations' full sizes, against the fp64 CPU oracle.

The benchmark's numbers come from these sizes, so each configuration is checked where it is
measured, on the benchmark's seeded input distributions:

* C1 rms_norm fp32 [8, 512, 4096]: every element;
* C2 each elementwise op at 2^28 elements: the first and last 64 Ki elements plus 4 Mi sampled
  indices (the oracle is elementwise, so it is evaluated on the gathered inputs); the broadcast
  add [4096, 1] + [1, 65536] in full;
* C4 softmax fp32 [4096, 32768] and layer_norm bf16 [32768, 8192]: every row, in row blocks;
* C5 attention bf16 [8, 32, 8192, 128], causal and not: 4 (batch, head) slices in full;
  addmm bf16 [16384, 8192] x [8192, 8192] + bias: 256 sampled rows, all columns;
* C3 the Llama-3-8B layer chain at 16 x 2048 tokens: one whole sequence through
  oracle/chain.py.

Tolerances are those of tests/utils.py (fp32 1e-5, bf16 1.6e-2 / 1e-5, fp16 1e-2, bit-exact for
integer / bool results); contractions 1e-2 relative with the absolute part scaled to the
output's RMS; attention 2.5e-2 (the reference's 16-bit bound,
tests/test_scaled_dot_product_attention.py:58-63 in the ntops project).
"""

import math

import pytest
import torch

import oracle.chain as OC
import oracle.ops as O
from tests.utils import TOL, assert_close

pytestmark = pytest.mark.gpu

nt = pytest.importorskip("ntops_b200.torch") if torch.cuda.is_available() else None
DEV = "cuda"
N2 = 1 << 28


def _gen(seed):
    return torch.Generator(device=DEV).manual_seed(seed)


def _sample_idx(n, seed, k=1 << 22, edge=1 << 16):
    g = torch.Generator(device=DEV).manual_seed(seed)
    mid = torch.randint(0, n, (k,), generator=g, device=DEV)
    return torch.cat((torch.arange(edge, device=DEV), torch.arange(n - edge, n, device=DEV), mid))


def _rel_close(got, want, rtol, atol_frac):
    """|got - want| <= rtol |want| + atol_frac * rms(want), elementwise (float64 on the CPU)."""
    g, w = got.detach().cpu().double(), want.detach().cpu().double()
    assert g.shape == w.shape
    rms = w.pow(2).mean().sqrt().item()
    err = (g - w).abs()
    bound = rtol * w.abs() + atol_frac * rms
    bad = int((err > bound).sum())
    assert bad == 0, f"{bad} of {err.numel()} elements out of bound; max err / rms {err.max().item() / rms:.4g}"
    assert torch.isfinite(g).all()


# ----------------------------------------------------------------------------- C1 --------
def test_c1_rms_norm_full():
    g = _gen(0)
    x = torch.randn(8, 512, 4096, generator=g, device=DEV)
    w = 1 + 0.1 * torch.randn(4096, generator=g, device=DEV)
    got = nt.rms_norm(x, (4096,), w, 1e-6)
    assert_close(got, O.rms_norm(x.cpu(), (4096,), w.cpu(), 1e-6))


# ----------------------------------------------------------------------------- C2 --------
FLOAT_OPS = ["add", "mul", "div", "silu", "gelu_tanh", "sigmoid", "exp", "clamp", "pow"]


def _c2_gpu(op, a, b, e):
    return {
        "add": lambda: nt.add(a, b), "mul": lambda: nt.mul(a, b), "div": lambda: nt.div(a, b),
        "silu": lambda: nt.silu(a), "gelu_tanh": lambda: nt.gelu(a, approximate="tanh"),
        "sigmoid": lambda: nt.sigmoid(a), "exp": lambda: nt.exp(a), "clamp": lambda: nt.clamp(a, -1, 1),
        "pow": lambda: nt.pow(a, e),
    }[op]()


def _c2_oracle(op, a, b, e):
    return {
        "add": lambda: O.add(a, b), "mul": lambda: O.mul(a, b), "div": lambda: O.div(a, b),
        "silu": lambda: O.silu(a), "gelu_tanh": lambda: O.gelu(a, "tanh"), "sigmoid": lambda: O.sigmoid(a),
        "exp": lambda: O.exp(a), "clamp": lambda: O.clamp(a, -1, 1), "pow": lambda: O.pow(a, e),
    }[op]()


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16], ids=str)
@pytest.mark.parametrize("op", FLOAT_OPS)
def test_c2_float_op_full_size(op, dtype):
    g = _gen(1)
    a = (torch.rand(N2, generator=g, device=DEV) * 8 - 4).to(dtype)
    b = (torch.rand(N2, generator=g, device=DEV) * 8 - 4).to(dtype) if op in ("add", "mul", "div") else None
    e = (torch.rand(N2, generator=g, device=DEV) * 1.5 + 0.5).to(dtype) if op == "pow" else None
    out = _c2_gpu(op, a, b, e)
    assert out.shape == (N2,) and out.dtype == dtype
    idx = _sample_idx(N2, 2)
    pick = (lambda t: None if t is None else t[idx].cpu())
    want = _c2_oracle(op, pick(a), pick(b), pick(e))
    assert_close(out[idx], want, equal_nan=(op == "pow"))
    del a, b, e, out


@pytest.mark.parametrize("op", ["eq", "lt"])
def test_c2_compare_fp16_full_size(op):
    g = _gen(3)
    a = torch.randn(N2, generator=g, device=DEV).to(torch.float16)
    b = torch.randn(N2, generator=g, device=DEV).to(torch.float16)
    b[::5] = a[::5]  # ties, so eq sees both answers
    out = getattr(nt, op)(a, b)
    assert out.dtype == torch.bool
    idx = _sample_idx(N2, 4)
    assert torch.equal(out[idx].cpu(), getattr(O, op)(a[idx].cpu(), b[idx].cpu()))
    # the whole bool tensor against torch's own comparison (bit-exact, computed on the device)
    assert torch.equal(out, getattr(torch, op)(a, b))


@pytest.mark.parametrize("op", ["bitwise_and", "bitwise_or", "bitwise_not"])
def test_c2_bitwise_int32_full_size(op):
    g = _gen(5)
    a = torch.randint(-2**31, 2**31 - 1, (N2,), generator=g, device=DEV, dtype=torch.int32)
    b = torch.randint(-2**31, 2**31 - 1, (N2,), generator=g, device=DEV, dtype=torch.int32)
    out = nt.bitwise_not(a) if op == "bitwise_not" else getattr(nt, op)(a, b)
    idx = _sample_idx(N2, 6)
    want = O.bitwise_not(a[idx].cpu()) if op == "bitwise_not" else getattr(O, op)(a[idx].cpu(), b[idx].cpu())
    assert torch.equal(out[idx].cpu(), want)
    ref = torch.bitwise_not(a) if op == "bitwise_not" else getattr(torch, op)(a, b)
    assert torch.equal(out, ref)


def test_c2_broadcast_add_full():
    g = _gen(7)
    c = torch.randn(4096, 1, generator=g, device=DEV)
    r = torch.randn(1, 65536, generator=g, device=DEV)
    out = nt.add(c, r)
    assert out.shape == (4096, 65536)
    assert_close(out, O.add(c.cpu(), r.cpu()))


# ----------------------------------------------------------------------------- C4 --------
def test_c4_softmax_full():
    g = _gen(8)
    x = torch.randn(4096, 32768, generator=g, device=DEV) * 2
    got = nt.softmax(x, -1).cpu()
    xc = x.cpu()
    del x
    for r in range(0, 4096, 512):
        assert_close(got[r:r + 512], O.softmax(xc[r:r + 512], -1, block=4096))


def test_c4_layer_norm_full():
    g = _gen(9)
    x = torch.randn(32768, 8192, generator=g, device=DEV).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(8192, generator=g, device=DEV)).to(torch.bfloat16)
    b = (0.1 * torch.randn(8192, generator=g, device=DEV)).to(torch.bfloat16)
    got = nt.layer_norm(x, (8192,), w, b, 1e-5).cpu()
    xc, wc, bc = x.cpu(), w.cpu(), b.cpu()
    del x
    for r in range(0, 32768, 2048):
        assert_close(got[r:r + 2048], O.layer_norm(xc[r:r + 2048], (8192,), wc, bc, 1e-5))


# ----------------------------------------------------------------------------- C5 --------
@pytest.mark.parametrize("causal", [False, True], ids=["noncausal", "causal"])
def test_c5_attention_full(causal):
    g = _gen(10)
    shape = (8, 32, 8192, 128)
    q = torch.randn(shape, generator=g, device=DEV).to(torch.bfloat16)
    k = torch.randn(shape, generator=g, device=DEV).to(torch.bfloat16)
    v = torch.randn(shape, generator=g, device=DEV).to(torch.bfloat16)
    out = nt.scaled_dot_product_attention(q, k, v, is_causal=causal, scale=1 / math.sqrt(128))
    assert torch.isfinite(out).all()
    for b, h in ((0, 0), (3, 17), (5, 8), (7, 31)):
        want = O.scaled_dot_product_attention(q[b:b + 1, h:h + 1].cpu(), k[b:b + 1, h:h + 1].cpu(),
                                              v[b:b + 1, h:h + 1].cpu(), None, causal, block=1024)
        assert_close(out[b:b + 1, h:h + 1], want, tol=(2.5e-2, 2.5e-2))


def test_c5_addmm_full():
    g = _gen(11)
    a = torch.randn(16384, 8192, generator=g, device=DEV).to(torch.bfloat16)
    bm = (torch.randn(8192, 8192, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    bias = torch.randn(8192, generator=g, device=DEV).to(torch.bfloat16)
    out = nt.addmm(bias, a, bm)
    rows = torch.randperm(16384, generator=torch.Generator().manual_seed(12))[:256].sort().values
    want = O.addmm(bias.cpu(), a[rows.to(DEV)].cpu(), bm.cpu())
    _rel_close(out[rows.to(DEV)], want, 1e-2, 1e-2)


# ----------------------------------------------------------------------------- C3 --------
def test_c3_layer_chain_full_one_sequence_checked():
    from ntops_b200 import chain

    B, S = 16, 2048
    wts = chain.LayerWeights(DEV, seed=0)
    sin, cos = chain.rope_tables(S, DEV)
    x = torch.randn((B, S, chain.HIDDEN), generator=_gen(13), device=DEV).to(torch.bfloat16)
    got = chain.layer_forward(x, wts, sin, cos)
    assert got.shape == (B, S, chain.HIDDEN) and torch.isfinite(got).all()
    seq = 11
    w_cpu = [t.cpu() for t in wts.tensors()]
    xs = x[seq:seq + 1].cpu()
    want = OC.layer_forward(xs, w_cpu, sin.cpu(), cos.cpu())
    # Intermediates are rounded to bf16 at different points on the two sides: single-element
    # outliers of PyTorch's own bf16 CPU chain reach ~0.04 rms against the same fp64 oracle.
    _rel_close(got[seq:seq + 1], want, 1e-2, 5e-2)
    torch_bf16 = OC.layer_forward_torch_cpu(xs, w_cpu, sin.cpu(), cos.cpu()).double()
    rms = want.double().pow(2).mean().sqrt()
    err_gpu = (got[seq:seq + 1].cpu().double() - want.double()).abs().mean() / rms
    err_torch = (torch_bf16 - want.double()).abs().mean() / rms
    # no less accurate on average than PyTorch computing the same chain in bf16
    assert err_gpu <= 1.25 * err_torch, (float(err_gpu), float(err_torch))


def test_tolerances_are_the_spec():
    assert TOL[torch.float32] == (1e-5, 1e-5)
    assert TOL[torch.float16] == (1e-2, 1e-2)


# ------------------------------------------------------- the other per-op bench lines --------
# The non-BASELINE lines of the benchmark's per-op table, at the sizes they are timed on.


def test_bench_dropout_2p28_bf16():
    """2^28 bf16 elements, p = 0.1: bit-exact to the oracle on the first / last 64 Ki and 4 Mi
    sampled elements (the keep mask is Triton's Philox for the same seed)."""
    import random

    n = 1 << 28
    x = torch.randn(n, generator=_gen(20), device=DEV).to(torch.bfloat16)
    random.seed(77)
    got = nt.dropout(x, 0.1)
    random.seed(77)
    seed = random.randrange(0, 2**31)
    idx = _sample_idx(n, 21)
    r = O.philox_rand(seed, idx.cpu().numpy()).double()
    xs = x[idx].cpu()
    want = O.round_once(torch.where(r > 0.1, xs.double() / 0.9, torch.zeros((), dtype=torch.float64)), torch.bfloat16)
    assert torch.equal(got[idx].cpu(), want)
    kept = (got != 0).sum().item() / n
    assert abs(kept - 0.9) < 1e-3


def test_bench_conv2d_resnet_layer():
    """32 x 256 x 56 x 56 bf16 through 256 3x3 filters (the implicit GEMM): images 0 and 31
    against the oracle; the channels-last input (no transposed copy) gives the same bits."""
    g = _gen(22)
    x = torch.randn((32, 256, 56, 56), generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.randn((256, 256, 3, 3), generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    out = nt.conv2d(x, w, None, 1, 1)
    for n in (0, 31):
        want = O.conv2d(x[n:n + 1].cpu(), w.cpu(), None, stride=1, padding=1)
        _rel_close(out[n:n + 1], want, 1e-2, 1e-2)
    out_cl = nt.conv2d(x.contiguous(memory_format=torch.channels_last), w, None, 1, 1)
    assert torch.equal(out_cl, out)


def test_bench_sdpa_fp32():
    """fp32 attention 2 x 32 x 8192 x 128 (tensor cores through staged fp16 copies): two
    (batch, head) slices against the oracle within the reference's fp32 tolerance (1e-2)."""
    g = _gen(23)
    shape = (2, 32, 8192, 128)
    q, k, v = (torch.randn(shape, generator=g, device=DEV) for _ in range(3))
    for causal in (False, True):
        out = nt.scaled_dot_product_attention(q, k, v, is_causal=causal)
        for b, h in ((0, 3), (1, 30)):
            want = O.scaled_dot_product_attention(q[b:b + 1, h:h + 1].cpu(), k[b:b + 1, h:h + 1].cpu(),
                                                  v[b:b + 1, h:h + 1].cpu(), None, causal, block=1024)
            assert_close(out[b:b + 1, h:h + 1], want, tol=(1e-2, 1e-2))
