"""Parity of the fused SwiGLU projection, the fused Q / K / V projection with RoPE, and of the
whole Llama layer chain (fused and unfused) against the CPU oracle, at a small token count."""

import pytest
import torch

import oracle.chain as OC
import oracle.ops as O
from tests.utils import assert_close

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,k,n", [(256, 512, 384), (200, 256, 128), (1000, 1024, 640), (128, 4096, 1024)])
def test_swiglu_linear(m, k, n, dtype):
    from ntops_b200.fused import pack_swiglu_weight, swiglu_linear

    x = torch.randn(m, k).to(dtype)
    wg = (torch.randn(k, n) * 0.05).to(dtype)
    wu = (torch.randn(k, n) * 0.05).to(dtype)
    packed = pack_swiglu_weight(wg.to(DEV), wu.to(DEV))
    ref_packed = torch.stack((wg.view(k, n // 128, 128), wu.view(k, n // 128, 128)), 2).reshape(k, 2 * n)
    assert torch.equal(packed.cpu(), ref_packed)
    got = swiglu_linear(x.to(DEV), packed)
    g64 = x.double() @ wg.double()
    u64 = x.double() @ wu.double()
    want = (g64 / (1 + torch.exp(-g64)) * u64).to(dtype)
    assert_close(got, want, tol=(2e-2, 2e-2))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("batch,seq,k,heads,kv_heads", [(2, 128, 512, 4, 2), (1, 300, 256, 2, 1), (3, 64, 4096, 3, 1)])
def test_qkv_rope_linear(batch, seq, k, heads, kv_heads, dtype):
    from ntops_b200.fused import pack_qkv_weight, qkv_rope_linear

    g = torch.Generator().manual_seed(11)
    hd = 128
    x = torch.randn(batch * seq, k, generator=g).to(dtype)
    wq = (torch.randn(k, heads * hd, generator=g) * 0.05).to(dtype)
    wk = (torch.randn(k, kv_heads * hd, generator=g) * 0.05).to(dtype)
    wv = (torch.randn(k, kv_heads * hd, generator=g) * 0.05).to(dtype)
    sin, cos = O.rope_tables(seq, hd, base=500000.0, dtype=dtype)
    packed = pack_qkv_weight(wq.to(DEV), wk.to(DEV), wv.to(DEV))
    assert torch.equal(packed.cpu(), torch.cat((wq, wk, wv), 1))
    nq, nk = heads * hd, kv_heads * hd
    got = qkv_rope_linear(x.to(DEV), packed, sin.to(DEV), cos.to(DEV), nq + nk).cpu()
    # oracle: fp64 products, RoPE on the unrounded q / k (as the epilogue does), one rounding
    p64 = x.double() @ torch.cat((wq, wk, wv), 1).double()
    q = O.rotary_position_embedding(p64[:, :nq].view(batch, seq, heads, hd), sin, cos, interleaved=False)
    kk = O.rotary_position_embedding(p64[:, nq:nq + nk].view(batch, seq, kv_heads, hd), sin, cos, interleaved=False)
    want = torch.cat((q.reshape(batch * seq, nq), kk.reshape(batch * seq, nk), p64[:, nq + nk:]), 1).to(dtype)
    assert_close(got, want, tol=(2e-2, 2e-2))


@pytest.mark.parametrize("fused", [True, False])
def test_layer_chain_small(fused):
    from ntops_b200 import chain

    B, S = 1, 256
    wts = chain.LayerWeights(DEV, seed=3)
    sin, cos = chain.rope_tables(S, DEV)
    x = torch.randn((B, S, chain.HIDDEN), generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    got = chain.layer_forward(x.to(DEV), wts, sin, cos, fused=fused).cpu()
    w_cpu = [t.cpu() for t in (wts.wq, wts.wk, wts.wv, wts.wo, wts.wg, wts.wu, wts.wd, wts.norm1, wts.norm2)]
    want = OC.layer_forward(x, w_cpu, sin.cpu(), cos.cpu())
    # bf16 intermediates are rounded at different points on the two sides.  Every element is held
    # to |got - want| <= 1e-2 |want| + 5e-2 rms(want) (single-element outliers of PyTorch's own
    # bf16 CPU chain, oracle/chain.py:layer_forward_torch_cpu, reach ~0.04 rms against the same
    # fp64 oracle), the mean error to 1e-2 rms, and the mean error may not exceed 1.25 times that
    # of PyTorch's bf16 chain on the same inputs.
    w64 = want.double()
    rms = w64.pow(2).mean().sqrt().item()
    err = (got.double() - w64).abs()
    bad = int((err > 1e-2 * w64.abs() + 5e-2 * rms).sum())
    assert bad == 0, (bad, err.max().item() / rms)
    assert err.mean().item() < 1e-2 * rms, (err.mean().item(), rms)
    torch_err = (OC.layer_forward_torch_cpu(x, w_cpu, sin.cpu(), cos.cpu()).double() - w64).abs().mean().item()
    assert err.mean().item() <= 1.25 * torch_err, (err.mean().item(), torch_err)
    assert torch.isfinite(got.float()).all()
