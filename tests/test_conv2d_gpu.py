"""Parity of conv2d against the oracle on the reference test's grid (tests/test_conv2d.py:9-35:
n, c, h, w, k = 2, 3, 112, 112, 4; 1x1 and 3x3 kernels; strides, paddings and dilations as ints
and pairs; fp32 1e-5 and fp16 1e-3) plus bf16 and a wider channel case on the tensor cores."""

import pytest
import torch

import oracle.ops as O
from tests.utils import assert_close

pytestmark = pytest.mark.gpu

nt = pytest.importorskip("ntops_b200.torch") if torch.cuda.is_available() else None
DEV = "cuda"


@pytest.mark.parametrize("dtype, rtol, atol", ((torch.float32, 1e-5, 1e-5), (torch.float16, 1e-3, 1e-3)))
@pytest.mark.parametrize("dilation", (1, 2, (2, 3)))
@pytest.mark.parametrize("padding", (0, 1, (2, 3)))
@pytest.mark.parametrize("stride", (1, 2, (2, 3)))
@pytest.mark.parametrize("r, s", ((1, 1), (3, 3)))
def test_conv2d_reference_grid(r, s, stride, padding, dilation, dtype, rtol, atol):
    g = torch.Generator().manual_seed(0)
    n, c, h, w, k = 2, 3, 112, 112, 4
    x = torch.randn((n, c, h, w), generator=g).to(dtype)
    wt = torch.randn((k, c, r, s), generator=g).to(dtype)
    b = torch.randn((k,), generator=g).to(dtype)
    got = nt.conv2d(x.to(DEV), wt.to(DEV), bias=b.to(DEV), stride=stride, padding=padding, dilation=dilation)
    want = O.conv2d(x, wt, b, stride=stride, padding=padding, dilation=dilation)
    assert got.shape == want.shape
    assert_close(got, want, tol=(rtol, atol))


@pytest.mark.parametrize("dtype", (torch.bfloat16, torch.float16))
@pytest.mark.parametrize("n,c,h,w,k,r,stride,padding", [(2, 64, 28, 28, 128, 3, 1, 1), (1, 32, 17, 23, 48, 5, 2, 2),
                                                         (3, 16, 9, 9, 8, 1, 1, 0)])
def test_conv2d_channels(n, c, h, w, k, r, stride, padding, dtype):
    g = torch.Generator().manual_seed(1)
    x = torch.randn((n, c, h, w), generator=g).to(dtype)
    wt = (torch.randn((k, c, r, r), generator=g) * 0.1).to(dtype)
    got = nt.conv2d(x.to(DEV), wt.to(DEV), stride=stride, padding=padding)
    want = O.conv2d(x, wt, None, stride=stride, padding=padding)
    assert_close(got, want, tol=(2e-2, 2e-2))


def test_conv2d_valid_padding_and_strided_input():
    g = torch.Generator().manual_seed(2)
    x = torch.randn((2, 4, 20, 30), generator=g)
    wt = torch.randn((6, 4, 3, 3), generator=g)
    got = nt.conv2d(x.to(DEV).transpose(2, 3).contiguous().transpose(2, 3), wt.to(DEV), padding="valid")
    assert_close(got, O.conv2d(x, wt), tol=(1e-5, 1e-5))
    with pytest.raises(AssertionError):
        nt.conv2d(x.to(DEV), wt.to(DEV), groups=2)
