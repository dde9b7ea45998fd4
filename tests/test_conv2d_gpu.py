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


@pytest.mark.parametrize("dtype", (torch.bfloat16, torch.float32))
def test_conv2d_chunked_workspace(dtype):
    """A workspace that holds the packed weight and two patch matrices: the five images run as
    batched GEMMs of 2, 2 and 1 images (broadcast weight, bias expanded over the batch) and
    match the oracle and the recommended-workspace call; a workspace short of one image is
    refused."""
    import ctypes

    from ntops_b200 import _lib as L

    lib = L.load()
    g = torch.Generator().manual_seed(3)
    n, c, h, w, k, r = 5, 24, 19, 21, 40, 3
    x = torch.randn((n, c, h, w), generator=g).to(dtype)
    wt = (torch.randn((k, c, r, r), generator=g) * 0.2).to(dtype)
    b = torch.randn((k,), generator=g).to(dtype)
    want = O.conv2d(x, wt, b, stride=1, padding=1)
    xd_t, wd_t, bd_t = x.to(DEV), wt.to(DEV), b.to(DEV)
    full = nt.conv2d(xd_t, wd_t, bias=bd_t, stride=1, padding=1)
    params = (ctypes.c_int * 6)(1, 1, 1, 1, 1, 1)
    xd, wd, bd = L.describe(xd_t), L.describe(wd_t), L.describe(bd_t)
    es = x.element_size()
    crs_pad = (c * r * r + 7) // 8 * 8
    pq_pad = (h * w + 7) // 8 * 8
    wbytes = (k * crs_pad * es + 255) // 256 * 256
    ws_bytes = wbytes + 2 * crs_pad * pq_pad * es + 100
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV)
    y = torch.full_like(full, float("nan"))
    yd = L.describe(y)
    rc = lib.ntb_conv2d(ctypes.byref(xd), ctypes.byref(wd), ctypes.byref(bd), ctypes.byref(yd), params,
                        L.PRECISION_IEEE, ctypes.c_void_p(ws.data_ptr()), ws_bytes, None)
    torch.cuda.synchronize()
    assert rc == L.OK
    tol = (1e-5, 1e-5) if dtype == torch.float32 else (2e-2, 2e-2)
    assert_close(y.cpu(), want, tol=tol)
    assert_close(y.cpu(), full.cpu(), tol=tol)
    small = torch.empty(wbytes + crs_pad * pq_pad * es - 16, dtype=torch.uint8, device=DEV)
    rc = lib.ntb_conv2d(ctypes.byref(xd), ctypes.byref(wd), ctypes.byref(bd), ctypes.byref(yd), params,
                        L.PRECISION_IEEE, ctypes.c_void_p(small.data_ptr()), small.numel(), None)
    assert rc == L.ERR_INVALID


def test_conv2d_wide_rows_gather_path():
    """Input rows too wide for the shared-memory staged patch copy (the rows a 256-column range
    needs exceed 48 KB) take the plain gather kernel."""
    g = torch.Generator().manual_seed(4)
    x = torch.randn((2, 2, 16, 4096), generator=g)
    wt = torch.randn((3, 2, 3, 3), generator=g)
    b = torch.randn((3,), generator=g)
    got = nt.conv2d(x.to(DEV), wt.to(DEV), bias=b.to(DEV), stride=4, padding=2, dilation=3)
    assert_close(got, O.conv2d(x, wt, b, stride=4, padding=2, dilation=3), tol=(1e-5, 1e-5))


# 16-bit convolutions with at least 64 input channels run as an implicit GEMM (TMA im2col loads
# of the channels-innermost input): strides, dilations, asymmetric padding, a partial channel
# block (96 = 64 + 32), output channels below / above one 128-row block and not a multiple of it,
# 1x1 and 5x5 filters, one image, a partial last pixel tile.
IMPLICIT_CASES = [
    # n, c, h, w, k, (r, s), stride, padding, dilation
    (2, 64, 28, 28, 128, (3, 3), 1, 1, 1),
    (3, 96, 17, 23, 64, (3, 3), 2, (1, 2), 1),
    (2, 64, 20, 20, 300, (3, 3), 1, 2, 2),
    (1, 128, 14, 14, 256, (1, 1), 1, 0, 1),
    (2, 64, 31, 29, 96, (5, 5), (2, 1), 2, (1, 2)),
    (4, 256, 9, 9, 512, (3, 3), 1, 1, 1),
    (2, 72, 12, 40, 40, (3, 1), (1, 3), (1, 0), (2, 1)),
]


@pytest.mark.parametrize("dtype", (torch.bfloat16, torch.float16))
@pytest.mark.parametrize("case", IMPLICIT_CASES)
def test_conv2d_implicit_gemm(case, dtype):
    n, c, h, w, k, (r, s), stride, padding, dilation = case
    g = torch.Generator().manual_seed(5)
    x = torch.randn((n, c, h, w), generator=g).to(dtype)
    wt = (torch.randn((k, c, r, s), generator=g) * (1.0 / (c * r * s) ** 0.5)).to(dtype)
    b = torch.randn((k,), generator=g).to(dtype)
    got = nt.conv2d(x.to(DEV), wt.to(DEV), bias=b.to(DEV), stride=stride, padding=padding, dilation=dilation)
    want = O.conv2d(x, wt, b, stride=stride, padding=padding, dilation=dilation)
    assert got.shape == want.shape
    assert_close(got, want, tol=(2e-2, 2e-2))


def test_conv2d_implicit_channels_last_input():
    """A channels-last input is read in place (no transposed copy) and matches the NCHW call."""
    g = torch.Generator().manual_seed(6)
    x = torch.randn((3, 64, 15, 15), generator=g).to(torch.bfloat16)
    wt = (torch.randn((128, 64, 3, 3), generator=g) * 0.05).to(torch.bfloat16)
    xd = x.to(DEV)
    xcl = xd.contiguous(memory_format=torch.channels_last)
    got_cl = nt.conv2d(xcl, wt.to(DEV), padding=1)
    got = nt.conv2d(xd, wt.to(DEV), padding=1)
    assert torch.equal(got_cl, got)
    assert_close(got, O.conv2d(x, wt, None, padding=1), tol=(2e-2, 2e-2))
