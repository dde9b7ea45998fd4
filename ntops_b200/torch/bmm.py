"""ntops.torch.bmm drop-in: src/ntops/torch/bmm.py:7-18 (kernel src/ntops/kernels/bmm.py:8-67)."""

from ntops_b200.torch._gemm import gemm


def bmm(input, mat2, *, out=None):
    if input.ndim != 3 or mat2.ndim != 3:
        raise RuntimeError("bmm: expected 3-D tensors")
    b, m, k = input.shape
    b2, k2, n = mat2.shape
    if b != b2 or k != k2:
        raise RuntimeError(f"bmm: shapes cannot be multiplied ({b}x{m}x{k} and {b2}x{k2}x{n})")
    return gemm(input, mat2, None, out, 1.0, 0.0, (b, m, n), "bmm")
