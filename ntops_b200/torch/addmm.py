"""ntops.torch.addmm drop-in: src/ntops/torch/addmm.py:7-18 (kernel src/ntops/kernels/addmm.py:10-94).

beta * input + alpha * (mat1 @ mat2), fused into the GEMM epilogue (:64-67); the output has
input's dtype (:12).  ``input`` broadcasts to [m, n] as in torch (a bias [n] or [1, n] is read
through a stride-0 view, never materialised).
"""

from ntops_b200.torch._gemm import gemm


def addmm(input, mat1, mat2, *, beta=1, alpha=1, out=None):
    if mat1.ndim != 2 or mat2.ndim != 2:
        raise RuntimeError("addmm: expected 2-D matrices")
    m, k = mat1.shape
    k2, n = mat2.shape
    if k != k2:
        raise RuntimeError(f"addmm: mat1 and mat2 shapes cannot be multiplied ({m}x{k} and {k2}x{n})")
    return gemm(mat1, mat2, input, out, alpha, beta, (m, n), "addmm")
