"""ntops.torch.mm drop-in: src/ntops/torch/mm.py:7-18 (kernel src/ntops/kernels/mm.py:19-89).

Output [m, n] in the input dtype (:11-12); fp32 uses TF32 tensor cores unless torch's float32
matmul precision is "highest" (src/ntops/torch/utils.py:218-222).
"""

from ntops_b200.torch._gemm import gemm


def mm(input, mat2, *, out=None):
    if input.ndim != 2 or mat2.ndim != 2:
        raise RuntimeError("mm: expected 2-D tensors")
    m, k = input.shape
    k2, n = mat2.shape
    if k != k2:
        raise RuntimeError(f"mm: mat1 and mat2 shapes cannot be multiplied ({m}x{k} and {k2}x{n})")
    return gemm(input, mat2, None, out, 1.0, 0.0, (m, n), "mm")
