"""ntops.torch.sub drop-in: src/ntops/torch/sub.py:7-15 (kernel src/ntops/kernels/sub.py:9-10)."""

from ntops_b200.torch.utils import binary


def sub(input, other, *, alpha=1, out=None):
    return binary("sub", input, other, out=out, alpha=alpha)
