"""ntops.torch.add drop-in: src/ntops/torch/add.py:7-15 (kernel src/ntops/kernels/add.py:9-10)."""

from ntops_b200.torch.utils import binary


def add(input, other, *, alpha=1, out=None):
    return binary("add", input, other, out=out, alpha=alpha)
