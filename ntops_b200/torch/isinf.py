"""ntops.torch.isinf drop-in: src/ntops/torch/isinf.py:7-11 (kernel src/ntops/kernels/isinf.py:8-11); returns bool like torch."""

import torch

from ntops_b200.torch.utils import unary


def isinf(input):
    return unary("isinf", input, out_dtype=torch.bool)
