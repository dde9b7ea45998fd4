"""ntops.torch.isnan drop-in: src/ntops/torch/isnan.py:7-11 (kernel src/ntops/kernels/isnan.py:8); returns bool like torch."""

import torch

from ntops_b200.torch.utils import unary


def isnan(input):
    return unary("isnan", input, out_dtype=torch.bool)
