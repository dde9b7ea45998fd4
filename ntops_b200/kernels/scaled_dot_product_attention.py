"""``CausalVariant`` of src/ntops/kernels/scaled_dot_product_attention.py:12-17
(UPPER_LEFT = 1, LOWER_RIGHT = 2; same meaning as torch.nn.attention.bias.CausalVariant)."""

import enum


class CausalVariant(enum.IntEnum):
    UPPER_LEFT = enum.auto()

    LOWER_RIGHT = enum.auto()
