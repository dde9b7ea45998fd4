"""Kernel-side enums of the reference kept importable at the same paths
(``ntops.kernels.mm.InputPrecisionVariant``, ``ntops.kernels.scaled_dot_product_attention.CausalVariant``).
The kernels themselves are the sm_100a CUDA sources in ``ntops_b200/csrc``."""

from ntops_b200.kernels import mm, scaled_dot_product_attention

__all__ = ["mm", "scaled_dot_product_attention"]
