"""``InputPrecisionVariant`` of src/ntops/kernels/mm.py:13-16 (TF32 = 1, IEEE = 2)."""

import enum


class InputPrecisionVariant(enum.IntEnum):
    TF32 = enum.auto()

    IEEE = enum.auto()
