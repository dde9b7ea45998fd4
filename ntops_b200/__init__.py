"""ntops_b200 — B200 (sm_100a) implementation of the ntops LLM operator hot path.

``ntops_b200.torch.<op>`` keeps the signatures of ``ntops.torch.<op>`` (src/ntops/torch/__init__.py
in the reference) and runs every operator on hand-written CUDA kernels in ``libntops_b200.so``
through its C ABI (include/ntops_b200.h).  There is no Triton, no code generation and no CPU
fallback: importing fails if the kernel library is missing.
"""

from ntops_b200 import _lib

_lib.load()

from ntops_b200 import kernels, torch  # noqa: E402

__all__ = ["kernels", "torch"]
