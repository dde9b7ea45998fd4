"""CPU oracle for the ntops LLM operator hot path — TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the algorithm of each reference operator (the NineToothed
``application`` functions under src/ntops/kernels/ of the ntops project) in float64, so the
CUDA kernels of ``ntops_b200`` can be checked against it.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may import it, and
only as the checker or the timed CPU baseline: the product path (``ntops_b200``) never calls it
and has no CPU fallback.

Pinning.  The reference's kernels cannot execute in this environment: ``ninetoothed``, the
package that turns them into Triton (``pyproject.toml`` requires ``ninetoothed>=0.16.0``), is
not installed and cannot be.  The reference ships no golden vectors or known-answer files; its
own tests (tests/test_<op>.py) define correctness as agreement with PyTorch's implementation
of the same operator within per-dtype tolerances (tests/utils.py:18-23).  This oracle is
therefore pinned against exactly that test oracle — PyTorch's CPU operators — on the reference
tests' own case generators (``tests/test_oracle.py``) and on committed golden fixtures that
PyTorch produced (``tests/golden/``, generator script alongside).  It is not pinned against the
reference's own kernel outputs.
"""

from oracle import ops  # noqa: F401
