"""ntops.torch.matmul drop-in: src/ntops/torch/matmul.py:4-18 (2-D -> mm, otherwise bmm)."""

import ntops_b200


def matmul(input, other, *, out=None):
    assert input.ndim in (2, 3) and other.ndim in (2, 3), (
        "Currently, only 2D and 3D tensors are supported."
    )

    if input.ndim == 2 and other.ndim == 2:
        return ntops_b200.torch.mm(input, other, out=out)

    if input.ndim < 3:
        input = input.unsqueeze(0)

    if other.ndim < 3:
        other = other.unsqueeze(0)

    if input.shape[0] != other.shape[0]:
        b = max(input.shape[0], other.shape[0])
        input = input.expand(b, -1, -1)
        other = other.expand(b, -1, -1)

    return ntops_b200.torch.bmm(input, other, out=out)
