"""Sharding of the hot path's independent units across the GPUs of one box.

Every workload of the path partitions without any exchange: elementwise ops by flat ranges,
row ops (rms_norm, layer_norm, softmax) by rows, RoPE and the layer chain by sequences,
GEMM by M rows (weights replicated), attention by (batch x head) units with GQA groups kept
together.  One process drives one GPU; the only collectives are the ones below, used outside
the timed region (timing reduction and output gathering for verification).
"""

import torch
import torch.distributed as dist


def shard_range(total, rank, world):
    """Contiguous [start, stop) slice of `total` units owned by `rank` (sizes differ by <= 1)."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} / world {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def attention_units(batch, kv_heads, rank, world):
    """(batch, kv_head) pairs owned by `rank`; a kv head carries its whole GQA group of q heads."""
    units = [(b, h) for b in range(batch) for h in range(kv_heads)]
    s, e = shard_range(len(units), rank, world)
    return units[s:e]


def max_over_ranks(value, device=None):
    """Maximum of a Python float across ranks (the benchmark's timing rule)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_rows(local, device=None):
    """Concatenates every rank's [rows, ...] shard along dim 0 (equal shard sizes), for
    verification only."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return local
    parts = [torch.empty_like(local) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, local.contiguous())
    return torch.cat(parts, 0)
