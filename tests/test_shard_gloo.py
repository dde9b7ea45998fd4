"""CPU tests of the multi-GPU partitioning and the verification / timing collectives, run as
world_size-2 gloo process groups (no GPU needed)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ntops_b200.shard import attention_units, gather_rows, max_over_ranks, shard_range


def test_shard_range_covers_exactly():
    for total in [0, 1, 7, 16, 32768, 1000003]:
        for world in [1, 2, 3, 4, 8]:
            seen = []
            for r in range(world):
                s, e = shard_range(total, r, world)
                assert 0 <= s <= e <= total
                seen.extend(range(s, e)) if total < 5000 else seen.append((s, e))
            if total < 5000:
                assert seen == list(range(total))
            else:
                assert seen[0][0] == 0 and seen[-1][1] == total
                assert all(seen[i][1] == seen[i + 1][0] for i in range(len(seen) - 1))
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def test_attention_units_keep_gqa_groups():
    units = [u for r in range(8) for u in attention_units(8, 8, r, 8)]
    assert sorted(units) == [(b, h) for b in range(8) for h in range(8)]
    assert len(attention_units(8, 8, 0, 8)) == 8


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rows = 10
        s, e = shard_range(rows, rank, world)
        local = torch.arange(s, e, dtype=torch.float32)[:, None].repeat(1, 3)
        full = gather_rows(local)
        t = max_over_ranks(1.5 + rank)
        q.put((rank, full.tolist(), t))
    finally:
        dist.destroy_process_group()


def test_gather_and_max_over_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, full, t in results:
        assert full == [[float(i)] * 3 for i in range(10)]
        assert t == 2.5
