"""Host logic of orth_batched: the partition, the output layout, and the multi-rank exchange (gloo ranks on CPU)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from spanqr_b200.batched import partition, layout, exchange


def test_partition_equal_costs_is_contiguous_and_balanced():
    for B, W in [(96, 8), (96, 1), (10, 4), (3, 8), (12, 5)]:
        o = partition([7] * B, W)
        assert o == sorted(o)
        counts = [o.count(q) for q in range(W)]
        assert max(counts) - min(counts) <= 1 and sum(counts) == B


def test_partition_mixed_batch_balances_cost_exactly():
    costs = [6144 * 256] * 256 + [17408 * 256] * 64          # config 4
    o = partition(costs, 8)
    loads = [sum(c for c, q in zip(costs, o) if q == w) for w in range(8)]
    assert len(set(loads)) == 1
    assert partition(costs, 8) == o                          # deterministic


def test_layout_owner_major():
    owner = [1, 0, 1, 0, 2]
    offs, slab, sizes = layout([4, 5, 6, 7, 8], owner, 3)
    assert slab == [0, 12, 22, 30] and sizes == [12, 10, 8]
    assert offs == [12, 0, 16, 5, 22]
    offs, slab, sizes = layout([4, 4], [0, 0], 3)             # empty slabs
    assert slab == [0, 8, 8, 8] and sizes == [8, 0, 0]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, sizes_per_rank, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        numels = [n for n in sizes_per_rank]
        owner = list(range(world))
        offs, slab, sizes = layout(numels, owner, world)
        out = torch.full((slab[world],), -1.0)
        out[slab[rank]:slab[rank + 1]] = rank + 0.5 + torch.arange(sizes[rank], dtype=torch.float32)
        exchange(out, slab, sizes)
        want = torch.cat([w + 0.5 + torch.arange(sizes[w], dtype=torch.float32) for w in range(world)])
        q.put((rank, bool(torch.equal(out, want))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("sizes", [[6, 6], [5, 9]])
def test_exchange_two_gloo_ranks(sizes):
    """equal slabs take the all-gather path, unequal ones the per-owner broadcasts"""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, sizes, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}
