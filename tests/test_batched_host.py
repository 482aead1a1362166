"""Host logic of orth_batched: the partition, the output layout, and the multi-rank exchange (gloo ranks on CPU)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from spanqr_b200 import batched
from spanqr_b200.batched import partition, layout, exchange, wave_of, wave_layout, pull_plan


def test_partition_equal_costs_is_contiguous_and_balanced():
    for B, W in [(96, 8), (96, 1), (10, 4), (3, 8), (12, 5)]:
        o = partition([7] * B, W)
        assert o == sorted(o)
        counts = [o.count(q) for q in range(W)]
        assert max(counts) - min(counts) <= 1 and sum(counts) == B


@pytest.mark.parametrize("n,chunks", [(96, 16), (96, 12), (40, 12), (13, 4), (8, 12), (96, 1), (5, 3)])
def test_host_parts_tile_the_batch_in_order(n, chunks):
    """the host path's chunks: consecutive, in index order, none above ceil(n / chunks); with the ramp the first two
    and last two are smaller than the middle ones"""
    idx = list(range(100, 100 + n))
    parts, step = batched._host_parts(idx, chunks)
    assert [i for p in parts for i in p] == idx
    assert step == -(-n // max(1, min(chunks, n))) and all(0 < len(p) <= step for p in parts)
    sizes = [len(p) for p in parts]
    if batched.HOST_RAMP and min(chunks, n) >= batched.HOST_RAMP_MIN and step >= 4 and len(parts) > 4:
        assert sizes[0] < sizes[1] < sizes[2] and sizes[-1] < sizes[-2] < sizes[-3]
    elif min(chunks, n) < batched.HOST_RAMP_MIN:
        assert len(parts) == -(-n // step)   # no ramp: equal parts


def test_default_host_chunks():
    """few chunks of several matrices for a small batch (each chunk costs a kernel-chain latency), HOST_CHUNKS for a
    large one, never more chunks than matrices"""
    d = batched._default_chunks
    assert [d(n) for n in (1, 3, 12, 24, 48, 96, 500)] == [1, 3, 4, 4, 8, 16, 16]


def test_partition_mixed_batch_balances_cost_exactly():
    costs = [6144 * 256] * 256 + [17408 * 256] * 64          # config 4
    o = partition(costs, 8)
    loads = [sum(c for c, q in zip(costs, o) if q == w) for w in range(8)]
    assert len(set(loads)) == 1
    assert partition(costs, 8) == o                          # deterministic


@pytest.mark.parametrize("numels", [[4, 4, 4, 4, 4, 4, 4, 4], [9, 1, 7, 3, 5, 2], [6, 6, 1]])
@pytest.mark.parametrize("world", [2, 3, 8])
def test_pull_plan_tiles_every_wave(numels, world):
    """the peer pulls of all waves together copy every float of the output exactly once, each owner's run from the
    owner that computed it"""
    owner = partition(numels, world)
    wave = wave_of(owner, world, 4)
    offs, bounds = wave_layout(numels, owner, world, wave, 4)
    seen = [None] * bounds[-1][world]
    for b in bounds:
        for q, off, n in pull_plan(b, world):
            assert n > 0
            for k in range(off, off + n):
                assert seen[k] is None
                seen[k] = q
    for i, n in enumerate(numels):
        assert seen[offs[i]:offs[i] + n] == [owner[i]] * n


@pytest.mark.parametrize("world", [2, 3, 8])
def test_pull_plan_staggers_the_owners(world):
    """with every run non-empty, the k-th pull of each rank reads a different owner (a permutation at every k), each
    rank's own run comes last, and each rank's plan covers the same runs as the unordered plan"""
    b = [10 * q for q in range(world + 1)]
    plans = [pull_plan(b, world, r) for r in range(world)]
    for k in range(world):
        assert sorted(p[k][0] for p in plans) == list(range(world))
    for r, p in enumerate(plans):
        assert p[-1][0] == r
        assert sorted(p) == pull_plan(b, world)
    b = [0, 5, 5, 9]                                  # an empty run is skipped, the order kept
    assert [q for q, _, _ in pull_plan(b, 3, 0)] == [2, 0]
    assert [q for q, _, _ in pull_plan(b, 3, 1)] == [2, 0]


def test_peer_slab_cache(monkeypatch):
    """exchange slabs are made once per (device, group), reused while large enough, regrown (old ones released first)
    to at least twice their size, never retried for a group whose mapping failed, and kept apart per group object"""
    from spanqr_b200 import batched
    made = []

    class FakeSlabs:
        def __init__(self, dev, nbytes, group):
            self.nbytes, self.group, self.released = nbytes, group, False
            self.ok = not getattr(group, "fail", False)
            made.append(self)

        def release(self):
            self.released = True

    class Group:
        def __init__(self, fail=False):
            self.fail = fail

    monkeypatch.setattr(batched, "PeerSlabs", FakeSlabs)
    monkeypatch.setattr(batched, "_PEERS", {})
    g1, g2, bad = Group(), Group(), Group(fail=True)
    a = batched._peer_slabs("cuda:0", 1000, g1)
    assert a is made[0] and a.nbytes == 1000
    assert batched._peer_slabs("cuda:0", 800, g1) is a
    b = batched._peer_slabs("cuda:0", 1500, g1)
    assert a.released and b is made[1] and b.nbytes == 2000
    c = batched._peer_slabs("cuda:0", 100, g2)
    assert c is made[2] and c is not b
    assert batched._peer_slabs("cuda:1", 100, g1) is made[3]
    assert batched._peer_slabs("cuda:0", 100, bad) is None
    assert batched._peer_slabs("cuda:0", 100, bad) is None and len(made) == 5


def test_layout_owner_major():
    owner = [1, 0, 1, 0, 2]
    offs, slab, sizes = layout([4, 5, 6, 7, 8], owner, 3)
    assert slab == [0, 12, 22, 30] and sizes == [12, 10, 8]
    assert offs == [12, 0, 16, 5, 22]
    offs, slab, sizes = layout([4, 4], [0, 0], 3)             # empty slabs
    assert slab == [0, 8, 8, 8] and sizes == [8, 0, 0]


def test_wave_of_cuts_each_owner_in_index_order():
    owner = partition([7] * 13, 3)                            # 5, 4, 4 matrices
    wave = wave_of(owner, 3, 2)
    for q in range(3):
        mine = [wave[i] for i in range(13) if owner[i] == q]
        assert mine == sorted(mine) and mine.count(0) == -(-len(mine) // 2)
    assert wave_of([0, 0, 1], 2, 4) == [0, 2, 0]              # fewer matrices than waves


@pytest.mark.parametrize("nwaves", [1, 2, 3])
def test_wave_layout_tiles_the_buffer_wave_then_owner(nwaves):
    numels = [4, 5, 6, 7, 8, 9, 3, 2]
    owner = partition(numels, 3)
    wave = wave_of(owner, 3, nwaves)
    offs, bounds = wave_layout(numels, owner, 3, wave, nwaves)
    cells = sorted((offs[i], offs[i] + numels[i]) for i in range(len(numels)))
    assert cells[0][0] == 0 and cells[-1][1] == sum(numels) == bounds[-1][-1]
    assert all(a[1] == b[0] for a, b in zip(cells, cells[1:]))              # disjoint and gap-free
    for w in range(nwaves):
        assert w == 0 or bounds[w][0] == bounds[w - 1][-1]
        for q in range(3):
            run = sorted(i for i in range(len(numels)) if wave[i] == w and owner[i] == q)
            assert sum(numels[i] for i in run) == bounds[w][q + 1] - bounds[w][q]
            assert [offs[i] for i in run] == sorted(offs[i] for i in run)   # index order inside a run
            assert all(bounds[w][q] <= offs[i] < bounds[w][q + 1] for i in run)


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


def _slab_worker(rank, world, port, what, bad_rank, q):
    """PeerSlabs set-up on gloo ranks with a fake library whose alloc or open fails on `bad_rank`"""
    import contextlib
    import ctypes
    from spanqr_b200 import batched
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    calls = []

    class FakeLib:
        def spanqr_peer_slab_alloc(self, nbytes, ptr, handle):
            if what == "alloc" and rank == bad_rank:
                return 4
            ptr._obj.value = 0x10000 * (rank + 1)
            ctypes.memmove(handle, bytes([rank + 1]) * 8, 8)
            return 0

        def spanqr_peer_slab_open(self, handle, ptr):
            calls.append(("open", handle[0]))
            if what == "open" and rank == bad_rank:
                return 4
            ptr._obj.value = 0x100 * handle[0]
            return 0

        def spanqr_peer_slab_close(self, p):
            calls.append(("close", p))
            return 0

        def spanqr_peer_slab_free(self, p):
            calls.append(("free", p))
            return 0

    try:
        batched._lib.lib = lambda: FakeLib()
        torch.cuda.device = lambda d: contextlib.nullcontext()
        torch.cuda.synchronize = lambda *a: None
        slabs = batched.PeerSlabs(torch.device("cpu"), 1 << 20, None)
        q.put((rank, slabs.ok, calls))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("what,bad_rank", [("open", 1), ("open", 0), ("alloc", 1)])
def test_peer_slabs_fail_together_on_gloo_ranks(what, bad_rank):
    """when one rank cannot allocate or map, every rank gives up the peer exchange: each unmaps what it mapped and
    frees its own slab (after the barrier), and none keeps a mapping"""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_slab_worker, args=(r, 2, port, what, bad_rank, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {r: (ok, calls) for r, ok, calls in (q.get(timeout=120) for _ in procs)}
    for p in procs:
        p.join(timeout=60)
    for r, (ok, calls) in res.items():
        assert ok is False, r
        opened = [c for c in calls if c[0] == "open"]
        closes = [c for c in calls if c[0] == "close"]
        frees = [c for c in calls if c[0] == "free"]
        if what == "alloc":
            assert opened == [] and closes == []                            # nothing mapped once a handle is bad
        else:
            assert opened == [("open", 2 - r)]                              # the other rank's handle
            assert len(closes) == (0 if r == bad_rank else 1)               # what was mapped is unmapped
        assert frees == ([] if what == "alloc" and r == bad_rank else [("free", 0x10000 * (r + 1))])
        assert calls.index(frees[0]) > max((calls.index(c) for c in closes), default=-1) if frees else True


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


def _wave_worker(rank, world, port, numels, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        owner = partition(numels, world)
        wave = wave_of(owner, world, 2)
        offs, bounds = wave_layout(numels, owner, world, wave, 2)
        out = torch.full((bounds[-1][world],), -1.0)
        fill = lambda i: i * 100.0 + torch.arange(numels[i], dtype=torch.float32)
        for i in range(len(numels)):
            if owner[i] == rank:
                out[offs[i]:offs[i] + numels[i]] = fill(i)
        for b in bounds:
            if b[world] > b[0]:
                exchange(out[b[0]:b[world]], [x - b[0] for x in b], [b[p + 1] - b[p] for p in range(world)])
        q.put((rank, all(torch.equal(out[offs[i]:offs[i] + numels[i]], fill(i)) for i in range(len(numels)))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("numels", [[6] * 8, [6, 9, 4, 4, 7, 3, 5]])
def test_wave_exchange_two_gloo_ranks(numels):
    """per-wave exchanges over the wave-major layout leave every rank with every matrix at its offset"""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_wave_worker, args=(r, 2, port, numels, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}
