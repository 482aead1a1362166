"""orth_batched: orth of many independent layer matrices at once, on one GPU or spread over the GPUs of one node.

The reference has no batched entry point (batching same-shape layers is named as future work in METHODS.md:90-93,
102-103).  Semantics per matrix equal orth(X): every matrix gets exactly the bits orth would give it, whatever the
batch, the grouping or the number of GPUs (the kernels' arithmetic does not depend on the batch).

Multi-GPU (torch.distributed initialised, one process per GPU): every rank passes the same list of matrices; the
matrices are partitioned by cost K * r with a deterministic greedy (largest first, to the least-loaded rank, ties to
the lower rank); each rank computes its share into its slab of one output buffer laid out owner by owner; then the
slabs are exchanged over NCCL (all_gather_into_tensor when the slabs are equal, else one broadcast per owner), so every
rank returns every Q.  With gather=False each rank returns only its own Qs (None elsewhere).  For a list input each
rank computes its share in WAVES waves (consecutive runs of its matrices), the earlier waves on higher-priority streams,
and the output is laid out wave by wave, owner by owner inside a wave: wave w's exchange, issued on one exchange stream
in wave order, runs while wave w+1 still computes.  By default (EXCHANGE "peer") that exchange needs no SM: each rank's
waves write into its exchange slab (PeerSlabs: one cudaMalloc per rank, mapped into every other rank through CUDA IPC),
a one-element NCCL all-reduce per wave is the barrier that says every owner's run is written, and every rank pulls the
runs into its output with one copy-engine copy per owner over NVLink.  EXCHANGE "nccl" (or slabs that cannot be mapped
on some rank, decided by all ranks together) keeps the all_gather_into_tensor per wave.

Host-resident matrices (CPU tensors, pinned for the copies to overlap): the batch is cut into chunks (HOST_CHUNKS), and
per chunk the copy in (one stream), the orth (HOST_COMPUTE streams in turn) and the copy out (one stream) run on the
current device, through HOST_SLOTS device buffers in turn, so the PCIe transfers in both directions overlap each other
and the kernels.  Results land in `out` (pinned CPU
tensors) or in newly allocated pinned tensors; under torch.distributed each rank computes and returns its own share
(gather=False).
"""
import ctypes
import os

import torch
import torch.distributed as dist

from . import _lib
from .core import check_input, aligned, zdust, workspace, TB, MAX_R


def partition(costs, world):
    """owner rank of each matrix.  Equal costs: contiguous blocks (sizes differ by at most one), so the owner-major
    output order is the index order.  Otherwise: largest cost first, to the least-loaded rank (lowest rank on ties)."""
    B = len(costs)
    if B and all(c == costs[0] for c in costs):
        base, extra = divmod(B, world)
        owner, q, left = [], 0, base + (1 if extra > 0 else 0)
        for i in range(B):
            while left == 0:
                q += 1
                left = base + (1 if q < extra else 0)
            owner.append(q)
            left -= 1
        return owner
    owner = [0] * B
    loads = [0] * world
    for i in sorted(range(B), key=lambda i: (-costs[i], i)):
        w = min(range(world), key=lambda q: (loads[q], q))
        owner[i] = w
        loads[w] += costs[i]
    return owner


def layout(numels, owner, world):
    """offsets of each matrix in the flat output (owner by owner, index order inside a slab), the slab bounds
    slab[q]..slab[q+1] of each owner and the slab sizes"""
    order = sorted(range(len(numels)), key=lambda i: (owner[i], i))
    offs = [0] * len(numels)
    slab = [0] * (world + 1)
    off = 0
    for i in order:
        offs[i] = off
        off += numels[i]
        slab[owner[i] + 1] = off
    for q in range(1, world + 1):
        slab[q] = max(slab[q], slab[q - 1])
    return offs, slab, [slab[q + 1] - slab[q] for q in range(world)]


def wave_of(owner, world, nwaves):
    """wave of each matrix: each owner's matrices, in index order, cut in nwaves consecutive runs whose counts differ by
    at most one (the earlier runs the larger)"""
    wave = [0] * len(owner)
    for q in range(world):
        mine = [i for i, o in enumerate(owner) if o == q]
        for j, i in enumerate(mine):
            wave[i] = j * nwaves // len(mine)
    return wave


def wave_layout(numels, owner, world, wave, nwaves):
    """offsets of each matrix in the flat output laid out wave by wave, owner by owner inside a wave (index order inside
    one owner's run), and each wave's bounds: owner q's run of wave w is bounds[w][q]..bounds[w][q + 1]"""
    seg = [[0] * world for _ in range(nwaves)]
    for i, n in enumerate(numels):
        seg[wave[i]][owner[i]] += n
    bounds, off = [], 0
    for w in range(nwaves):
        b = [off]
        for q in range(world):
            off += seg[w][q]
            b.append(off)
        bounds.append(b)
    pos = [list(b[:world]) for b in bounds]
    offs = [0] * len(numels)
    for i, n in enumerate(numels):
        offs[i] = pos[wave[i]][owner[i]]
        pos[wave[i]][owner[i]] += n
    return offs, bounds


def exchange(out, slab, sizes, group=None):
    """every rank's slab of `out` to every rank: one all-gather when the slabs are equal, else a broadcast per owner"""
    rank = dist.get_rank(group)
    world = len(sizes)
    if all(sz == sizes[0] for sz in sizes):
        dist.all_gather_into_tensor(out, out[slab[rank]:slab[rank + 1]], group=group)
        return
    ranks = dist.get_process_group_ranks(group) if group is not None else list(range(world))
    works = [dist.broadcast(out[slab[q]:slab[q + 1]], src=ranks[q], group=group, async_op=True)
             for q in range(world) if sizes[q] > 0]
    for w in works:
        w.wait()


def pull_plan(b, world, rank=None):
    """the copies of one wave's exchange by peer pulls: (owner, offset, count) per owner with a non-empty run, b the
    wave's bounds (owner q's run is b[q]..b[q + 1] of the flat buffer, in floats).  For `rank` the owners come in the
    order rank + 1, rank + 2, ... (mod world), its own run last: at every position of the sequence the ranks read
    from as many different owners, so no GPU's links serve several readers at once."""
    first = 0 if rank is None else rank + 1
    order = [(first + k) % world for k in range(world)]
    return [(q, b[q], b[q + 1] - b[q]) for q in order if b[q + 1] > b[q]]


EXCHANGE = os.environ.get("SPANQR_EXCHANGE", "peer")   # "peer" or "nccl": the same on every rank
PEER_HANDLE_BYTES = 64  # SPANQR_PEER_HANDLE_BYTES
PULL_STREAMS = 1       # streams the pulls are spread over (owner q on stream q % PULL_STREAMS).  2 B200s, 44 MB per
                       # copy, both ranks at once: one copy-engine copy pulls 590 GB/s, the same bytes cut in 2 / 4 / 8
                       # copies on as many streams 550 / 450 / 380 GB/s (a local copy 1.94 TB/s alone, 0.83 on 4)


class _SlabArray:
    """a device pointer as a __cuda_array_interface__ object: torch.as_tensor wraps it without a copy"""

    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3}


class PeerSlabs:
    """one exchange slab of `nbytes` on every rank of `group`, each mapped into every other rank (CUDA IPC handles
    exchanged with all_gather_object).  Collective: every rank constructs it with the same size.  `ok` is False on
    every rank when any rank could not allocate or map (the caller then uses the NCCL exchange)."""

    def __init__(self, dev, nbytes, group):
        L = _lib.lib()
        self.dev, self.nbytes, self.group = dev, nbytes, group
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.own, self.opened, self.ptrs, self.ok = None, [], None, False
        with torch.cuda.device(dev):
            ptr = ctypes.c_void_p()
            handle = ctypes.create_string_buffer(PEER_HANDLE_BYTES)
            rc = L.spanqr_peer_slab_alloc(nbytes, ctypes.byref(ptr), handle)
            if rc == 0:
                self.own = ptr.value
            handles = [None] * self.world
            dist.all_gather_object(handles, (rc, handle.raw), group=group)
            ok = all(h[0] == 0 for h in handles)
            ptrs = [0] * self.world
            for q in range(self.world):
                if not ok:
                    break
                if q == self.rank:
                    ptrs[q] = self.own
                    continue
                pq = ctypes.c_void_p()
                if L.spanqr_peer_slab_open(handles[q][1], ctypes.byref(pq)) != 0:
                    ok = False
                    break
                self.opened.append(pq.value)
                ptrs[q] = pq.value
            flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
            dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
            self.ok = bool(flag.item())
            if not self.ok:
                self.release()   # every rank reaches this (the MIN above), and unmaps before any owner frees
                return
            self.ptrs = ptrs
            self.local = torch.as_tensor(_SlabArray(self.own, nbytes // 4), device=dev)
            self.flag = torch.zeros(1, dtype=torch.int32, device=dev)
            self.pulls = tuple(torch.cuda.Stream(dev, priority=-3) for _ in range(PULL_STREAMS))

    def release(self):
        """unmap the peers' slabs, then, once every rank has, free this rank's own: collective"""
        L = _lib.lib()
        with torch.cuda.device(self.dev):
            torch.cuda.synchronize(self.dev)
            for p in self.opened:
                L.spanqr_peer_slab_close(p)
            self.opened = []
            dist.barrier(group=self.group)
            if self.own is not None:
                self.local = None
                L.spanqr_peer_slab_free(self.own)
                self.own = None
        self.ok = False

    def pull(self, out, b, after):
        """every owner's run of one wave, from its slab into the same place of `out`, once event `after` is done"""
        L = _lib.lib()
        base = out.data_ptr()
        for q, off, n in pull_plan(b, self.world, self.rank):
            ps = self.pulls[q % len(self.pulls)]
            ps.wait_event(after)
            _lib.check(L.spanqr_peer_copy(base + 4 * off, self.ptrs[q] + 4 * off, 4 * n, ps.cuda_stream),
                       f"pull of rank {q}'s run")


_PEERS = {}


def _peer_slabs(dev, nbytes, group):
    """the exchange slabs of (device, process group), (re)made collectively when absent or too small; None when
    mapping failed on some rank (then, for that group, the NCCL exchange).  The key holds the group object itself
    (WORLD's for None), so a process group created after another was destroyed never finds the old group's slabs."""
    g = group if group is not None else dist.group.WORLD
    key = (str(dev), id(g))
    entry = _PEERS.get(key)
    have = entry[1] if entry is not None and entry[0] is g else None
    if have is False:
        return None
    if have is not None and have.nbytes >= nbytes:
        return have
    if have is not None:
        have.release()
    slabs = PeerSlabs(dev, max(nbytes, 2 * (have.nbytes if have is not None else 0)), group)
    _PEERS[key] = (g, slabs if slabs.ok else False)
    return slabs if slabs.ok else None


_LAST_MODE = {}


def exchange_mode():
    """the exchange the last multi-GPU wave call on the current device used: "peer" or "nccl" (None before one)"""
    return _LAST_MODE.get(str(torch.device("cuda", torch.cuda.current_device())))


def _run_group(Xs, Qs, stream):
    """orth of same-shape matrices Xs -> Qs (lists of contiguous aligned tensors) in one library call"""
    K, r = Xs[0].shape
    dev = Xs[0].device
    B = len(Xs)
    Z = zdust(K, r, dev)
    ws = workspace(dev, K, r, B, stream)
    L = _lib.lib()
    PP = _lib.ctypes.c_void_p * B
    hx = PP(*[x.data_ptr() for x in Xs])
    hq = PP(*[q.data_ptr() for q in Qs])
    _lib.check(L.spanqr_orth_ptrs_f32(_lib.ctypes.cast(hx, _lib.ctypes.c_void_p), _lib.ctypes.cast(hq, _lib.ctypes.c_void_p),
                                      K, r, B, Z.data_ptr(), ws.data_ptr(), ws.numel(), stream.cuda_stream),
               f"orth_batched({B}x{K}x{r})")


SPLIT_MIN = 16   # a shape group of at least this many matrices runs as NSTREAMS parts on as many streams
NSTREAMS = 2      # config 3 on one B200, A/B on one box: 1 part 25.6k, 2 27.2k, 3 27.2k, 4 26.9k, 6 26.6k matrices/s
WAVES = 4        # waves per rank under torch.distributed with gather=True (list inputs); 2 GPUs, config 3:
                 # 3.02 ms per step in one wave, 2.82 in four (2.55 without the gather)
_SIDE = {}


def _side_streams(dev, n, priority=0):
    key = (str(dev), n, priority)
    if key not in _SIDE:
        _SIDE[key] = tuple(torch.cuda.Stream(dev, priority=priority) for _ in range(n))
    return _SIDE[key]


def _wave_priority(w, nwaves):
    """stream priority of wave w: earlier waves higher (more negative), at most three levels above the default; the
    exchange stream (w = -1) the highest, so the collective's kernels take SMs as soon as its wave is done"""
    return -3 if w < 0 else -min(nwaves - 1 - w, 3)


def _wave_stream(dev, w, nwaves):
    key = (str(dev), "wave", w, nwaves)
    if key not in _SIDE:
        _SIDE[key] = torch.cuda.Stream(dev, priority=_wave_priority(w, nwaves))
    return _SIDE[key]


def _run_local(Xs, Qs, priority=0):
    """orth of a list of matrices on this GPU, one library call per shape.  A large same-shape group is cut in
    NSTREAMS parts that run on as many streams: many kernels leave SMs idle (one Cholesky CTA per matrix, partial last
    waves), and the other parts' kernels fill them.  Each matrix's arithmetic does not depend on the grouping."""
    if not Xs:
        return
    dev = Xs[0].device
    stream = torch.cuda.current_stream(dev)
    groups = {}
    for x, q in zip(Xs, Qs):
        groups.setdefault(tuple(x.shape), ([], []))
        groups[tuple(x.shape)][0].append(x)
        groups[tuple(x.shape)][1].append(q)
    for xs, qs in groups.values():
        if len(xs) < SPLIT_MIN:
            _run_group(xs, qs, stream)
            continue
        side = _side_streams(dev, NSTREAMS, priority)
        cuts = [len(xs) * i // NSTREAMS for i in range(NSTREAMS + 1)]
        # The caller's stream waits for every part before this returns, so anything later on it (a free and a reuse
        # of these tensors' memory included) comes after the parts' work: no record_stream, and the output slab's
        # memory block is reused call after call.
        for s, a, b in zip(side, cuts[:-1], cuts[1:]):
            s.wait_stream(stream)
            _run_group(xs[a:b], qs[a:b], s)
        for s in side:
            stream.wait_stream(s)


def _check_host(X, name):
    if not torch.is_tensor(X) or X.dim() != 2 or X.dtype != torch.float32 or X.is_cuda:
        raise TypeError(f"{name} must be a 2-D fp32 CPU tensor")
    K, r = X.shape
    if r % TB or r < TB or r > MAX_R or K < r:
        raise ValueError(f"unsupported shape {K}x{r}: r must be a multiple of {TB} in [{TB}, {MAX_R}] and K >= r")


HOST_SLOTS = 4        # device buffers in flight in the host path
HOST_COMPUTE = 2      # compute streams in the host path (consecutive chunks' kernels overlap)
HOST_RAMP = True      # smaller first and last chunks (batches cut into at least HOST_RAMP_MIN chunks)
HOST_RAMP_MIN = 12
HOST_PER_CHUNK = 6    # default chunking: about this many matrices per chunk, 4 to HOST_CHUNKS chunks


def _default_chunks(n):
    """chunks for n host matrices: every chunk's orth costs a kernel-chain latency (~0.5 ms) on top of its share of
    the work, so small batches (a rank's share of a multi-GPU batch) use few chunks of several matrices and large ones
    HOST_CHUNKS (config-3 shares on one B200: 12 matrices 3.8 -> 1.9 ms as 4 chunks instead of 12, 24 matrices 4.2 ->
    3.1 ms)"""
    return max(1, min(n, HOST_CHUNKS, max(4, n // HOST_PER_CHUNK)))


def _host_parts(idx, chunks):
    """idx cut into consecutive parts of at most ceil(len / chunks) items; with HOST_RAMP (at least HOST_RAMP_MIN
    chunks) the first two parts hold a quarter and a half of that and so do the last two, so that the first kernels
    start, and the last copies out end, sooner (the link is idle in one direction until the first chunk is computed,
    and in the other after the last chunk is copied in)"""
    n = len(idx)
    nch = max(1, min(chunks, n))
    step = -(-n // nch)
    sizes = None
    if HOST_RAMP and nch >= HOST_RAMP_MIN and step >= 4:
        head = [step // 4, step // 2]
        rest = n - 2 * sum(head)
        if rest >= step:
            mid = -(-rest // step)
            sizes = head + [rest // mid + (1 if k < rest % mid else 0) for k in range(mid)] + head[::-1]
    if sizes is None:
        sizes = [min(step, n - k) for k in range(0, n, step)]
    parts, o = [], 0
    for z in sizes:
        parts.append(idx[o:o + z])
        o += z
    return parts, step


def _run_host(Xs, Qs, device, chunks):
    """Qs[i] = orth(Xs[i]) for CPU tensors, copies in and out overlapped with the kernels (see the module docstring):
    chunk k is copied in on one stream, computed on compute stream k % HOST_COMPUTE and copied out on a third, in
    device buffer slot k % HOST_SLOTS"""
    cur = torch.cuda.current_stream(device)
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    s_cmp = [torch.cuda.Stream(device) for _ in range(HOST_COMPUTE)]
    for s in [s_in, s_out] + s_cmp:
        s.wait_stream(cur)
    groups = {}
    for i, x in enumerate(Xs):
        groups.setdefault(tuple(x.shape), []).append(i)
    last = None
    for (K, r), idx in groups.items():
        zdust(K, r, device)   # drawn on the current stream, which every stream here follows
        parts, step = _host_parts(idx, chunks)
        nslot = min(HOST_SLOTS, len(parts))
        din = [torch.empty((step, K, r), dtype=torch.float32, device=device) for _ in range(nslot)]
        dout = [torch.empty((step, K, r), dtype=torch.float32, device=device) for _ in range(nslot)]
        for t in din + dout:
            for s in [s_in, s_out] + s_cmp:
                t.record_stream(s)
        ev_out = []
        for k, part in enumerate(parts):
            slot = k % nslot
            with torch.cuda.stream(s_in):
                if k >= nslot:
                    s_in.wait_event(ev_out[k - nslot])   # chunk k - nslot is copied out: its slot is free
                for j, i in enumerate(part):
                    din[slot][j].copy_(Xs[i], non_blocking=True)
                ev_in = torch.cuda.Event()
                ev_in.record(s_in)
            sc = s_cmp[k % len(s_cmp)]
            with torch.cuda.stream(sc):
                sc.wait_event(ev_in)
                if k >= nslot:
                    sc.wait_event(ev_out[k - nslot])
                _run_group([din[slot][j] for j in range(len(part))], [dout[slot][j] for j in range(len(part))], sc)
                ev_cmp = torch.cuda.Event()
                ev_cmp.record(sc)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_cmp)
                for j, i in enumerate(part):
                    Qs[i].copy_(dout[slot][j], non_blocking=True)
                e = torch.cuda.Event()
                e.record(s_out)
                ev_out.append(e)
        last = ev_out[-1]
    if last is not None:
        cur.wait_event(last)   # work on the caller's stream after this call sees every result


HOST_CHUNKS = 16      # pieces of a host batch: config 3 on one B200, 10.3k matrices/s at 16 with the ramp (10.2k at 12)


def orth_batched(Xs, *, gather=True, group=None, out=None, chunks=None):
    """Q_i = orth(X_i) for every matrix.  Xs: a list of fp32 CUDA [K_i, r_i] tensors on one device, or one
    [B, K, r] tensor.  Returns a list of Qs (a [B, K, r] tensor for a tensor input).  Under torch.distributed the
    work is split across the ranks of `group` (default: the world) and the results all-gathered (gather=True).
    A list of CPU tensors runs on the current CUDA device with the copies overlapped (`chunks` pieces; by default about
    HOST_PER_CHUNK matrices per piece, 4 to HOST_CHUNKS pieces) and returns CPU
    tensors (`out`, if given); under torch.distributed that needs gather=False."""
    if not torch.is_tensor(Xs) and len(Xs) and torch.is_tensor(Xs[0]) and not Xs[0].is_cuda:
        Xs = list(Xs)
        for i, x in enumerate(Xs):
            _check_host(x, f"Xs[{i}]")
        distributed = dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1
        if distributed and gather:
            raise ValueError("CPU inputs under torch.distributed: pass gather=False (each rank gets its own share)")
        world = dist.get_world_size(group) if distributed else 1
        rank = dist.get_rank(group) if distributed else 0
        owner = partition([x.shape[0] * x.shape[1] for x in Xs], world)
        if out is None:
            out = [torch.empty(x.shape, dtype=torch.float32, pin_memory=True) if owner[i] == rank else None
                   for i, x in enumerate(Xs)]
        mine = [i for i in range(len(Xs)) if owner[i] == rank]
        _run_host([Xs[i].contiguous() for i in mine], [out[i] for i in mine], torch.cuda.current_device(),
                  _default_chunks(len(mine)) if chunks is None else chunks)
        return [out[i] if owner[i] == rank else None for i in range(len(Xs))]
    stacked = torch.is_tensor(Xs)
    if stacked:
        if Xs.dim() != 3:
            raise ValueError("a tensor input must be [B, K, r]")
        Xs = list(Xs.unbind(0))
    Xs = list(Xs)
    if stacked and not gather:
        raise ValueError("gather=False needs a list input")
    if not Xs:
        return [] if not stacked else torch.empty(0)
    for i, x in enumerate(Xs):
        check_input(x, f"Xs[{i}]")
    dev = Xs[0].device
    if any(x.device != dev for x in Xs):
        raise ValueError("all matrices must be on one device")
    Xs = [aligned(x) for x in Xs]
    distributed = dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1
    world = dist.get_world_size(group) if distributed else 1
    rank = dist.get_rank(group) if distributed else 0
    owner = partition([x.shape[0] * x.shape[1] for x in Xs], world)
    if distributed and gather and not stacked and WAVES > 1:
        return _waves(Xs, owner, world, rank, group, WAVES)

    offs, slab, sizes = layout([x.numel() for x in Xs], owner, world)
    with torch.cuda.device(dev):
        out = torch.empty(slab[world], dtype=torch.float32, device=dev)
        Qs = [out[offs[i]:offs[i] + Xs[i].numel()].view(Xs[i].shape) for i in range(len(Xs))]
        mine = [i for i in range(len(Xs)) if owner[i] == rank]
        _run_local([Xs[i] for i in mine], [Qs[i] for i in mine])
        if distributed and gather:
            exchange(out, slab, sizes, group)
    if distributed and not gather:
        return [Qs[i] if owner[i] == rank else None for i in range(len(Xs))]
    if stacked:
        # equal shapes give a contiguous partition, so the buffer is already in index order
        return out.view(len(Xs), *Xs[0].shape)
    return Qs


def _waves(Xs, owner, world, rank, group, nwaves):
    """the distributed gather path in waves: wave w of this rank computes on a stream of priority
    _wave_priority(w, nwaves) (parts on side streams of that priority); its exchange is issued on one exchange stream
    that waits for that wave only, so the next waves' kernels overlap it.  All collectives of a call go through that
    one stream in wave order (a collective issued with async_op=False runs on the current stream, and two collectives
    of one communicator must not run at once), and every rank issues those of the non-empty waves in the same order.
    With peer slabs the collective of a wave is a one-element all-reduce (a barrier: when it completes on a rank, every
    rank's wave w kernels, which precede it on their streams, are done) and the pulls follow it on the pull streams;
    one more all-reduce after the last pulls keeps the slabs from being rewritten while a peer still reads them."""
    dev = Xs[0].device
    wave = wave_of(owner, world, nwaves)
    offs, bounds = wave_layout([x.numel() for x in Xs], owner, world, wave, nwaves)
    total = bounds[-1][world]
    with torch.cuda.device(dev):
        if EXCHANGE not in ("peer", "nccl"):
            raise ValueError(f"SPANQR_EXCHANGE / batched.EXCHANGE must be 'peer' or 'nccl', not {EXCHANGE!r}")
        peers = _peer_slabs(dev, 4 * total, group) if EXCHANGE == "peer" else None
        _LAST_MODE[str(dev)] = "nccl" if peers is None else "peer"
        cur = torch.cuda.current_stream(dev)
        out = torch.empty(total, dtype=torch.float32, device=dev)
        Qs = [out[offs[i]:offs[i] + Xs[i].numel()].view(Xs[i].shape) for i in range(len(Xs))]
        # this rank's waves write into its exchange slab (same offsets as `out`) when the peers pull from there
        dst = Qs if peers is None else [peers.local[offs[i]:offs[i] + Xs[i].numel()].view(Xs[i].shape)
                                        if owner[i] == rank else None for i in range(len(Xs))]
        for K, r in {tuple(Xs[i].shape) for i in range(len(Xs)) if owner[i] == rank}:
            zdust(K, r, dev)   # drawn on the caller's stream, which every wave's stream follows
        xs_stream = _wave_stream(dev, -1, nwaves)
        xs_stream.wait_stream(cur)
        used = [xs_stream]
        for w in range(nwaves):
            b = bounds[w]
            if b[world] == b[0]:
                continue   # empty on every rank: the bounds are the same everywhere
            s = _wave_stream(dev, w, nwaves)
            s.wait_stream(cur)
            with torch.cuda.stream(s):
                mine = [i for i in range(len(Xs)) if owner[i] == rank and wave[i] == w]
                _run_local([Xs[i] for i in mine], [dst[i] for i in mine], _wave_priority(w, nwaves))
            used.append(s)
            xs_stream.wait_stream(s)
            with torch.cuda.stream(xs_stream):
                if peers is None:
                    exchange(out[b[0]:b[world]], [x - b[0] for x in b], [b[q + 1] - b[q] for q in range(world)], group)
                else:
                    dist.all_reduce(peers.flag, group=group)   # every owner's run of wave w is in its slab
            if peers is not None:
                peers.pull(out, b, xs_stream.record_event())
        if peers is not None:
            # no rank writes its slab again (its next call's waves follow this call on its stream) while another
            # still pulls from it
            for ps in peers.pulls:
                xs_stream.wait_stream(ps)
            with torch.cuda.stream(xs_stream):
                dist.all_reduce(peers.flag, group=group)
        for s in used:
            cur.wait_stream(s)
    return Qs
