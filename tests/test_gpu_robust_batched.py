"""BASELINE config 2 (robustness sweep at the 27B shapes), the exact power-of-2 scale invariance, and orth_batched:
batch-independent bits, every batched entry point, mixed shapes, and (with 2+ GPUs) the multi-rank path over NCCL."""
import os
import socket

import numpy as np
import pytest
import torch

from spanqr_b200 import orth, orth_batched, zdust, workspace, _lib
from tests import cases, metrics

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("K", [5120, 17408])
def test_robustness_sweep(K):
    for name in cases.CFG2_CASES:
        X = cases.cfg2(K, name)
        ev = metrics.evaluate(orth(X.cuda()), X)
        assert ev["finite"] and ev["bad_cols"] == 0, (K, name, ev)
        assert ev["orth"] <= 2e-7, (K, name, ev)
        assert ev["span_n"] <= 100, (K, name, ev)


@pytest.mark.parametrize("K", [5120, 17408])
def test_pow2_scaling_is_exact(K):
    """Q(2^83 X) and Q(2^-83 X) equal Q(X) bit for bit: the scale is an exact power of 2 applied on load"""
    Q = orth(cases.cfg2(K, "base83").cuda())
    for name in ("scale_p83", "scale_m83"):
        assert torch.equal(orth(cases.cfg2(K, name).cuda()).view(torch.int32), Q.view(torch.int32)), name


def _bits(a, b):
    return torch.equal(a.contiguous().view(torch.int32), b.contiguous().view(torch.int32))


def test_batched_equals_single_bitwise():
    Xs = [cases.cfg3_matrix(i, K=1024).cuda() for i in range(13)]
    single = [orth(x) for x in Xs]
    for got in (orth_batched(Xs), list(orth_batched(torch.stack(Xs)).unbind(0))):
        assert all(_bits(a, b) for a, b in zip(got, single))


def test_batched_split_over_streams_equals_single_bitwise():
    """a group large enough to run in parts on several streams gives every matrix the bits of a lone orth"""
    from spanqr_b200 import batched
    Xs = [cases.cfg3_matrix(i, K=640).cuda() for i in range(batched.SPLIT_MIN + 5)]
    single = [orth(x) for x in Xs]
    got = orth_batched(Xs)
    torch.cuda.synchronize()
    assert all(_bits(a, b) for a, b in zip(got, single))


def test_host_inputs_pipelined_match_device_bitwise():
    """CPU inputs: copies in, kernels and copies out overlapped chunk by chunk; same bits as the device path"""
    Xs = [cases.cfg3_matrix(i, K=1024).pin_memory() for i in range(11)]
    Xs.append(cases.make_case(768, 512, "mixed_c6").pin_memory())
    want = [orth(x.cuda()).cpu() for x in Xs]
    out = [torch.full(x.shape, float("nan")).pin_memory() for x in Xs]
    for chunks in (1, 3, 8):
        got = orth_batched(Xs, out=out, chunks=chunks)
        torch.cuda.synchronize()
        assert all(g is o for g, o in zip(got, out))
        assert all(not g.is_cuda and _bits(g, w) for g, w in zip(got, want)), chunks
    got = orth_batched([x.clone() for x in Xs])   # unpinned inputs, outputs allocated by the call
    torch.cuda.synchronize()
    assert all(_bits(g, w) for g, w in zip(got, want))


def test_batched_mixed_shapes():
    Xs = [cases.cfg4_matrix(i, n_small=3, K_small=1024, K_big=2048, N=512).cuda() for i in range(5)]
    Xs.append(cases.make_case(768, 512, "mixed_c6").cuda())
    got = orth_batched(Xs)
    for x, q in zip(Xs, got):
        assert q.shape == x.shape and _bits(q, orth(x))


def test_mixed_height_entry_point():
    """spanqr_orth_mixed_f32: one call over matrices of two heights, interleaved; each gets its lone orth bits"""
    import ctypes
    r = 256
    Xs = [cases.cfg3_matrix(i, K=(1024 if i % 2 else 640), r=r).cuda() for i in range(7)]
    want = [orth(x) for x in Xs]
    Qs = [torch.empty_like(x) for x in Xs]
    B = len(Xs)
    Ks = (ctypes.c_int * B)(*[x.shape[0] for x in Xs])
    Zs = [zdust(x.shape[0], r, x.device) for x in Xs]
    P = ctypes.c_void_p * B
    hx, hq, hz = P(*[x.data_ptr() for x in Xs]), P(*[q.data_ptr() for q in Qs]), P(*[z.data_ptr() for z in Zs])
    need = ctypes.c_size_t(0)
    L = _lib.lib()
    _lib.check(L.spanqr_workspace_bytes_mixed(ctypes.cast(Ks, ctypes.c_void_p), r, B, ctypes.byref(need)), "ws")
    assert need.value >= _lib.workspace_bytes(1024, r, 3) + _lib.workspace_bytes(640, r, 4)
    ws = torch.empty(need.value, dtype=torch.uint8, device="cuda")
    _lib.check(L.spanqr_orth_mixed_f32(ctypes.cast(hx, ctypes.c_void_p), ctypes.cast(hq, ctypes.c_void_p),
                                       ctypes.cast(Ks, ctypes.c_void_p), r, B, ctypes.cast(hz, ctypes.c_void_p),
                                       ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream), "mixed")
    torch.cuda.synchronize()
    assert all(_bits(q, w) for q, w in zip(Qs, want))


def test_strided_and_device_pointer_entry_points():
    B, K, r = 4, 512, 128
    X = torch.stack([cases.cfg3_matrix(i, K=K, r=r) for i in range(B)]).cuda()
    want = torch.stack([orth(X[b]) for b in range(B)])
    Z = zdust(K, r, X.device)
    st = torch.cuda.current_stream().cuda_stream
    ws = workspace(X.device, K, r, B)
    Q = torch.empty_like(X)
    _lib.check(_lib.lib().spanqr_orth_strided_f32(X.data_ptr(), r, K * r, Q.data_ptr(), r, K * r, K, r, B,
                                                  Z.data_ptr(), ws.data_ptr(), ws.numel(), st), "strided")
    assert _bits(Q, want)
    Q2 = torch.empty_like(X)
    dX = torch.tensor([X[b].data_ptr() for b in range(B)], dtype=torch.int64, device=X.device)
    dQ = torch.tensor([Q2[b].data_ptr() for b in range(B)], dtype=torch.int64, device=X.device)
    _lib.check(_lib.lib().spanqr_orth_batched_f32(dX.data_ptr(), dQ.data_ptr(), K, r, B, Z.data_ptr(), ws.data_ptr(),
                                                  ws.numel(), st), "batched")
    assert _bits(Q2, want)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    from datetime import timedelta
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from spanqr_b200 import batched
        Xs = [cases.cfg4_matrix(i, n_small=6, K_small=1024, K_big=2048, N=512).cuda() for i in range(12)]
        runs = []
        # peer pulls: first call maps the slabs, the second (larger) regrows them, the third reuses them
        for n in (9, 12, 9):
            Qs = orth_batched(Xs[:n])
            torch.cuda.synchronize()
            runs.append(("peer", batched.exchange_mode(), [x.cpu() for x in Qs]))
        batched.EXCHANGE = "nccl"
        Qs = orth_batched(Xs[:9])
        torch.cuda.synchronize()
        runs.append(("nccl", batched.exchange_mode(), [x.cpu() for x in Qs]))
        q.put((rank, runs))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_multi_gpu_matches_single_gpu_bitwise():
    """2 ranks, every result with the single-GPU bits: through the peer-pull exchange (slabs mapped, regrown for a
    larger batch, reused) and through the NCCL all-gather"""
    import torch.multiprocessing as mp
    Xs = [cases.cfg4_matrix(i, n_small=6, K_small=1024, K_big=2048, N=512).cuda() for i in range(12)]
    want = [orth(x).cpu() for x in Xs]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    for rank in range(2):
        for mode, used, Qs in res[rank]:
            assert used == mode, (rank, mode, used)
            assert len(Qs) in (9, 12)
            assert all(_bits(a, b) for a, b in zip(Qs, want)), (rank, mode, len(Qs))


def test_concurrent_streams_bitwise_stress():
    """48 matrices at the batched shape, orth'd one per call on 12 streams at once (60 rounds) and in 3 waves of
    4 parts on stream-priority levels (20 rounds): every result has the bits of a serial run.  Guards the ordering of
    shared-memory reuse between generic loads and TMA writes, which broke about one call in a thousand under load."""
    from spanqr_b200 import batched
    Xs = [cases.cfg3_matrix(i).cuda() for i in range(48)]
    K, r = Xs[0].shape
    Z = zdust(K, r, Xs[0].device)
    cur = torch.cuda.current_stream()
    ws = [torch.empty(_lib.workspace_bytes(K, r, 1), dtype=torch.uint8, device="cuda") for _ in Xs]
    Qs = [torch.empty(K, r, device="cuda") for _ in Xs]

    def one(i, st):
        _lib.check(_lib.lib().spanqr_orth_f32(Xs[i].data_ptr(), r, Qs[i].data_ptr(), r, K, r, Z.data_ptr(),
                                              ws[i].data_ptr(), ws[i].numel(), st.cuda_stream), "orth")

    def serial():
        for i in range(len(Xs)):
            one(i, cur)
        torch.cuda.synchronize()
        return [q.clone() for q in Qs]

    want = serial()
    assert all(_bits(a, b) for a, b in zip(serial(), want))
    streams = [torch.cuda.Stream() for _ in range(12)]
    for _ in range(60):
        for k, st in enumerate(streams):
            st.wait_stream(cur)
            for i in range(k, len(Xs), len(streams)):
                one(i, st)
        for st in streams:
            cur.wait_stream(st)
        torch.cuda.synchronize()
        assert all(_bits(a, b) for a, b in zip(Qs, want))
    out = torch.empty(len(Xs), K, r, device="cuda")
    for _ in range(20):
        qv = list(out.unbind(0))
        used = []
        for w in range(3):
            p = batched._wave_priority(w, 3)
            s = batched._wave_stream(out.device, w, 3)
            s.wait_stream(cur)
            with torch.cuda.stream(s):
                batched._run_local(Xs[16 * w:16 * w + 16], qv[16 * w:16 * w + 16], p)
            used.append(s)
        for s in used:
            cur.wait_stream(s)
        torch.cuda.synchronize()
        assert all(_bits(out[i], want[i]) for i in range(len(Xs)))
