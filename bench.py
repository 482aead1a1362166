"""Benchmark of spanqr_b200's orth_batched (BASELINE metric: batched matrices/s at 1/2/4/8 GPUs).

    python bench.py [--gpus N --steps K --warmup W]           # this implementation, one JSON line on rank 0
    python bench.py --impl reference [...]                     # the reference's CPU path (oracle port), host cores
    torchrun --nproc-per-node N bench.py --gpus N ...          # N GPUs (one rank per GPU, NCCL)

Workload (default): BASELINE config 3, 96 matrices of 3584 x 256 fp32 (Haar-mixed, kappa log-uniform in [1e2, 1e10],
8 exactly rank 192), seeded synthetic inputs of the reference's shapes.  A step is one orth_batched call over the whole
batch (the matrices partitioned over the ranks, results all-gathered over NCCL); total work is fixed as N grows
(strong scaling).  The inputs (352 MB) are larger than L2 (126 MB), so no flush is needed between steps.

`value` is device time (CUDA events, max over ranks) with inputs resident; `e2e` adds each step's host-to-device copy
of the rank's inputs (pinned) and device-to-host copy of its results.  `roofline` is the dominant kernel's achieved
bandwidth (algorithmic bytes per launch / live CUDA-event duration per launch) over the measured HBM copy bandwidth,
with the whole step's fraction beside it.  On one GPU the line also carries `orth_latency`: orth() microseconds per
call at the eight TTF shapes (isolated calls with L2 flushed, and back-to-back bursts, as the reference's
qrbench/bench.py:28-53 times them), with cuSOLVER Householder (torch.linalg.qr) on the same GPU beside each.
`cpu_baseline` (and `--impl reference`) time the reference's pure-PyTorch CPU path (rcholqr, restated in
oracle/rcholqr.py) on the host cores, with LAPACK Householder (torch.linalg.qr) and the C restatement of the GPU
recipe (oracle/spanqr_oracle.c) beside it.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "orth() us/call at KxR (768x512...17408x256); batched matrices/s at 1/2/4/8 GPU"


def parse():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", choices=["cfg3", "cfg4"], default="cfg3")
    ap.add_argument("--batch", type=int, default=None, help="override the batch size (tests / profiling)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-latency", action="store_true", help="skip the per-shape orth() latency block")
    return ap.parse_args()


# ---------------------------------------------------------------------------------------------------------------
# workload

def workload_spec(name, batch=None):
    if name == "cfg3":
        B = batch or 96
        return {"name": "cfg3", "shapes": [(3584, 256)] * B,
                "desc": f"orth_batched config 3: {B} x 3584x256 fp32 (kappa log-uniform 1e2..1e10, 8/96 rank 192)"}
    B_small, B_big = (256, 64) if batch is None else (batch * 4 // 5, batch - batch * 4 // 5)
    return {"name": "cfg4", "shapes": [(6144, 256)] * B_small + [(17408, 256)] * B_big,
            "desc": f"orth_batched config 4: {B_small} x 6144x256 + {B_big} x 17408x256 fp32 TTF form (N 5120)"}


def make_inputs(spec, device):
    from tests import cases
    out = []
    for i, (K, r) in enumerate(spec["shapes"]):
        if spec["name"] == "cfg3":
            out.append(cases.cfg3_matrix(i, K, r).to(device))
        else:
            out.append(_cfg4_on_device(i, K, r, device))
    return out


def _cfg4_on_device(i, K, r, device, N=5120):
    """config 4 member on the GPU (fp64, seeded CUDA generator): X = V (U^T U) + u^T U, V Haar, U columns scaled
    logspace(0, -cu) with cu log-uniform in [1, 4] (kappa(U) in [1e1, 1e4]), u unit-RMS Gaussian"""
    g = torch.Generator(device=device).manual_seed(10_000 + i)
    cu = 1.0 + 3.0 * torch.rand(1, generator=g, device=device, dtype=torch.float64).item()
    Qv, Rv = torch.linalg.qr(torch.randn(K, r, generator=g, device=device, dtype=torch.float64))
    V = Qv * torch.sign(torch.diagonal(Rv))
    U = torch.randn(N, r, generator=g, device=device, dtype=torch.float64) * torch.logspace(
        0, -cu, r, device=device, dtype=torch.float64)
    u = torch.randn(N, K, generator=g, device=device, dtype=torch.float64)
    u = u / u.pow(2).mean().sqrt()
    return (V @ (U.T @ U) + u.T @ U).to(torch.float32)


# ---------------------------------------------------------------------------------------------------------------
# clocks during the timed region

class ClockSampler:
    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, uuids):
        self.uuids = {u.lower() for u in uuids}
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-f", self.path], stdout=subprocess.DEVNULL,
                                         stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        sm, mx, reasons = [], [], set()
        try:
            lines = Path(self.path).read_text().strip().splitlines()
        except (OSError, TypeError):
            lines = []
        for ln in lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 8:
                continue
            uuid = f[0].lower().replace("gpu-", "")
            if self.uuids and not any(uuid.endswith(u.replace("gpu-", "")[-12:]) for u in self.uuids):
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        if self.path:
            try:
                os.unlink(self.path)
            except OSError:
                pass
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------------------------------------------
# measurement helpers

def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def ncu_traffic(kernel):
    """dram bytes per launch of `kernel` recorded in profiles/*.txt lines 'traffic_bytes_per_launch <kernel> <N>'"""
    for p in sorted((ROOT / "profiles").glob("*.txt")):
        for ln in p.read_text().splitlines():
            f = ln.split()
            if len(f) == 3 and f[0] == "traffic_bytes_per_launch" and f[1] == kernel:
                return float(f[2])
    return None


def alg_bytes_per_call(kind, K, r):
    """algorithmic bytes of one orth call of one K x r matrix spent in the launches of one kernel kind (each input
    read once, each output written once): k_trsm: three passes, each reading its input (X or Y) and writing Y (the
    dust Z of pass 1 is one matrix shared by the batch and left out); k_gram_tc: the Grams of passes 1-3 and of the
    first polish step, each reading Y once; k_gram_tc_acc: the last polish step's Gram; k_ns_update: two polish
    updates, each reading and writing Y; k_absmax: one read of X.  Divided by that kind's launches per call it gives
    the bytes per launch and matrix."""
    kr4 = 4.0 * K * r
    return {"k_absmax": kr4, "k_gram_tc": 4 * kr4, "k_gram_tc_acc": kr4, "k_trsm": 3 * 2 * kr4,
            "k_ns_update": 2 * 2 * kr4, "k_gram_reduce": 5 * 4.0 * r * r,
            "k_chol": 3 * 3 * 4.0 * r * r, "k_trsm_w": 3 * 4.0 * r * r, "k_setup": 16.0}.get(kind, 0.0)


def alg_bytes_orth(K, r):
    """the whole orth call's algorithmic bytes, 17 reads or writes of a K x r fp32 matrix (absmax 1, Grams 5, the
    three solves 2 each, the two polish updates 2 each)"""
    return 17 * 4.0 * K * r


def dist_max(x, device):
    if not (dist.is_available() and dist.is_initialized()):
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------------------------------------------
# arms

def _host_sample(K, r, n):
    """n config-3 members (at most 64 distinct matrices, reused beyond that), fp32 CPU tensors"""
    from tests import cases
    distinct = [cases.cfg3_matrix(i, K, r) for i in range(min(n, 64))]
    return [distinct[i % len(distinct)] for i in range(n)]


def _time_cpu(fn, xs, budget_s):
    """matrices/s of fn over the sample xs, one warm-up call, then whole passes over xs for about budget_s seconds"""
    fn(xs[0])
    t = time.perf_counter()
    n = 0
    while True:
        for x in xs:
            fn(x)
        n += len(xs)
        dt = time.perf_counter() - t
        if dt >= budget_s:
            return n / dt, n, dt


def cpu_baselines(K, r, budget_s=8.0):
    """The reference's CPU path on this host's cores, on config-3 members: its pure-PyTorch rcholqr (the value), LAPACK
    Householder torch.linalg.qr and the C restatement of the GPU recipe kcholqr_f (one matrix per OpenMP thread)."""
    import oracle
    from oracle.rcholqr import rcholqr
    th = os.cpu_count() or 1
    prev = torch.get_num_threads()
    torch.set_num_threads(th)
    try:
        xs = _host_sample(K, r, 8)
        v_rc, n_rc, t_rc = _time_cpu(rcholqr, xs, budget_s)
        v_hh, n_hh, t_hh = _time_cpu(lambda x: torch.linalg.qr(x)[0], xs, budget_s / 2)
    finally:
        torch.set_num_threads(prev)
    oth = oracle.num_threads()
    Z = oracle.dust(K, r)
    Xo = [x.numpy() for x in _host_sample(K, r, oth)]
    t = time.perf_counter()
    oracle.orth_batch(Xo, [Z] * oth)
    t_or = time.perf_counter() - t
    return {"value": v_rc, "unit": "matrices/s", "cores": th, "kind": "port",
            "sample": f"rcholqr (reference candidates/rcholqr.py:61-65, restated in oracle/rcholqr.py) on {n_rc} "
                      f"config-3 members of {K}x{r} (8 distinct), torch CPU on {th} threads, {t_rc:.1f} s",
            "householder_cpu": {"value": v_hh, "unit": "matrices/s", "cores": th,
                                "sample": f"torch.linalg.qr(X)[0] (LAPACK) on {n_hh} of the same matrices, {t_hh:.1f} s"},
            "kcholqr_f_port": {"value": oth / t_or, "unit": "matrices/s", "cores": oth,
                               "sample": f"the C restatement of kcholqr_f (oracle/spanqr_oracle.c) on {oth} matrices, "
                                         f"one per OpenMP thread, {t_or:.1f} s"}}


def run_reference(a, spec):
    """--impl reference: the reference's CPU path on the host cores -- its pure-PyTorch rcholqr (restated in
    oracle/rcholqr.py; the reference's GPU path needs Triton and NVRTC on a GPU and has no CPU form), torch on every
    host thread, one step = one pass over a sample of config-3 members; LAPACK Householder timed beside it"""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from oracle.rcholqr import rcholqr
    K, r = spec["shapes"][0]
    th = os.cpu_count() or 1
    torch.set_num_threads(th)
    xs = _host_sample(K, r, 8)
    for _ in range(a.warmup):
        for x in xs:
            rcholqr(x)
    t = time.perf_counter()
    for _ in range(a.steps):
        for x in xs:
            rcholqr(x)
    dt = time.perf_counter() - t
    v = len(xs) * a.steps / dt
    v_hh, n_hh, t_hh = _time_cpu(lambda x: torch.linalg.qr(x)[0], xs, 4.0)
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "matrices/s", "n_gpus": a.gpus,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": 1e3 * dt / a.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": spec["desc"] + f"; each step a host sample of {len(xs)} of its matrices"},
            "cpu_baseline": {"value": v, "unit": "matrices/s", "cores": th, "kind": "port",
                             "sample": f"rcholqr (reference candidates/rcholqr.py:61-65, restated in oracle/rcholqr.py)"
                                       f", {len(xs)} config-3 members of {K}x{r} per step, torch CPU on {th} threads",
                             "householder_cpu": {"value": v_hh, "unit": "matrices/s", "cores": th,
                                                 "sample": f"torch.linalg.qr(X)[0] on {n_hh} of the same matrices"}},
            "e2e": {"value": v, "unit": "matrices/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


TTF_SHAPES = [(768, 512), (2048, 512), (1024, 256), (2048, 256), (3584, 256), (5120, 256), (6144, 256), (17408, 256)]


def _time_calls(fn, X, flush, reps=20, bursts=5, burst=20):
    """(lat, thr) in microseconds, medians of CUDA-event times as the reference's qrbench/bench.py:28-53 takes them:
    lat = one call, synchronised before and after, L2 flushed before each (a write of 2x L2); thr = a burst of calls
    back to back, per call"""
    for _ in range(5):
        fn(X)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    lat = []
    for _ in range(reps):
        flush.zero_()
        torch.cuda.synchronize()
        s.record()
        fn(X)
        e.record()
        torch.cuda.synchronize()
        lat.append(s.elapsed_time(e) * 1e3)
    thr = []
    for _ in range(bursts):
        torch.cuda.synchronize()
        s.record()
        for _ in range(burst):
            fn(X)
        e.record()
        torch.cuda.synchronize()
        thr.append(s.elapsed_time(e) * 1e3 / burst)
    return statistics.median(lat), statistics.median(thr)


def orth_latency(device, hbm):
    """orth() per call at the TTF shapes on the reference bench's default case (ttf_cu4_t1e-2), with cuSOLVER
    Householder (torch.linalg.qr, the reference's "householder" method, qrbench/methods.py) on the same GPU"""
    from spanqr_b200 import orth
    from tests import cases
    flush = torch.empty(2 * 126 * 2 ** 20, dtype=torch.uint8, device=device)
    rows = []
    for K, r in TTF_SHAPES:
        X = cases.make_case(K, r, "ttf_cu4_t1e-2").to(device)
        lat, thr = _time_calls(orth, X, flush)
        hl, ht = _time_calls(lambda x: torch.linalg.qr(x)[0], X, flush)
        rows.append({"shape": f"{K}x{r}", "lat_us": round(lat, 1), "thr_us": round(thr, 1),
                     "householder_lat_us": round(hl, 1), "householder_thr_us": round(ht, 1),
                     "speedup_lat": round(hl / lat, 2), "speedup_thr": round(ht / thr, 2),
                     "hbm_frac_lat": round(alg_bytes_orth(K, r) / (lat * 1e-6) / 1e9 / hbm, 4)})
    del flush
    return rows


def gather_desc(world):
    """how the timed calls exchanged results between the ranks"""
    from spanqr_b200 import batched as _batched
    if world == 1:
        return "none (1 GPU)"
    if _batched.exchange_mode() == "peer":
        return (f"peer pulls: each rank's {_batched.WAVES} waves write into its IPC-mapped slab; per wave a one-element "
                f"NCCL all-reduce as the barrier, then one copy-engine copy per owner over NVLink")
    return f"NCCL all_gather_into_tensor per wave, {_batched.WAVES} waves overlapped with compute"


def main():
    a = parse()
    spec = workload_spec(a.workload, a.batch)
    if a.impl == "reference":
        return run_reference(a, spec)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        # NCCL's kernels (the exchange's barriers or all-gathers) on high-priority streams: the waves run on raised
        # priorities, and at the default priority a collective's CTAs would queue behind every wave's pending CTAs
        opts = dist.ProcessGroupNCCL.Options()
        opts.is_high_priority_stream = True
        opts._timeout = timedelta(seconds=300)   # the same as the timeout below (torch warns when they differ)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device, pg_options=opts)
    from spanqr_b200 import orth_batched
    from spanqr_b200 import _lib
    from spanqr_b200.batched import partition

    Xs = make_inputs(spec, device)
    B = len(Xs)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(a.warmup):
        orth_batched(Xs)
    barrier()
    uuids = [str(torch.cuda.get_device_properties(i).uuid) for i in range(torch.cuda.device_count())]
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(uuids) as clk, _lib.KernelTimer(count_only=True) as kt:
        barrier()
        ev0.record(stream)
        for _ in range(a.steps):
            orth_batched(Xs)
        ev1.record(stream)
        barrier()
        kernels = kt.collect()
    ms = dist_max(ev0.elapsed_time(ev1), device)
    clocks = clk.summary()
    value = B * a.steps / (ms / 1e3)
    gpu_launches = sum(n for _, n in kernels.values())

    # the same steps without the exchange (each rank computes its share only), for the cost of the gather
    no_gather = None
    if world > 1:
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        orth_batched(Xs, gather=False)
        barrier()
        g0.record(stream)
        for _ in range(a.steps):
            orth_batched(Xs, gather=False)
        g1.record(stream)
        barrier()
        gms = dist_max(g0.elapsed_time(g1), device)
        no_gather = {"value": B * a.steps / (gms / 1e3), "unit": "matrices/s", "ms_per_step": gms / a.steps}

    # Per-kernel device times for the roofline: the timed region runs large groups on several streams at once, where
    # one launch's CUDA-event span includes the other streams' work; so the same steps are timed again on one stream
    # (same kernels, same launch shapes per part), and the dominant kernel's average launch time is taken from there.
    from spanqr_b200 import batched as _batched
    nstreams = _batched.NSTREAMS
    _batched.NSTREAMS = 1
    try:
        with _lib.KernelTimer() as kt1:
            for _ in range(a.steps):
                orth_batched(Xs)
            barrier()
            kernels = kt1.collect()
    finally:
        _batched.NSTREAMS = nstreams
    steps_1 = a.steps

    # dominant kernel and its roofline (this rank's launches; per-rank work is balanced): the kind's algorithmic bytes
    # per call, summed over this rank's matrices, divided by the kind's launches per step (each launch covers all of
    # them on the one-stream pass)
    hbm, bf16, src = peaks()
    dom = max(kernels.items(), key=lambda kv: kv[1][0])[0]
    dom_ms, dom_n = kernels[dom]
    owner = partition([K * r for K, r in spec["shapes"]], world)
    mine = [spec["shapes"][i] for i in range(B) if owner[i] == rank]
    launches_per_step = dom_n / steps_1
    bytes_per_launch = sum(alg_bytes_per_call(dom, K, r) for K, r in mine) / max(launches_per_step, 1)
    achieved = bytes_per_launch / (dom_ms / dom_n / 1e3) / 1e9
    step_bytes = sum(alg_bytes_orth(K, r) for K, r in mine)
    step_gbs = step_bytes / (ms / a.steps / 1e3) / 1e9

    # end to end through the public API: pinned host inputs of this rank's share in, its results out
    e2e = None
    if not a.no_e2e:
        # every rank passes the whole list (host copies of all inputs) and gets its own share back in pinned memory
        hosts = [Xs[i].cpu().pin_memory() if owner[i] == rank else torch.zeros(1, 1).expand(Xs[i].shape)
                 for i in range(B)]
        hq = [torch.empty(Xs[i].shape, dtype=torch.float32).pin_memory() if owner[i] == rank else None
              for i in range(B)]
        h2d = sum(hosts[i].numel() * 4 for i in range(B) if owner[i] == rank)
        for _ in range(max(1, a.warmup)):
            orth_batched(hosts, gather=False, out=hq)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(a.steps):
            orth_batched(hosts, gather=False, out=hq)
        e1.record(stream)
        barrier()
        ems = dist_max(e0.elapsed_time(e1), device)
        e2e = {"value": B * a.steps / (ems / 1e3), "unit": "matrices/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": h2d, "ms_per_step": ems / a.steps}

    lat_rows = None
    if world == 1 and not a.no_latency:
        lat_rows = orth_latency(device, hbm)

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cpu = cpu_baselines(*spec["shapes"][0])

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "matrices/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": ms / a.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": spec["desc"], "batch": B, "partition": "contiguous blocks by cost",
                       "gather": gather_desc(world),
                       "l2": "inputs larger than L2 (352 MB per step for config 3), no flush"},
            "roofline": {"kernel": dom, "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "peak_source": src, "traffic": ncu_traffic(dom),
                         "alg_bytes_per_launch": bytes_per_launch, "avg_launch_ms": dom_ms / dom_n,
                         "launches_per_step": launches_per_step,
                         "step": {"alg_bytes": step_bytes, "achieved": step_gbs, "frac": step_gbs / hbm,
                                  "what": "17 reads/writes of every K x r matrix per orth over the timed step"},
                         "timing": f"CUDA events around every launch, {steps_1} steps on one stream after the timed "
                                   f"region (the timed region runs each step in {nstreams} parts on {nstreams} streams)"},
            "kernels_ms_per_step": {k: v[0] / steps_1 for k, v in sorted(kernels.items(), key=lambda kv: -kv[1][0])},
            "gpu_launches": gpu_launches,
            "without_gather": no_gather,
            "clocks": clocks,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "orth_latency": lat_rows,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
