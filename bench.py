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
bandwidth (algorithmic bytes / live CUDA-event duration) over the measured HBM copy bandwidth.
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


def alg_bytes_per_matrix(kind, K, r):
    """algorithmic bytes one launch moves per matrix (the minimum: each input read once, each output written once),
    averaged over that kind's launches in one orth (k_trsm: every pass reads its input, X or Y, and writes Y; the
    dust Z of pass 1 is one matrix for the whole batch and is left out)"""
    kr4 = 4.0 * K * r
    return {"k_absmax": kr4, "k_gram_tc": kr4, "k_gram_tc_acc": kr4, "k_trsm": 2 * kr4,
            "k_ns_update": 2 * kr4, "k_gram_reduce": 4.0 * r * r,
            "k_chol": 3 * 4.0 * r * r, "k_trsm_w": 4.0 * r * r, "k_setup": 16.0}.get(kind, 0.0)


def dist_max(x, device):
    if not (dist.is_available() and dist.is_initialized()):
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------------------------------------------
# arms

def _host_sample(K, r, th):
    """one config-3 member per OpenMP thread (at most 64 distinct matrices, reused beyond that)"""
    from tests import cases
    distinct = [cases.cfg3_matrix(i, K, r).numpy() for i in range(min(th, 64))]
    return [distinct[i % len(distinct)] for i in range(th)]


def cpu_baseline(spec, budget_s=20.0):
    """the oracle (a C restatement of the reference's kcholqr_f) on this host's cores, one matrix per thread, for
    about `budget_s` seconds"""
    import oracle
    K, r = spec["shapes"][0]
    th = oracle.num_threads()
    Z = oracle.dust(K, r)
    Xs = _host_sample(K, r, th)
    t = time.perf_counter()
    oracle.orth_batch(Xs, [Z] * th)
    one = time.perf_counter() - t
    rounds = int(min(32, max(1, budget_s / max(one, 1e-3))))
    t = time.perf_counter()
    for _ in range(rounds):
        oracle.orth_batch(Xs, [Z] * th)
    dt = time.perf_counter() - t
    return {"value": rounds * th / dt, "unit": "matrices/s", "cores": th, "kind": "port",
            "sample": f"{rounds} x {th} matrices of {K}x{r} (config-3 members), one per OpenMP thread, {dt:.1f} s"}


def run_reference(a, spec):
    """--impl reference: the reference's CPU path (the oracle port of kcholqr_f) on the host cores"""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import oracle
    K, r = spec["shapes"][0]
    th = oracle.num_threads()
    Z = oracle.dust(K, r)
    Xs = _host_sample(K, r, th)
    for _ in range(a.warmup):
        oracle.orth_batch(Xs, [Z] * th)
    t = time.perf_counter()
    for _ in range(a.steps):
        oracle.orth_batch(Xs, [Z] * len(Xs))
    dt = time.perf_counter() - t
    v = len(Xs) * a.steps / dt
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "matrices/s", "n_gpus": a.gpus,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": 1e3 * dt / a.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": spec["desc"] + f"; host sample of {len(Xs)} matrices per step"},
            "cpu_baseline": {"value": v, "unit": "matrices/s", "cores": th, "kind": "port",
                             "sample": f"{len(Xs)} matrices of {K}x{r} per step, one per OpenMP thread"},
            "e2e": {"value": v, "unit": "matrices/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


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
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
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

    # dominant kernel and its roofline (this rank's launches; per-rank work is balanced)
    hbm, bf16, src = peaks()
    dom = max(kernels.items(), key=lambda kv: kv[1][0])[0]
    dom_ms, dom_n = kernels[dom]
    owner = partition([K * r for K, r in spec["shapes"]], world)
    mine = [spec["shapes"][i] for i in range(B) if owner[i] == rank]
    per_step_bytes = sum(alg_bytes_per_matrix(dom, K, r) for K, r in mine)
    launches_per_step = dom_n / steps_1
    bytes_per_launch = per_step_bytes / max(launches_per_step, 1)
    achieved = bytes_per_launch / (dom_ms / dom_n / 1e3) / 1e9

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

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cpu = cpu_baseline(spec)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "matrices/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": ms / a.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": spec["desc"], "batch": B, "partition": "contiguous blocks by cost",
                       "gather": f"NCCL all_gather_into_tensor per wave, {_batched.WAVES} waves overlapped with "
                                 f"compute" if world > 1 else "none (1 GPU)",
                       "l2": "inputs larger than L2 (352 MB per step for config 3), no flush"},
            "roofline": {"kernel": dom, "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "peak_source": src, "traffic": ncu_traffic(dom),
                         "alg_bytes_per_launch": bytes_per_launch, "avg_launch_ms": dom_ms / dom_n,
                         "timing": f"CUDA events around every launch, {steps_1} steps on one stream after the timed "
                                   f"region (the timed region runs each step in {nstreams} parts on {nstreams} streams)"},
            "kernels_ms_per_step": {k: v[0] / steps_1 for k, v in sorted(kernels.items(), key=lambda kv: -kv[1][0])},
            "gpu_launches": gpu_launches,
            "without_gather": no_gather,
            "clocks": clocks,
            "e2e": e2e,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
