"""Generate tests/golden/golden.npz from the REFERENCE implementation run on CPU.

Run in a container that has the reference checkout (it is never read at test time):

    python tests/golden/make_golden.py --ref /path/to/spanqr

What runs, and what is substituted:
  * the reference's own orchestration ``candidates.kcholqr.kcholqr_f`` (kcholqr.py:92-112), its ``_pow2_scale``,
    ``_zdust`` (on the CPU generator, seed 20261018), ``_ns_mm``, and its Triton kernels ``tri.gram_f`` /
    ``tri.gram_split`` / ``tri._trsm_f_kernel`` executed by Triton's CPU interpreter (TRITON_INTERPRET=1);
  * the reference's test-matrix builders ``qrbench.gen`` (cases and seed formula, gen.py:171-182), kept on CPU;
  * ``kchol.chol32`` (CUDA C++, cannot run on CPU) is replaced by this repo's oracle restatement of chol.cu;
  * the interpreter loads a kernel's own earlier stores from the pre-launch buffer, so ``trsm_f``'s reload of
    finished column blocks (tri.py:395-398) is reproduced by relaunching the unmodified kernel r/32 times with the
    previous output as the buffer (each launch finalises one more block; the fixed point is the sequential result);
  * ``torch.cuda.get_device_properties`` reports 148 SMs (a B200) for the Gram split count (tri.py:365-370).

Outputs (float32): per case X, Q_ref; the dust checksum; component fixtures (gram_f, trsm_f, gram_split outputs on
one case); a sweep of _pow2_scale values.  Everything is small (K x r <= 256 x 128).
"""
import argparse
import hashlib
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent

# (K, r, case names); r a multiple of 64: the reference's Gram tiles are 64 wide with unmasked columns
# (tri.py:346-347), so r % 64 == 32 reads and writes past the matrix there.
# ttf_first_rank32 is left out at 128 x 64: there the fp32 Schur complements of the last columns fall below the
# Cholesky's own rounding noise, the pivots are clamped at tau and the 32 x 32 tile inverse (chol.cu:151-168)
# overflows to inf/NaN.  That is the reference algorithm's behaviour at this size, not a fixture worth pinning;
# at the TTF shapes the same case passes.
PLAN = [
    (128, 64, ["mixed_c2", "mixed_c4", "mixed_c6", "mixed_c8", "zero", "rank_half", "dup_cols",
               "ttf_cu2_t1e-1", "ttf_cu4_t1e-2", "ttf_first", "mixed_c14", "zero_block", "rank_1",
               "tiny_1e-25", "huge_1e25"]),
    (256, 128, ["mixed_c2", "mixed_c6", "ttf_cu4_t1", "dup_cols"]),
]


def reference_on_cpu(ref):
    """import the reference from `ref` with the CPU substitutions listed above; returns (torch, triton, gen, kcholqr,
    kchol, tri, chol32_oracle, trsm_f_interp)"""
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, ref)
    sys.path.insert(0, str(REPO))
    import torch

    class _Props:
        multi_processor_count = 148
    torch.cuda.get_device_properties = lambda *args, **kw: _Props()

    import triton
    from qrbench import gen
    from candidates import kcholqr, kchol, tri
    import oracle

    gen._finish = lambda X64: X64.to(torch.float32).contiguous()

    def chol32_oracle(G, tau):
        L, Li = oracle.chol32(G.numpy(), float(tau.reshape(-1)[0]))
        return torch.from_numpy(L), torch.from_numpy(Li)

    def trsm_f_interp(X, L, Li, s=None, Z=None, eps=0.0, bm=16, bs=32, prec="tf32x3", warps=4, stages=2):
        K, n = X.shape
        Y = torch.zeros_like(X)
        for _ in range(n // bs):
            Yn = Y.clone()
            tri._trsm_f_kernel[(triton.cdiv(K, bm),)](
                X, Z if Z is not None else X, s if s is not None else X, float(eps), L, Li, Yn, K, n,
                BM=bm, BS=bs, PREC=prec, HAS_S=s is not None, HAS_Z=Z is not None, num_warps=warps,
                num_stages=stages)
            Y = Yn
        return Y

    kchol.chol32 = chol32_oracle
    tri.trsm_f = trsm_f_interp
    return torch, triton, gen, kcholqr, kchol, tri, chol32_oracle, trsm_f_interp


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("SPANQR_REF"),
                    help="checkout of oguzeldereli/spanqr (or set SPANQR_REF)")
    ap.add_argument("--out", default=str(HERE / "golden.npz"))
    a = ap.parse_args()
    if not a.ref:
        ap.error("give the reference checkout with --ref or SPANQR_REF")
    torch, triton, gen, kcholqr, kchol, tri, chol32_oracle, trsm_f_interp = reference_on_cpu(a.ref)

    out = {}
    names = []
    for K, r, cases in PLAN:
        Z = kcholqr._zdust(K, r, torch.device("cpu"))
        zd = Z.numpy()
        out[f"Z_sha1/{K}x{r}"] = np.frombuffer(hashlib.sha1(zd.tobytes()).digest(), dtype=np.uint8)
        for c in gen.make_cases(K, r, cases, (0,)):
            if c.name.split("/")[0] not in cases:      # make_cases also matches by prefix
                continue
            X = c.X
            Q = kcholqr.kcholqr_f(X)
            key = f"{K}x{r}/{c.name}"
            out[f"X/{key}"] = X.numpy().copy()
            out[f"Q/{key}"] = Q.numpy().copy()
            names.append(key)
            print(f"{key:32s} orth {float((Q.double().T @ Q.double() - torch.eye(r, dtype=torch.float64)).abs().max()):.2e}",
                  flush=True)

    # component fixtures on one case: s, gram_f(X, s), trsm_f pass 0 (given the oracle's L, Li), gram_split
    K, r = 256, 128
    X = next(gen.make_cases(K, r, ["mixed_c6"], (0,))).X
    Z = kcholqr._zdust(K, r, torch.device("cpu"))
    s = kcholqr._pow2_scale(torch.linalg.vector_norm(X, ord=float("inf"))).reshape(1)
    G0 = tri.gram_f(X, s=s)
    nrm = torch.linalg.matrix_norm(G0)
    Gs = G0.clone()
    Gs.diagonal().add_(1e-7 * nrm)
    tau = (1e-8 * nrm + 1e-30).reshape(1)
    L, Li = chol32_oracle(Gs, tau)
    Y1 = trsm_f_interp(X, L, Li, s=s, Z=Z, eps=5e-7)
    G1 = tri.gram_split(Y1, bt=64)
    out.update({"comp/X": X.numpy(), "comp/s": s.numpy(), "comp/G0": G0.numpy(), "comp/nrm": nrm.reshape(1).numpy(),
                "comp/tau": tau.numpy(), "comp/Gs": Gs.numpy(), "comp/L": L.numpy(), "comp/Li": Li.numpy(),
                "comp/Y1": Y1.numpy(), "comp/G1": G1.numpy()})

    # _pow2_scale over a sweep (powers of 2, near sqrt(2) boundaries, tiny, subnormal, zero, inf, nan)
    rng = np.random.default_rng(1)
    ms = [0.0, float("inf"), float("nan"), 1e-45, 1e-40, 1e-38, 1.2e-38, 1.0, 2.0 ** 0.5, 3e38]
    for k in range(-130, 128):
        b = np.float32(2.0 ** (k + 0.5)) if -149 < k + 0.5 < 128 else None
        if b is not None and np.isfinite(b):
            ms += [float(np.nextafter(b, np.float32(0))), float(b), float(np.nextafter(b, np.float32(np.inf)))]
    ms += list((np.float32(2.0) ** rng.uniform(-140, 127, 300)).astype(np.float32))
    m = torch.tensor(np.array(ms, dtype=np.float32))
    out["pow2/m"] = m.numpy()
    out["pow2/s"] = kcholqr._pow2_scale(m).numpy()

    out["names"] = np.array(names)
    np.savez_compressed(a.out, **out)
    print("wrote", a.out, os.path.getsize(a.out), "bytes")

    # fingerprints of the reference generator's matrices (tests/cases.py must reproduce them) and the reference's
    # published per-case metrics (results/synth_kcholf.json, results/synth_kcholf_rtx5060ti.json)
    import json
    fps = {}
    for K, r in [(768, 512), (2048, 512), (3584, 256), (5120, 256), (17408, 256)]:
        for c in gen.make_cases(K, r, None, (0,)):
            fps[f"{K}x{r}/{c.name}"] = hashlib.sha1(c.X.numpy().tobytes()).hexdigest()[:16]
    pub = {}
    for fn in ("synth_kcholf.json", "synth_kcholf_rtx5060ti.json"):
        d = json.load(open(os.path.join(a.ref, "results", fn)))
        pub[fn] = {"device": d["device"],
                   "rows": [{k: w[k] for k in ("K", "r", "case", "hard", "cond", "orth", "span_n", "hh_span_n", "fails")}
                            for w in d["rows"]]}
    side = os.path.join(os.path.dirname(a.out), "reference_fixtures.json")
    with open(side, "w") as f:
        json.dump({"gen_fingerprints": fps, "published": pub}, f, indent=0, sort_keys=True)
    print("wrote", side, os.path.getsize(side), "bytes")


if __name__ == "__main__":
    main()
