"""Generate tests/golden/golden_borth.npz from the REFERENCE's borth run on CPU.

    python tests/golden/make_golden_borth.py --ref /path/to/spanqr

The reference's own ``candidates.kbig.borth(X, 256)`` (kbig.py:66-95; orth.py:18-19 sends r > 512, r a multiple of
256, there) runs with the substitutions of make_golden.py: its Triton kernels under Triton's CPU interpreter, the
CUDA Cholesky ``kchol.chol32`` replaced by this repo's oracle restatement, the dust drawn on the CPU generator
(seed 20261018), the projections as torch CPU fp32 GEMMs.  Cases: the reference generator's matrices at 768 x 768
(three 256-column blocks), about 13 minutes each.  Outputs per case: the SHA-1 of X (tests/cases.py rebuilds X bit
for bit), every 8th row of Q_ref (float32; 768 x 768 is the smallest borth shape, and all of Q would not compress),
and Q_ref's max |Q^T Q - I|.
"""
import hashlib
import argparse
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from make_golden import reference_on_cpu  # noqa: E402

CASES = [(768, 768, "mixed_c2"), (768, 768, "mixed_c4")]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("SPANQR_REF"),
                    help="checkout of oguzeldereli/spanqr (or set SPANQR_REF)")
    ap.add_argument("--out", default=str(HERE / "golden_borth.npz"))
    ap.add_argument("--cases", type=int, default=len(CASES))
    a = ap.parse_args()
    if not a.ref:
        ap.error("give the reference checkout with --ref or SPANQR_REF")
    torch, triton, gen, kcholqr, kchol, tri, _, _ = reference_on_cpu(a.ref)
    from candidates import kbig
    out = {}
    names = []
    for K, r, name in CASES[:a.cases]:
        X = next(c for c in gen.make_cases(K, r, [name], (0,)) if c.name.split("/")[0] == name).X
        Q = kbig.borth(X, 256)
        key = f"{K}x{r}/{name}"
        E = (Q.double().T @ Q.double() - torch.eye(r, dtype=torch.float64)).abs().max()
        out[f"X_sha1/{key}"] = np.frombuffer(hashlib.sha1(X.numpy().tobytes()).digest(), dtype=np.uint8)
        out[f"Q_rows8/{key}"] = Q.numpy()[::8].copy()
        out[f"orth/{key}"] = np.array([float(E)])
        names.append(key)
        print(f"{key:24s} orth {float(E):.2e}", flush=True)
    out["names"] = np.array(names)
    np.savez_compressed(a.out, **out)
    print("wrote", a.out, os.path.getsize(a.out), "bytes")


if __name__ == "__main__":
    main()
