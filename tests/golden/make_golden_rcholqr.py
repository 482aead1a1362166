"""Golden outputs of the reference's own pure-PyTorch rcholqr (candidates/rcholqr.py:61-65) on CPU, which pin the
restatement in oracle/rcholqr.py.  Run where a checkout of the reference exists (it is never read at test time):

    python tests/golden/make_golden_rcholqr.py --ref /path/to/spanqr

Stores per case the SHA-1 of X (tests/cases.py rebuilds X) and every 8th row of Q = rcholqr(X) with the
reference's default arguments, into tests/golden/golden_rcholqr.npz.
"""
import argparse
import hashlib
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

CASES = [(384, 128, "mixed_c2"), (1024, 256, "ttf_cu4_t1e-2"), (768, 512, "mixed_c6")]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("SPANQR_REF"),
                    help="checkout of oguzeldereli/spanqr (or set SPANQR_REF)")
    ap.add_argument("--out", default=str(HERE / "golden_rcholqr.npz"))
    a = ap.parse_args()
    if not a.ref:
        ap.error("give the reference checkout with --ref or SPANQR_REF")
    sys.path.insert(0, a.ref)
    import torch
    from candidates.rcholqr import rcholqr
    from tests import cases
    torch.set_num_threads(1)
    out = {}
    for K, r, name in CASES:
        X = cases.make_case(K, r, name)
        Q = rcholqr(X)
        key = f"{K}x{r}/{name}"
        out[f"X_sha1/{key}"] = np.frombuffer(hashlib.sha1(X.numpy().tobytes()).digest(), dtype=np.uint8)
        out[f"Q_rows8/{key}"] = Q.numpy()[::8].copy()
    out["names"] = np.array([f"{K}x{r}/{n}" for K, r, n in CASES])
    np.savez_compressed(a.out, **out)
    print("wrote", a.out, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
