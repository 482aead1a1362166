"""oracle/rcholqr.py (the reference's pure-PyTorch CPU path, restated) against the reference's own rcholqr outputs
(tests/golden/golden_rcholqr.npz, made by tests/golden/make_golden_rcholqr.py)."""
import hashlib
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.rcholqr import rcholqr
from tests import cases

GOLD = Path(__file__).resolve().parent / "golden" / "golden_rcholqr.npz"


@pytest.fixture(scope="module")
def g():
    return np.load(GOLD)


def test_restatement_reproduces_reference_rcholqr(g):
    """same torch CPU operations in the same order: bit-identical to the reference's output on one thread (the golden
    ran on one thread; the CPU GEMMs' summation order depends on the thread count, so on all threads the result is
    only checked to be orthonormal)"""
    prev = torch.get_num_threads()
    for key in g["names"]:
        key = str(key)
        K, r = map(int, key.split("/")[0].split("x"))
        X = cases.make_case(K, r, key.split("/")[1])
        assert hashlib.sha1(X.numpy().tobytes()).digest() == g["X_sha1/" + key].tobytes(), key
        ref = g["Q_rows8/" + key]
        try:
            torch.set_num_threads(1)
            one = rcholqr(X).numpy()[::8]
        finally:
            torch.set_num_threads(prev)
        assert np.array_equal(one.view(np.uint32), ref.view(np.uint32)), key
        many = rcholqr(X).double()
        assert (many.T @ many - torch.eye(r, dtype=torch.float64)).abs().max() < 1e-6, key


def test_orthonormal_on_the_baseline_configuration():
    X = cases.cfg3_matrix(3, K=1024)
    Q = rcholqr(X).double()
    assert (Q.T @ Q - torch.eye(256, dtype=torch.float64)).abs().max() < 1e-6
