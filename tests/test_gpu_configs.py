"""The BASELINE configurations at their own full shapes, through the product entry points (orth, orth_batched, with the
dust drawn on the CUDA generator as the reference draws it), elementwise against the CPU oracle; and each Gram mode the
orth sequence runs, on its own, against the exact Gram and the oracle's restatement of the reference's compensated
gram_f.

Elementwise bound: max |Q - Q_oracle| <= elementwise_tol(kappa) for kappa <= 1e6 (tests/test_oracle.py gives the
measured curve it is set from); above kappa 1e6 and for rank-deficient members the completion directions are
arbitrary, and the members are held to orthogonality and to the oracle's span error instead."""
import numpy as np
import pytest
import torch

import oracle
from spanqr_b200 import orth, orth_batched, zdust, _lib
from tests import cases, metrics
from tests import gpu_util as gu
from tests.test_oracle import elementwise_tol

pytestmark = pytest.mark.gpu
U32 = 2.0 ** -24


def _orth_err(Q):
    Qd = Q.astype(np.float64)
    return float(np.abs(Qd.T @ Qd - np.eye(Q.shape[1])).max())


def _check_member(Q, Qo, X, kappa, what):
    assert np.isfinite(Q).all(), what
    assert _orth_err(Q) <= 2e-7, (what, _orth_err(Q))
    if kappa <= 1e6:
        d = float(np.abs(Q.astype(np.float64) - Qo).max())
        assert d <= elementwise_tol(kappa), (what, kappa, d)
    else:
        Xt = torch.from_numpy(X)
        ref = metrics.reference(Xt)
        mine = metrics.evaluate(torch.from_numpy(Q), Xt, ref)["span_n"]
        theirs = metrics.evaluate(torch.from_numpy(Qo), Xt, ref)["span_n"]
        assert mine <= 2 * theirs + 1.0, (what, mine, theirs)


def _cfg3_kappa(i):
    """the member's condition number as the generator draws it (inf for the rank-192 members)"""
    g = cases.gen(i)
    logk = 2.0 + 8.0 * torch.rand(1, generator=g, dtype=torch.float64).item()
    return float("inf") if i % 12 == 0 else 10.0 ** logk


def test_cfg3_members_at_full_size():
    """16 config-3 members (3584 x 256; two of them rank 192, kappa drawn log-uniform in 1e2..1e10, up to 2e9 here)
    through orth_batched, against the oracle member by member"""
    idx = list(range(16))
    Xs = [cases.cfg3_matrix(i) for i in idx]
    Z = zdust(3584, 256, "cuda").cpu().numpy()
    Qs = [q.cpu().numpy() for q in orth_batched([x.cuda() for x in Xs])]
    Qo = oracle.orth_batch([x.numpy() for x in Xs], [Z] * len(Xs))
    assert sum(1 for i in idx if i % 12 == 0) == 2 and max(_cfg3_kappa(i) for i in idx if i % 12) > 1e9
    for i, X, Q, q in zip(idx, Xs, Qs, Qo):
        _check_member(Q, q, X.numpy(), _cfg3_kappa(i), f"cfg3 member {i}")


def test_cfg4_members_at_full_size():
    """config 4 in TTF form at its own shapes (6144 x 256 and 17408 x 256, N 5120): two members of each shape in one
    mixed-shape orth_batched call, against the oracle"""
    idx = [0, 1, 256, 257]
    Xs = [cases.cfg4_matrix(i) for i in idx]
    Qs = [q.cpu().numpy() for q in orth_batched([x.cuda() for x in Xs])]
    for i, X, Q in zip(idx, Xs, Qs):
        K, r = X.shape
        Qo = oracle.orth(X.numpy(), zdust(K, r, "cuda").cpu().numpy())
        s = np.linalg.svd(X.double().numpy(), compute_uv=False)
        _check_member(Q, Qo, X.numpy(), float(s[0] / s[-1]), f"cfg4 member {i} ({K}x{r})")


@pytest.mark.parametrize("name", ["cfg0", "cfg1s0", "cfg1s1"])
def test_cfg0_cfg1_against_oracle(name):
    """config 0 (768 x 512, kappa 1e6) and config 1 (TTF form 2048 x 512, N 768) through orth"""
    X = cases.cfg0(0) if name == "cfg0" else cases.cfg1(int(name[-1]))
    K, r = X.shape
    Q = orth(X.cuda()).cpu().numpy()
    Qo = oracle.orth(X.numpy(), zdust(K, r, "cuda").cpu().numpy())
    s = np.linalg.svd(X.double().numpy(), compute_uv=False)
    _check_member(Q, Qo, X.numpy(), float(s[0] / s[-1]), name)


# ---- each Gram of the orth sequence on its own (spanqr_gram_mode_f32) ----
# Measured on B200 (units of u32 of sum_k |y_ki| |y_kj| per entry, worst over Gaussian, orthonormal and graded inputs
# at the shapes below): the pass mode (two-way split TF32, whole 512-row split in TMEM) 6.4 against the exact Gram,
# the polish mode (drained every 128 rows) 1.7, the oracle's compensated gram_f 1.9.
GRAM_BOUND = {1: 8.0, 2: 3.0, 0: 3.0}        # against the exact (fp64) Gram
GRAM_VS_ORACLE = {1: 8.0, 2: 3.0, 0: 3.0}    # against the oracle's restatement of gram_f


def gram_mode(Y, mode, s=None):
    Yt = gu.cu(Y)
    K, n = Yt.shape
    G = torch.empty(n, n, device="cuda")
    w = gu.ws(K, n)
    sp = gu.cu(np.array([s], np.float32)) if s is not None else None
    _lib.check(_lib.lib().spanqr_gram_mode_f32(Yt.data_ptr(), n, K, n, sp.data_ptr() if sp is not None else None, mode,
                                               G.data_ptr(), w.data_ptr(), w.numel(), gu.stream()), "gram_mode")
    return G.cpu().numpy()


def _ulps(G, Gref, Y, s):
    Y64 = Y.astype(np.float64) * (s if s is not None else 1.0)
    scale = np.abs(Y64).T @ np.abs(Y64)
    return float((np.abs(G.astype(np.float64) - Gref) / np.maximum(scale, 1e-300)).max() / U32)


@pytest.mark.parametrize("mode", [1, 2, 0], ids=["pass", "polish", "accurate"])
@pytest.mark.parametrize("K,n,kind,scaled", [(3584, 256, "gauss", True), (3584, 256, "orth", False),
                                             (768, 512, "gauss", False), (768, 512, "orth", True),
                                             (2048, 512, "orth", False), (17408, 256, "orth", False),
                                             (513, 160, "gauss", True), (3584, 256, "graded", False)])
def test_gram_mode_against_exact_and_oracle(mode, K, n, kind, scaled):
    rng = np.random.default_rng(K * 7 + n)
    if kind == "gauss":
        Y = (rng.standard_normal((K, n)) * 3).astype(np.float32)
    elif kind == "orth":
        Y = np.linalg.qr(rng.standard_normal((K, n)))[0].astype(np.float32)
    else:
        Y = (rng.standard_normal((K, n)) * np.logspace(0, -12, n)).astype(np.float32)
    s = 0.25 if scaled else None
    G = gram_mode(Y, mode, s)
    assert np.array_equal(G, G.T)
    Y64 = Y.astype(np.float64) * (s if s is not None else 1.0)
    assert _ulps(G, Y64.T @ Y64, Y, s) <= GRAM_BOUND[mode]
    Go = oracle.gram_kahan(Y, s=s).astype(np.float64)
    assert _ulps(G, Go, Y, s) <= GRAM_VS_ORACLE[mode]
