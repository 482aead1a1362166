"""Each CUDA kernel family against the oracle, through the C ABI.

The clamped Cholesky (k_chol) evaluates exactly the oracle's operation sequence (chol.cu's), so its output must equal
the oracle's bit for bit; so must the row-block solve (k_trsm, rows wider than 256).  The tensor-core solve
(k_trsm_tc) is held to the forward-error bound of a backward-stable solve.  The tensor-core Gram (k_gram_tc,
split-TF32) rounds differently from any CPU order: it is held to an elementwise bound of GRAM_ULPS units of fp32
rounding of sum_k |y_ki| |y_kj| against the exact (fp64) Gram (on its fixture the reference's own compensated gram_f
is 19.5 units off)."""
from pathlib import Path

import numpy as np
import pytest

import oracle
from tests import gpu_util as gu

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"


def spd(n, K, seed, shift_rel=1e-7):
    rng = np.random.default_rng(seed)
    M = rng.standard_normal((K, n)).astype(np.float32) * np.logspace(0, -3, n).astype(np.float32)
    G = oracle.gram_kahan(M)
    nrm = oracle.fro(G)
    G[np.diag_indices(n)] += np.float32(np.float32(shift_rel) * nrm)
    return G, np.float32(np.float32(np.float32(1e-8) * nrm) + np.float32(1e-30))


@pytest.mark.parametrize("n", [32, 64, 96, 128, 160, 256, 288, 480, 512])
def test_chol_bitwise(n):
    G, tau = spd(n, 3 * n, n)
    L, Li = gu.chol(G, tau)
    Lo, Lio = oracle.chol32(G, tau)
    assert gu.bits_equal(L, Lo) and gu.bits_equal(Li, Lio)


def test_chol_bitwise_golden_and_clamped():
    g = np.load(GOLD / "golden.npz")
    L, Li = gu.chol(g["comp/Gs"], g["comp/tau"][0])
    assert gu.bits_equal(L, g["comp/L"]) and gu.bits_equal(Li, g["comp/Li"])
    Z = np.zeros((128, 128), np.float32)                       # every pivot clamped
    L, Li = gu.chol(Z, 1e-6)
    Lo, Lio = oracle.chol32(Z, 1e-6)
    assert gu.bits_equal(L, Lo) and gu.bits_equal(Li, Lio)
    rng = np.random.default_rng(5)                              # rank-deficient Gram: some pivots clamped
    M = rng.standard_normal((300, 20)).astype(np.float32) @ rng.standard_normal((20, 256)).astype(np.float32)
    G = oracle.gram_kahan(M)
    tau = np.float32(1e-8 * oracle.fro(G))
    L, Li = gu.chol(G, tau)
    Lo, Lio = oracle.chol32(G, tau)
    assert gu.bits_equal(L, Lo) and gu.bits_equal(Li, Lio)


GRAM_ULPS = 8
U32 = 2.0 ** -24


def gram_bound_ok(G, Y, s=None):
    Y64 = Y.astype(np.float64) * (s if s is not None else 1.0)
    exact = Y64.T @ Y64
    scale = np.abs(Y64).T @ np.abs(Y64)
    err = np.abs(G.astype(np.float64) - exact)
    return float((err / np.maximum(scale, 1e-300)).max() / U32)


@pytest.mark.parametrize("K,n,scaled", [(100, 64, False), (777, 96, True), (3584, 256, True), (2048, 512, False),
                                        (17408, 256, False), (513, 160, True)])
def test_gram_within_bound(K, n, scaled):
    rng = np.random.default_rng(K + n)
    Y = (rng.standard_normal((K, n)) * 3.0).astype(np.float32)
    s = 0.25 if scaled else None
    G = gu.gram(Y, s)
    assert np.array_equal(G, G.T)
    ulps = gram_bound_ok(G, Y, s)
    assert ulps <= GRAM_ULPS, ulps


def test_gram_close_to_reference_gram_f():
    """the golden G0 is the reference's own tri.gram_f(X, s) (run by Triton's interpreter)"""
    g = np.load(GOLD / "golden.npz")
    X, s = g["comp/X"], float(g["comp/s"][0])
    G = gu.gram(X, s)
    mine, ref = gram_bound_ok(G, X, s), gram_bound_ok(g["comp/G0"], X, s)
    assert mine <= max(GRAM_ULPS, ref), (mine, ref)


def test_gram_ill_scaled_columns():
    """columns spanning 1e-12 .. 1: the bound holds column pair by column pair"""
    rng = np.random.default_rng(7)
    Y = (rng.standard_normal((1024, 128)) * np.logspace(0, -12, 128)).astype(np.float32)
    assert gram_bound_ok(gu.gram(Y), Y) <= GRAM_ULPS


def trsm_err(Y, X, L, s=1.0, Z=None, eps=0.0):
    """max |Y - Y_exact| / (max |Y_exact| kappa(L) u32) for Y_exact = (s X + eps Z) L^-T in fp64"""
    A = X.astype(np.float64) * s + (eps * Z.astype(np.float64) if Z is not None else 0.0)
    L64 = L.astype(np.float64)
    ex = np.linalg.solve(L64, A.T).T
    kappa = np.linalg.cond(L64)
    return float(np.abs(Y.astype(np.float64) - ex).max() / (np.abs(ex).max() * kappa * U32))


@pytest.mark.parametrize("K,n", [(100, 64), (1000, 256), (777, 160), (300, 128), (777, 512), (600, 352)])
def test_trsm_forward_error(K, n):
    """the solve's forward error stays within a few units of kappa(L) u32 of the exact solution, like the oracle's
    (wider than 256 columns the solve runs as two panels, the second started by the first's product)"""
    rng = np.random.default_rng(K * n)
    X = rng.standard_normal((K, n)).astype(np.float32)
    G, tau = spd(n, 2 * n, K)
    L, Li = oracle.chol32(G, tau)
    Z = oracle.dust(K, n)
    Y = gu.trsm(X, L, Li, s=0.5, Z=Z, eps=5e-7)
    Yo = oracle.trsm(X, L, Li, s=0.5, Z=Z, eps=5e-7)
    e_gpu, e_or = trsm_err(Y, X, L, 0.5, Z, 5e-7), trsm_err(Yo, X, L, 0.5, Z, 5e-7)
    assert e_gpu <= max(4.0, 2 * e_or), (e_gpu, e_or)
    Y2 = gu.trsm(X, L, Li, inplace=True)
    assert trsm_err(Y2, X, L) <= max(4.0, 2 * trsm_err(oracle.trsm(X, L, Li), X, L))
