"""CPU oracle for spanqr's orth(X) -- TEST INFRASTRUCTURE ONLY.

ctypes bindings to ``oracle/liboracle.so`` (built from ``oracle/spanqr_oracle.c`` by ``oracle/Makefile``), a
plain-C restatement of the reference's ``kcholqr_f`` (candidates/kcholqr.py:92-112) and of its kernels
(candidates/cuk/chol.cu, candidates/tri.py).  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline leg import this package; the product (``spanqr_b200``) never does.

Arrays are numpy float32, C-contiguous.  ``nsm`` is the SM count the reference's split-K Gram derives its split
count from (tri.py:365-370); 148 is a B200.
"""
import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_DIR = Path(__file__).resolve().parent
_LIB_PATH = _DIR / "liboracle.so"
_lib = None

_f = ctypes.c_float
_i = ctypes.c_int
_ll = ctypes.c_longlong
_P = ctypes.c_void_p

NSM_B200 = 148
EPS, ALPHA, TAU, NS = 5e-7, 1e-7, 1e-8, 2          # kcholqr.py:92


def build(force=False):
    """compile liboracle.so with oracle/Makefile (gcc + OpenMP)"""
    if force or not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < (_DIR / "spanqr_oracle.c").stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(_DIR)], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(_LIB_PATH))
        L.oracle_rsqrt.restype = _f
        L.oracle_rsqrt.argtypes = [_f]
        L.oracle_pow2_scale.restype = _f
        L.oracle_pow2_scale.argtypes = [_f]
        L.oracle_absmax.restype = _f
        L.oracle_absmax.argtypes = [_P, _ll, _i, _ll]
        L.oracle_gram_kahan.restype = None
        L.oracle_gram_kahan.argtypes = [_P, _i, _i, _ll, _f, _i, _i, _P]
        L.oracle_gram_plain.restype = None
        L.oracle_gram_plain.argtypes = [_P, _i, _i, _ll, _P]
        L.oracle_chol32.restype = _i
        L.oracle_chol32.argtypes = [_P, _i, _f, _P, _P]
        L.oracle_trsm.restype = None
        L.oracle_trsm.argtypes = [_P, _ll, _P, _f, _i, _f, _i, _P, _P, _i, _i, _P, _ll]
        L.oracle_fro.restype = _f
        L.oracle_fro.argtypes = [_P, _i]
        L.oracle_ns.restype = None
        L.oracle_ns.argtypes = [_P, _i, _i, _i, _i]
        L.oracle_kcholqr_f.restype = _i
        L.oracle_kcholqr_f.argtypes = [_P, _ll, _P, _i, _i, _f, _f, _f, _i, _i, _P]
        L.oracle_orth.restype = _i
        L.oracle_orth.argtypes = [_P, _ll, _P, _i, _i, _i, _P]
        L.oracle_orth_batch.restype = _i
        L.oracle_orth_batch.argtypes = [_P, _P, _P, _i, _i, _i, _P]
        L.oracle_num_threads.restype = _i
        L.oracle_num_threads.argtypes = []
        _lib = L
    return _lib


def _c32(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a


def _ptr(a):
    return a.ctypes.data_as(_P)


def rsqrt(x):
    return np.float32(lib().oracle_rsqrt(float(x)))


def pow2_scale(m):
    """kcholqr.py:29-30 _pow2_scale for one fp32 value"""
    return np.float32(lib().oracle_pow2_scale(float(np.float32(m))))


def absmax(X):
    X = _c32(X)
    return np.float32(lib().oracle_absmax(_ptr(X), X.shape[0], X.shape[1], X.shape[1]))


def gram_kahan(Y, s=None, nsm=NSM_B200):
    """tri.gram_f(Y, s=s) / tri.gram_split(Y, bt=64): Kahan split-K Gram of s*Y"""
    Y = _c32(Y)
    K, n = Y.shape
    G = np.empty((n, n), np.float32)
    lib().oracle_gram_kahan(_ptr(Y), K, n, n, float(s if s is not None else 1.0), int(s is not None), nsm, _ptr(G))
    return G


def gram_plain(Y):
    """Y.T @ Y as a plain fp32 GEMM"""
    Y = _c32(Y)
    K, n = Y.shape
    G = np.empty((n, n), np.float32)
    lib().oracle_gram_plain(_ptr(Y), K, n, n, _ptr(G))
    return G


def chol32(A, tau):
    """kchol.chol32: (L, Li) of A (lower tiles read) with pivots clamped at tau"""
    A = _c32(A)
    n = A.shape[0]
    L = np.empty((n, n), np.float32)
    Li = np.empty((n, 32), np.float32)
    if lib().oracle_chol32(_ptr(A), n, float(np.float32(tau)), _ptr(L), _ptr(Li)):
        raise ValueError(f"chol32: n={n} must be a positive multiple of 32")
    return L, Li


def trsm(X, L, Li, s=None, Z=None, eps=0.0):
    """tri.trsm_f: Y = (s X + eps Z) L^-T"""
    X, L, Li = _c32(X), _c32(L), _c32(Li)
    K, n = X.shape
    Zc = _c32(Z) if Z is not None else X
    Y = np.empty((K, n), np.float32)
    lib().oracle_trsm(_ptr(X), n, _ptr(Zc), float(s if s is not None else 1.0), int(s is not None),
                      float(np.float32(eps)), int(Z is not None), _ptr(L), _ptr(Li), K, n, _ptr(Y), n)
    return Y


def fro(G):
    G = _c32(G)
    return np.float32(lib().oracle_fro(_ptr(G), G.shape[0]))


def ns(Y, steps=NS, nsm=NSM_B200):
    Y = _c32(Y).copy()
    K, n = Y.shape
    lib().oracle_ns(_ptr(Y), K, n, steps, nsm)
    return Y


def orth(X, Z, nsm=NSM_B200, eps=EPS, alpha=ALPHA, tau=TAU, ns=NS):
    """kcholqr_f(X) with the dust Z (K x r, unit columns) given"""
    X, Z = _c32(X), _c32(Z)
    K, r = X.shape
    Q = np.empty((K, r), np.float32)
    if lib().oracle_kcholqr_f(_ptr(X), r, _ptr(Z), K, r, eps, alpha, tau, ns, nsm, _ptr(Q)):
        raise ValueError(f"orth: unsupported shape {K}x{r} (r must be a multiple of 32, 32..1024, K >= r)")
    return Q


def borth(X, Z, b=256, nsm=NSM_B200):
    """candidates/kbig.py:66-95 borth(X, b), reorth on: block Gram-Schmidt (BCGS2) over b-column blocks of
    s * X (s = pow2_scale(max |x|) of the whole X), each block orthonormalised by orth() with its own slice of the
    full-width dust Z, projected twice before and once after; projections as float32 GEMMs (numpy)"""
    X, Z = _c32(X), _c32(Z)
    K, r = X.shape
    if r <= b or r % b:
        return orth(X, Z, nsm=nsm)
    s = pow2_scale(absmax(X))
    Q = np.empty_like(X)
    for j in range(0, r, b):
        W = X[:, j:j + b] * s
        Zb = np.ascontiguousarray(Z[:, j:j + b])
        if j:
            P = Q[:, :j]
            W = W - P @ (P.T @ W)
            W = W - P @ (P.T @ W)
        W = orth(W, Zb, nsm=nsm)
        if j:
            W = W - P @ (P.T @ W)
            W = orth(W, Zb, nsm=nsm)
        Q[:, j:j + b] = W
    return Q


def orth_batch(Xs, Zs, nsm=NSM_B200):
    """one orth per matrix, matrices spread over the OpenMP threads (the CPU baseline for orth_batched)"""
    Xs = [_c32(x) for x in Xs]
    Zs = [_c32(z) for z in Zs]
    r = Xs[0].shape[1]
    B = len(Xs)
    Qs = [np.empty_like(x) for x in Xs]
    xp = (_P * B)(*[x.ctypes.data for x in Xs])
    zp = (_P * B)(*[z.ctypes.data for z in Zs])
    qp = (_P * B)(*[q.ctypes.data for q in Qs])
    ks = (_i * B)(*[x.shape[0] for x in Xs])
    if lib().oracle_orth_batch(ctypes.cast(xp, _P), ctypes.cast(zp, _P), ctypes.cast(ks, _P), r, B, nsm,
                               ctypes.cast(qp, _P)):
        raise ValueError("orth_batch: unsupported shape")
    return Qs


def num_threads():
    return lib().oracle_num_threads()


def dust(K, r, seed=20261018):
    """a CPU stand-in for the reference's dust (kcholqr.py:83-89 draws it on the CUDA generator): randn on
    the CPU generator with the same seed, unit columns.  Tests on CPU use it as an input like any other."""
    import torch
    g = torch.Generator().manual_seed(seed)
    Z = torch.randn(K, r, generator=g)
    return (Z / Z.norm(dim=0, keepdim=True)).numpy()


__all__ = ["build", "lib", "rsqrt", "pow2_scale", "absmax", "gram_kahan", "gram_plain", "chol32", "trsm",
           "fro", "ns", "orth", "borth", "orth_batch", "num_threads", "dust", "NSM_B200", "EPS", "ALPHA", "TAU", "NS"]
os.environ.setdefault("OMP_WAIT_POLICY", "PASSIVE")
