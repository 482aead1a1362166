"""Calls into libspanqr's C ABI with torch CUDA tensors (for the GPU tests)."""
import ctypes

import numpy as np
import torch

from spanqr_b200 import _lib


def dev():
    return torch.device("cuda", torch.cuda.current_device())


def cu(a):
    return torch.as_tensor(np.ascontiguousarray(a, dtype=np.float32)).to(dev())


def ws(K, r, B=1):
    return torch.empty(_lib.workspace_bytes(K, r, B), dtype=torch.uint8, device=dev())


def stream():
    return torch.cuda.current_stream().cuda_stream


def gram(Y, s=None):
    Y = cu(Y)
    K, n = Y.shape
    G = torch.empty(n, n, device=dev())
    w = ws(K, n)
    sp = cu(np.array([s], np.float32)) if s is not None else None
    _lib.check(_lib.lib().spanqr_gram_f32(Y.data_ptr(), n, K, n, sp.data_ptr() if sp is not None else None,
                                          G.data_ptr(), w.data_ptr(), w.numel(), stream()), "gram")
    return G.cpu().numpy()


def chol(G, tau):
    G = cu(G)
    n = G.shape[0]
    L = torch.full((n, n), float("nan"), device=dev())
    Li = torch.empty(n, 32, device=dev())
    t = cu(np.array([tau], np.float32))
    w = ws(n, n)
    G0 = G.clone()
    _lib.check(_lib.lib().spanqr_chol_f32(G.data_ptr(), n, t.data_ptr(), L.data_ptr(), Li.data_ptr(), w.data_ptr(),
                                          w.numel(), stream()), "chol")
    assert torch.equal(G, G0), "chol modified its input"
    return L.cpu().numpy(), Li.cpu().numpy()


def trsm(X, L, Li, s=None, Z=None, eps=0.0, inplace=False):
    X, L, Li = cu(X), cu(L), cu(Li)
    K, n = X.shape
    Y = X if inplace else torch.empty_like(X)
    Zt = cu(Z) if Z is not None else None
    sp = cu(np.array([s], np.float32)) if s is not None else None
    w = ws(K, n)
    _lib.check(_lib.lib().spanqr_trsm_f32(X.data_ptr(), n, Zt.data_ptr() if Zt is not None else None,
                                          sp.data_ptr() if sp is not None else None, ctypes.c_float(eps),
                                          L.data_ptr(), Li.data_ptr(), K, n, Y.data_ptr(), n, w.data_ptr(), w.numel(),
                                          stream()), "trsm")
    return Y.cpu().numpy()


def orth_with_dust(X, Z):
    """spanqr_orth_f32 with an explicit dust Z (the product draws Z on the CUDA generator; tests pass the oracle's)"""
    X, Z = cu(X), cu(Z)
    K, r = X.shape
    Q = torch.empty_like(X)
    w = ws(K, r)
    _lib.check(_lib.lib().spanqr_orth_f32(X.data_ptr(), r, Q.data_ptr(), r, K, r, Z.data_ptr(), w.data_ptr(), w.numel(),
                                          stream()), "orth")
    return Q.cpu().numpy()


def bits_equal(a, b):
    """bit-for-bit equality, every NaN counted as one value (the GPU's canonical NaN is 0x7fffffff, the CPU's
    0x7fc00000)"""
    a = np.ascontiguousarray(a, np.float32).view(np.uint32).copy()
    b = np.ascontiguousarray(b, np.float32).view(np.uint32).copy()
    if a.shape != b.shape:
        return False
    a[np.isnan(a.view(np.float32))] = 0x7FC00000
    b[np.isnan(b.view(np.float32))] = 0x7FC00000
    return bool(np.array_equal(a, b))
