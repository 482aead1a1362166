"""orth(X): the drop-in for spanqr's `orth` (orth.py:13-20 -> candidates/kcholqr.py:92-112, kcholqr_f).

    from spanqr_b200 import orth
    Q = orth(X)      # X: fp32 CUDA [K, r] -> Q: fp32 CUDA [K, r], Q^T Q = I, span(Q) = span(X)

Every call runs on libspanqr's CUDA kernels on the current stream, with no host synchronisation.  There is no
fallback: an unsupported shape raises (the reference silently falls back to torch.linalg.qr for r % 32 != 0,
kcholqr.py:98-99, and routes r > 512 to block Gram-Schmidt, orth.py:18-19).
"""
import os
import threading

import torch

from . import _lib

TB = 32               # tile width (candidates/kchol.py:9)
MAX_R = 512
DUST_SEED = 20261018  # candidates/kcholqr.py:86

_Z = {}
_WS = {}
_GRAPHS = {}
_lock = threading.RLock()
# orth() replays one CUDA graph per (device, stream, shape), created in the library, with the call's X and Q patched
# in: the ~30 launches of a call go to the GPU as one unit (SPANQR_GRAPHS=0 launches them one by one instead)
USE_GRAPHS = os.environ.get("SPANQR_GRAPHS", "1") != "0"


def zdust(K, r, device):
    """The dust Z of kcholqr.py:83-89: torch.randn(K, r) on the device's generator seeded 20261018, each column
    divided by its norm; cached per (K, r, device).  Drawn with torch on the same device as the reference draws it,
    so both see the same Z."""
    device = torch.device(device)
    key = (K, r, str(device))
    Z = _Z.get(key)
    if Z is None:
        g = torch.Generator(device=device).manual_seed(DUST_SEED)
        Z = torch.randn(K, r, device=device, generator=g)
        Z = Z / Z.norm(dim=0, keepdim=True)
        with _lock:
            Z = _Z.setdefault(key, Z)
    return Z


def workspace(device, K, r, batch=1, stream=None):
    """a cached device workspace for (device, stream, K, r, batch); calls on different streams never share one"""
    device = torch.device(device)
    if stream is None:
        stream = torch.cuda.current_stream(device)
    key = (str(device), stream.cuda_stream, K, r, batch)
    ws = _WS.get(key)
    if ws is None:
        ws = torch.empty(_lib.workspace_bytes(K, r, batch), dtype=torch.uint8, device=device)
        with _lock:
            ws = _WS.setdefault(key, ws)
    return ws


def check_input(X, name="X"):
    if not torch.is_tensor(X) or X.dim() != 2:
        raise ValueError(f"{name} must be a 2-D tensor [K, r]")
    if X.dtype != torch.float32 or not X.is_cuda:
        raise TypeError(f"{name} must be an fp32 CUDA tensor (got {X.dtype} on {X.device})")
    K, r = X.shape
    if r % TB or r < TB or r > MAX_R or K < r:
        raise ValueError(f"unsupported shape {K}x{r}: r must be a multiple of {TB} in [{TB}, {MAX_R}] and K >= r")


def aligned(X):
    """X itself when contiguous and 16-byte aligned, else a fresh contiguous copy (torch allocations are aligned)"""
    if X.is_contiguous() and X.data_ptr() % 16 == 0:
        return X
    return X.clone(memory_format=torch.contiguous_format)


def orth(X: torch.Tensor) -> torch.Tensor:
    """Orthonormal basis of the column span of X (fp32 CUDA, K >= r, r a multiple of 32 up to 512).  Where X is
    rank-deficient or zero, the missing directions are completed with arbitrary orthonormal ones (never zero or NaN
    columns).  Deterministic, no host sync, X left untouched.  Above r 512 with r a multiple of 256 the columns go
    through block Gram-Schmidt over 256-column blocks (orth.py:18-19, spanqr_b200.big.borth).  r % 32 != 0 is
    padded with zero columns to the next multiple of 32, and r > 512 that is not a multiple of 256 to the next multiple
    of 256 (K must reach it); the first r columns are returned."""
    if torch.is_tensor(X) and X.dim() == 2 and X.shape[1] > 0 and (X.shape[1] % TB or X.shape[1] > MAX_R):
        if X.dtype != torch.float32 or not X.is_cuda:
            raise TypeError(f"X must be an fp32 CUDA tensor (got {X.dtype} on {X.device})")
        K, r = X.shape
        if r % TB or (r > MAX_R and r % 256):
            # padded tiles instead of the reference's Householder fallback (kcholqr.py:98-99): zero columns up to
            # the next multiple of 32 (of 256 above 512, where the reference runs kcholqr_f at full width,
            # orth.py:18-20, and this build goes blockwise); the solves are triangular, so Q's first r columns span X
            rp = -(-r // TB) * TB if r <= MAX_R else -(-r // 256) * 256
            if K < rp:
                raise ValueError(f"unsupported shape {K}x{r}: r is padded to {rp} here, which needs K >= {rp}")
            Xp = torch.zeros((K, rp), dtype=torch.float32, device=X.device)
            Xp[:, :r] = X
            return orth(Xp)[:, :r].contiguous()
        if r % 256 == 0:
            if K < r:
                raise ValueError(f"unsupported shape {K}x{r}: K >= r")
            from .big import borth
            return borth(X)
    check_input(X)
    X = aligned(X)
    K, r = X.shape
    dev = X.device
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev)
        Q = torch.empty((K, r), dtype=torch.float32, device=dev)
        if USE_GRAPHS:
            g = _graph(dev, stream, K, r)
            _lib.check(_lib.lib().spanqr_orth_graph_launch(g.handle, X.data_ptr(), r, Q.data_ptr(), r,
                                                           stream.cuda_stream), f"orth({K}x{r})")
            return Q
        _call(X, Q, zdust(K, r, dev), workspace(dev, K, r, 1, stream), stream.cuda_stream)
    return Q


def _call(X, Q, Z, ws, stream_handle):
    K, r = X.shape
    _lib.check(_lib.lib().spanqr_orth_f32(X.data_ptr(), r, Q.data_ptr(), r, K, r, Z.data_ptr(), ws.data_ptr(),
                                          ws.numel(), stream_handle), f"orth({K}x{r})")


class _Graph:
    """one captured orth(K x r) call (spanqr_orth_graph_create) with its own workspace; each replay gets the call's X and
    Q patched into its set-up kernel, so nothing is copied in or out"""

    def __init__(self, dev, stream, K, r, Z):
        self.ws = torch.empty(_lib.workspace_bytes(K, r, 1), dtype=torch.uint8, device=dev)
        self.z = Z
        x = torch.zeros((K, r), dtype=torch.float32, device=dev)
        q = torch.empty_like(x)
        _call(x, q, self.z, self.ws, stream.cuda_stream)   # first run eagerly: kernels loaded, attributes set
        h = _lib.ctypes.c_void_p()
        _lib.check(_lib.lib().spanqr_orth_graph_create(K, r, r, r, Z.data_ptr(), self.ws.data_ptr(), self.ws.numel(),
                                                       _lib.ctypes.byref(h)), f"orth graph ({K}x{r})")
        self.handle = h

    def __del__(self):
        try:
            _lib.lib().spanqr_orth_graph_destroy(self.handle)
        except Exception:
            pass


def _graph(dev, stream, K, r):
    key = (str(dev), stream.cuda_stream, K, r)
    g = _GRAPHS.get(key)
    if g is None:
        Z = zdust(K, r, dev)   # outside the lock: zdust takes it too
        with _lock:
            g = _GRAPHS.get(key)
            if g is None:
                g = _GRAPHS[key] = _Graph(dev, stream, K, r, Z)
    return g
