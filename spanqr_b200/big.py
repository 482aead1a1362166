"""borth: orth for r > 512 (r a multiple of 256), as the reference dispatches it (orth.py:18-19 -> candidates/kbig.py:66-95).

Block Gram-Schmidt with reorthogonalisation (BCGS2) over 256-column blocks, all of it in libspanqr.so
(spanqr_borth_f32): block j (columns j .. j + 255, scaled by the power of 2 s of the whole X) has the span of the
finished blocks P = Q[:, :j] removed twice, W <- W - P (P^T W) (a band Gram and an in-place update on the tensor
cores), and is orthonormalised by the library's orth recipe with its own slice of the full-width dust (the K x r draw
of the 256-column-wide calls would differ); every later block is then projected and orthonormalised once more, so that
its dust completions are orthogonal to the earlier blocks too.  Every Cholesky stays 256 wide.
"""
import torch

from . import _lib
from .core import zdust, _lock

BLOCK = 256
_WS = {}


def _workspace(dev, stream, K, r):
    key = (str(dev), stream.cuda_stream, K, r)
    ws = _WS.get(key)
    if ws is None:
        n = _lib.ctypes.c_size_t()
        _lib.check(_lib.lib().spanqr_workspace_bytes_borth(K, r, _lib.ctypes.byref(n)), f"borth({K}x{r})")
        ws = torch.empty(n.value, dtype=torch.uint8, device=dev)
        with _lock:
            ws = _WS.setdefault(key, ws)
    return ws


def borth(X):
    """Q with orthonormal columns spanning X's (fp32 CUDA [K, r], r > 512 a multiple of 256, K >= r); deterministic,
    no host sync, X left untouched (candidates/kbig.py:66-95 with b = 256, reorth on)"""
    K, r = X.shape
    X = X.contiguous()
    dev = X.device
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev)
        Q = torch.empty_like(X)
        ws = _workspace(dev, stream, K, r)
        _lib.check(_lib.lib().spanqr_borth_f32(X.data_ptr(), r, Q.data_ptr(), r, K, r, zdust(K, r, dev).data_ptr(),
                                               ws.data_ptr(), ws.numel(), stream.cuda_stream), f"borth({K}x{r})")
    return Q
