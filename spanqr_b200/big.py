"""borth: orth for r > 512 (r a multiple of 256), as the reference dispatches it (orth.py:18-19 -> candidates/kbig.py:66-95).

Block Gram-Schmidt with reorthogonalisation (BCGS2) over 256-column blocks: block j (columns j .. j + 255, scaled by
the power of 2 s of the whole X) has the span of the finished blocks P = Q[:, :j] removed twice,
W <- W - P (P^T W), and is orthonormalised by the library's orth recipe with its own slice of the full-width dust
(the K x r draw of the 256-column-wide calls would differ); every later block is then projected and orthonormalised
once more, so that its dust completions are orthogonal to the earlier blocks too.  Every Cholesky stays 256 wide.
The projections are plain fp32 GEMMs (torch.mm, cuBLAS), as in the reference; each block's orth runs in
libspanqr.so through spanqr_orth_f32.
"""
import torch

from .core import zdust, workspace, _call

BLOCK = 256
_ZB = {}


def _pow2_scale(m):
    """candidates/kcholqr.py:29-30 on a device scalar: 2^-round(log2 m) for m > 0 (NaN and 0 give 1)"""
    return torch.where(m > 0, torch.exp2(-torch.round(torch.log2(m.clamp_min(1e-38)))), torch.ones_like(m))


def _block_dust(K, r, dev):
    """the full-width dust Z (K x r, seed 20261018, unit columns) cut into contiguous 256-column blocks"""
    key = (K, r, str(dev))
    if key not in _ZB:
        Z = zdust(K, r, dev)
        _ZB[key] = [Z[:, j:j + BLOCK].contiguous() for j in range(0, r, BLOCK)]
    return _ZB[key]


def _orth_z(W, Z, stream):
    K, b = W.shape
    Q = torch.empty_like(W)
    _call(W, Q, Z, workspace(W.device, K, b, 1, stream), stream.cuda_stream)
    return Q


def borth(X):
    """Q with orthonormal columns spanning X's (fp32 CUDA [K, r], r > 512 a multiple of 256, K >= r); deterministic,
    no host sync, X left untouched (candidates/kbig.py:66-95 with b = 256, reorth on)"""
    K, r = X.shape
    X = X.contiguous()
    dev = X.device
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev)
        Zs = _block_dust(K, r, dev)
        Q = torch.empty_like(X)
        s = _pow2_scale(torch.linalg.vector_norm(X, ord=float("inf")))
        for jb, j in enumerate(range(0, r, BLOCK)):
            W = X[:, j:j + BLOCK] * s
            if j:
                P = Q[:, :j]
                W = W - P @ (P.T @ W)
                W = W - P @ (P.T @ W)
            W = _orth_z(W, Zs[jb], stream)
            if j:
                W = W - P @ (P.T @ W)
                W = _orth_z(W, Zs[jb], stream)
            Q[:, j:j + BLOCK] = W
    return Q
