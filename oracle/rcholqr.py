"""The reference's pure-PyTorch CPU path, rcholqr (candidates/rcholqr.py:61-65) -- TEST AND BASELINE INFRASTRUCTURE ONLY.

This restates, with torch CPU operations, the robust Cholesky-QR recipe the reference ships as its pure-PyTorch
method `rcholqr` (its default registration "rchol3", candidates/rcholqr.py:68).  It is the "reference's CPU path"
that bench.py times on the host cores beside torch.linalg.qr (LAPACK Householder); tests/test_rcholqr.py pins it against
outputs of the reference's own rcholqr (tests/golden/golden_rcholqr.npz, made by tests/golden/make_golden_rcholqr.py).
The product (spanqr_b200) never imports it.

The recipe (a different one from the GPU path's kcholqr_f; its constants are rcholqr.py:61):
  1. Y = s1 X with s1 = 2^-round(log2 max|X|) (exact), then Y = s2 Y with s2 = the same power-of-2 scale of the
     largest column norm of Y (rcholqr.py:36-39);
  2. Y += eps Z, eps = 2e-7, Z the dust: randn(K, r) on the generator seeded 20261018, unit columns
     (rcholqr.py:22-29, 40-41);
  3. three passes Y <- Y R^-1 with R^T R = Y^T Y + (alpha ||Y^T Y||_F + 1e-30) I, alpha = 1e-6, 1e-6, 1e-7, R from
     a Cholesky and applied with a triangular solve (rcholqr.py:45-54);
  4. one Newton-Schulz step Y <- 1.5 Y - 0.5 Y (Y^T Y) (rcholqr.py:57-60).
"""
import torch

DUST_SEED = 20261018           # rcholqr.py:25
EPS = 2e-7                     # rcholqr.py:61
ALPHAS = (1e-6, 1e-6, 1e-7)    # rcholqr.py:61
NS = 1                         # rcholqr.py:61

_dust = {}


def dust(K, r):
    """rcholqr.py:22-29 on the CPU generator: randn(K, r) seeded 20261018, each column over its norm; cached"""
    Z = _dust.get((K, r))
    if Z is None:
        g = torch.Generator().manual_seed(DUST_SEED)
        Z = torch.randn(K, r, generator=g)
        Z = _dust[(K, r)] = Z / Z.norm(dim=0, keepdim=True)
    return Z


def pow2_scale(m):
    """rcholqr.py:32-33: 2^-round(log2 m) elementwise, 1 where m is 0"""
    e = torch.round(torch.log2(torch.clamp(m, min=1e-38)))
    return torch.where(m > 0, torch.exp2(-e), torch.ones_like(m))


def rcholqr(X, eps=EPS, alphas=ALPHAS, ns=NS):
    """orth(X) of a CPU fp32 [K, r] tensor by the reference's pure-PyTorch recipe (the steps listed above)"""
    Y = X * pow2_scale(X.abs().amax())
    cmax = Y.norm(dim=0).amax()
    Y = Y * pow2_scale(cmax)
    if eps > 0:
        Y = torch.addcmul(Y, dust(*X.shape), torch.full_like(cmax, eps))
    for a in alphas:
        G = Y.T @ Y
        shift = a * torch.linalg.matrix_norm(G) + 1e-30
        G = G + torch.diag_embed(shift.expand(G.shape[0]))
        R, _ = torch.linalg.cholesky_ex(G, upper=True)
        Y = torch.linalg.solve_triangular(R, Y, upper=True, left=False)
    for _ in range(ns):
        Y = 1.5 * Y - 0.5 * (Y @ (Y.T @ Y))
    return Y.contiguous()
