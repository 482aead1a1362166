"""Accuracy metrics of an orth output, restated from the reference's qrbench/metrics.py:23-99.

span_n: for each left singular direction u_i of X with sigma_i > 1e-6 sigma_1 (fp64 SVD of the fp32 input),
s_i = ||(I - Q Q^T) u_i||; span_n = max_i s_i (sigma_i / sigma_1) / 2^-24 ("units of fp32 rounding").
orth: max |Q^T Q - I| in fp64.  Pass (metrics.py:15-20, 46-62): finite, no column with norm < 0.5, orth <= 1e-6,
span_n <= max(10 x Householder's, 100).
"""
import torch

U32 = 2.0 ** -24
SPAN_THRESH = 1e-6


def reference(X):
    Xd = X.detach().double().cpu()
    Qd, Rd = torch.linalg.qr(Xd)
    Ur, S, _ = torch.linalg.svd(Rd)
    return S, Qd @ Ur


def evaluate(Q, X, ref=None):
    ref = ref if ref is not None else reference(X)
    K, r = X.shape
    Qd = Q.detach().double().cpu()
    fin = torch.isfinite(Qd).all(dim=0)
    out = {"finite": bool(fin.all()), "bad_cols": 0, "orth": float("nan"), "span_n": 0.0, "span_raw": 0.0}
    norms = torch.where(fin, Qd.norm(dim=0), torch.zeros(r, dtype=torch.float64))
    out["bad_cols"] = int(((~fin) | (norms < 0.5)).sum())
    if not out["finite"]:
        return out
    out["orth"] = float((Qd.T @ Qd - torch.eye(r, dtype=torch.float64)).abs().max())
    S, Ud = ref
    if S[0] > 0:
        keep = S > SPAN_THRESH * S[0]
        Uk = Ud[:, keep]
        s = (Uk - Qd @ (Qd.T @ Uk)).norm(dim=0)
        if int(keep.sum()):
            out["span_raw"] = float(s.max())
            out["span_n"] = float((s * (S[keep] / S[0]) / U32).max())
    return out


def cond(ref):
    S = ref[0]
    return float(S[0] / S[-1]) if S[-1] > 0 else float("inf")


def householder_span(X, ref):
    """span_n of fp32 Householder (torch.linalg.qr) on the same matrix: the yardstick of metrics.py:46-62"""
    Q = torch.linalg.qr(X.detach().float().cpu())[0]
    return evaluate(Q, X, ref)["span_n"]
