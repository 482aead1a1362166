"""Seeded test matrices: the reference's case families (qrbench/gen.py) and the BASELINE configurations.

Every matrix is built in fp64 on the CPU from a seeded torch generator, then rounded to fp32 (gen.py:33-48), so the
same seed gives the same fp32 matrix anywhere.  The case list, its order and the seed formula
1_000_003 * seed + 7919 * index + 31 * K + r follow gen.py:138-182, so a case here is the reference's matrix
(tests/test_cases.py checks fingerprints recorded from the reference's own generator).
"""
import math

import numpy as np
import torch

SHAPES = [(768, 512), (2048, 512), (1024, 256), (2048, 256), (3584, 256), (5120, 256), (6144, 256), (17408, 256)]


def gen(seed):
    return torch.Generator().manual_seed(seed)


def orth64(K, r, g):
    """random K x r orthonormal (fp64): QR of a Gaussian, signs fixed by R's diagonal (gen.py:37-40)"""
    Q, R = torch.linalg.qr(torch.randn(K, r, generator=g, dtype=torch.float64))
    return Q * torch.sign(torch.diagonal(R))


def mixed_spectrum(K, r, s, g):
    """Q1 diag(s) Q2^T, both factors Haar (gen.py:43-44)"""
    return orth64(K, r, g) @ torch.diag(s) @ orth64(r, r, g).T


def mixed(K, r, g, c):
    return mixed_spectrum(K, r, torch.logspace(0, -c, r, dtype=torch.float64), g)


def cluster(K, r, g, c):
    s = torch.ones(r, dtype=torch.float64)
    s[r // 2:] = 10.0 ** -c
    return mixed_spectrum(K, r, s[torch.randperm(r, generator=g)], g)


def zero(K, r, g):
    return torch.zeros(K, r, dtype=torch.float64)


def rank(K, r, g, k):
    return torch.randn(K, k, generator=g, dtype=torch.float64) @ torch.randn(k, r, generator=g, dtype=torch.float64)


def dup_cols(K, r, g):
    X = torch.randn(K, r, generator=g, dtype=torch.float64)
    X[:, r // 2: 2 * (r // 2)] = X[:, : r // 2]
    return X


def zero_block(K, r, g):
    X = torch.randn(K, r, generator=g, dtype=torch.float64)
    X[:, r // 4: r // 2] = 0
    return X


def graded(K, r, g, c):
    return torch.randn(K, r, generator=g, dtype=torch.float64) * torch.logspace(0, -c, r, dtype=torch.float64)


def ttf_parts(K, r, g, cu, tilt, sig_rank=32, noise=0.3):
    """TTF-structured X = V B + P, B = U^T U with U's spectrum logspace(0, -cu), P = u^T U scaled to tilt ||V B||
    (gen.py:95-115)"""
    su = torch.logspace(0, -cu, r, dtype=torch.float64)
    Qr = orth64(r, r, g)
    N = max(K, r)
    Qn = orth64(N, r, g)
    U_rs = torch.diag(su) @ Qr.T
    B = U_rs.T @ U_rs
    V = orth64(K, r, g)
    Lf = torch.randn(N, sig_rank, generator=g, dtype=torch.float64) / math.sqrt(N)
    Rf = torch.randn(K, sig_rank, generator=g, dtype=torch.float64)
    P = Rf @ ((Lf.T @ Qn) @ U_rs) + noise * torch.randn(K, r, generator=g, dtype=torch.float64) @ U_rs
    VB = V @ B
    P = P * (tilt * VB.norm() / P.norm()) if tilt > 0 else torch.zeros_like(P)
    return VB + P


def ttf_first(K, r, g, noise):
    N = max(K, r)
    Lf = torch.randn(N, 32, generator=g, dtype=torch.float64) / math.sqrt(N)
    Rf = torch.randn(K, 32, generator=g, dtype=torch.float64)
    G = torch.randn(N, r, generator=g, dtype=torch.float64)
    X = Rf @ (Lf.T @ G)
    if noise > 0:
        X = X + noise * math.sqrt(32) * torch.randn(K, r, generator=g, dtype=torch.float64)
    return X


def case_table(K, r):
    """(name, builder(g) -> fp64 X, hard) in the reference's order (gen.py:138-164)"""
    out = [(f"mixed_c{c}", (lambda g, c=c: mixed(K, r, g, c)), True) for c in (2, 4, 6, 8)]
    out += [
        ("zero", lambda g: zero(K, r, g), True),
        ("rank_half", lambda g: rank(K, r, g, r // 2), True),
        ("dup_cols", lambda g: dup_cols(K, r, g), True),
        ("ttf_cu2_t1e-1", lambda g: ttf_parts(K, r, g, 2, 1e-1), True),
        ("ttf_cu4_t1e-2", lambda g: ttf_parts(K, r, g, 4, 1e-2), True),
        ("ttf_cu4_t1", lambda g: ttf_parts(K, r, g, 4, 1.0), True),
        ("ttf_zero_grad_cu4.5", lambda g: ttf_parts(K, r, g, 4.5, 0.0), True),
        ("ttf_first", lambda g: ttf_first(K, r, g, 0.1), True),
        ("ttf_first_rank32", lambda g: ttf_first(K, r, g, 0.0), True),
        ("mixed_c10", lambda g: mixed(K, r, g, 10), False),
        ("mixed_c14", lambda g: mixed(K, r, g, 14), False),
        ("cluster_c5", lambda g: cluster(K, r, g, 5), False),
        ("cluster_c9", lambda g: cluster(K, r, g, 9), False),
        ("zero_block", lambda g: zero_block(K, r, g), False),
        ("rank_1", lambda g: rank(K, r, g, 1), False),
        ("graded_c8", lambda g: graded(K, r, g, 8), False),
        ("tiny_1e-25", lambda g: 1e-25 * mixed(K, r, g, 4), False),
        ("huge_1e25", lambda g: 1e25 * mixed(K, r, g, 4), False),
    ]
    return out


def case_names(K=768, r=512):
    return [n for n, _, _ in case_table(K, r)]


def make_case(K, r, name, seed=0):
    """fp32 CPU matrix of the named case (exact name)"""
    for i, (n, build, _) in enumerate(case_table(K, r)):
        if n == name:
            return build(gen(1_000_003 * seed + 7919 * i + K * 31 + r)).to(torch.float32).contiguous()
    raise KeyError(name)


def is_hard(name):
    return dict((n, h) for n, _, h in case_table(8, 8))[name]


def fingerprint(X):
    """a short fingerprint of a float32 matrix's bytes"""
    import hashlib
    return hashlib.sha1(np.ascontiguousarray(X.numpy() if torch.is_tensor(X) else X, dtype=np.float32).tobytes()).hexdigest()[:16]


# ---- BASELINE configurations (synthetic data of the reference's shapes, sizes and value distributions) ----

def cfg0(seed=0):
    """768 x 512: A diag(logspace(0, -6, 512)) B^T with A, B Haar, times 2^3"""
    g = gen(seed)
    s = torch.logspace(0, -6, 512, dtype=torch.float64)
    return (8.0 * mixed_spectrum(768, 512, s, g)).to(torch.float32)


def ttf_form(K, N, r, g, cu):
    """X = V (U^T U) + u^T U: V Haar K x r, U N x r Gaussian with column scales logspace(0, -cu, r), u an N x K
    Gaussian gradient normalised to unit RMS (fp64)"""
    V = orth64(K, r, g)
    U = torch.randn(N, r, generator=g, dtype=torch.float64) * torch.logspace(0, -cu, r, dtype=torch.float64)
    u = torch.randn(N, K, generator=g, dtype=torch.float64)
    u = u / u.pow(2).mean().sqrt()
    return V @ (U.T @ U) + u.T @ U


def cfg1(seed=0):
    """TTF form, K 2048, N 768, r 512, U scales logspace(0, -4)"""
    return ttf_form(2048, 768, 512, gen(seed), 4.0).to(torch.float32)


def cfg2(K, name, seed=0):
    """robustness sweep at K x 256: kappa1e14, rank1, zero_block64, dup32, scale_m83, scale_p83, zero"""
    r = 256
    g = gen(1_000_003 * seed + 31 * K + r + sum(map(ord, name)))
    if name == "kappa1e14":
        X = mixed(K, r, g, 14)
    elif name == "rank1":
        X = torch.randn(K, 1, generator=g, dtype=torch.float64) @ torch.randn(1, r, generator=g, dtype=torch.float64)
    elif name == "zero_block64":
        X = torch.randn(K, r, generator=g, dtype=torch.float64)
        X[:, 96:160] = 0
    elif name == "dup32":
        X = torch.randn(K, r, generator=g, dtype=torch.float64)
        X[:, 224:256] = X[:, 0:32]
    elif name in ("scale_m83", "scale_p83", "base83"):
        X = mixed(K, r, gen(1_000_003 * seed + 31 * K + r), 4)
        X = X * (2.0 ** (-83 if name == "scale_m83" else (83 if name == "scale_p83" else 0)))
    elif name == "zero":
        X = torch.zeros(K, r, dtype=torch.float64)
    else:
        raise KeyError(name)
    return X.to(torch.float32).contiguous()


CFG2_CASES = ["kappa1e14", "rank1", "zero_block64", "dup32", "scale_m83", "scale_p83", "zero"]


def cfg3_matrix(i, K=3584, r=256):
    """config 3 member i (seed i): Haar-mixed, kappa log-uniform in [1e2, 1e10]; members 0, 12, 24, ... (8 of 96)
    exactly rank 192"""
    g = gen(i)
    logk = 2.0 + 8.0 * torch.rand(1, generator=g, dtype=torch.float64).item()
    s = torch.logspace(0, -logk, r, dtype=torch.float64)
    if i % 12 == 0:
        s[192:] = 0.0
    return mixed_spectrum(K, r, s, g).to(torch.float32)


def cfg4_matrix(i, n_small=256, K_small=6144, K_big=17408, r=256, N=5120):
    """config 4 member i: TTF form with N 5120, kappa(U) log-uniform in [1e1, 1e4]; the first n_small are 6144 x 256,
    the rest 17408 x 256"""
    g = gen(10_000 + i)
    K = K_small if i < n_small else K_big
    cu = 1.0 + 3.0 * torch.rand(1, generator=g, dtype=torch.float64).item()
    return ttf_form(K, N, r, g, cu).to(torch.float32)
