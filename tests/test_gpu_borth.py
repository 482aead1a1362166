"""orth above r 512 (block Gram-Schmidt over 256-column blocks, orth.py:18-19 -> candidates/kbig.py:66-95) on the GPU
against the oracle's restatement with the same dust: elementwise for kappa <= 1e6, orthogonality, span, bits stable
from call to call, input untouched."""
import numpy as np
import pytest
import torch

import oracle
from spanqr_b200 import orth, zdust
from tests.test_oracle import _mixed, _kappa, elementwise_tol

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("K,r,kappa,deficient", [(2048, 768, 1e3, False), (5120, 1024, 1e5, False),
                                                 (2048, 768, 1e3, True)])
def test_borth_matches_oracle(K, r, kappa, deficient):
    X = _mixed(K, r, kappa, 11)
    if deficient:
        X[:, 512:768] = X[:, :256] @ np.random.default_rng(12).standard_normal((256, 256))
    X = X.astype(np.float32)
    Xg = torch.from_numpy(X).cuda()
    keep = Xg.clone()
    Q = orth(Xg)
    Q2 = orth(Xg)
    torch.cuda.synchronize()
    assert torch.equal(Xg, keep)
    assert torch.equal(Q.view(torch.int32), Q2.view(torch.int32))
    q = Q.cpu().numpy()
    qo = oracle.borth(X, zdust(K, r, "cuda").cpu().numpy())
    assert np.isfinite(q).all()
    qd, qod = q.astype(np.float64), qo.astype(np.float64)
    err = np.abs(qd.T @ qd - np.eye(r)).max()
    err_o = np.abs(qod.T @ qod - np.eye(r)).max()
    assert err <= max(2e-7, 1.5 * err_o), (err, err_o)
    Xd = X.astype(np.float64)
    assert np.linalg.norm(Xd - qd @ (qd.T @ Xd)) <= 1e-5 * np.linalg.norm(Xd)
    if not deficient:
        assert _kappa(X) <= 1e6
        assert np.abs(q - qo).max() <= elementwise_tol(_kappa(X))


def test_width_above_512_not_a_multiple_of_256_is_padded():
    """r in (512, 1024] that is not a multiple of 256 (the reference runs kcholqr_f there, orth.py:18-20): zero columns
    up to the next multiple of 256, blockwise, the first r columns returned; equal to the oracle's borth on the padded
    matrix within the elementwise bound, orthonormal and spanning X"""
    K, r, rp = 2048, 640, 768
    X = (_mixed(K, r, 1e3, 13) * 4.0).astype(np.float32)
    Q = orth(torch.from_numpy(X).cuda())
    torch.cuda.synchronize()
    assert Q.shape == (K, r)
    q = Q.cpu().numpy().astype(np.float64)
    Xp = np.zeros((K, rp), np.float32)
    Xp[:, :r] = X
    qo = oracle.borth(Xp, zdust(K, rp, "cuda").cpu().numpy())[:, :r]
    assert np.abs(q - qo).max() <= elementwise_tol(_kappa(X))
    assert np.abs(q.T @ q - np.eye(r)).max() <= 2e-7
    Xd = X.astype(np.float64)
    assert np.linalg.norm(Xd - q @ (q.T @ Xd)) <= 1e-5 * np.linalg.norm(Xd)


def test_borth_rejects_what_the_block_path_cannot_take():
    with pytest.raises(ValueError):
        orth(torch.zeros(700, 768, device="cuda"))    # K < r
    with pytest.raises(ValueError):
        orth(torch.zeros(700, 640, device="cuda"))    # r 640 is padded to 768 > K


def test_borth_c_abi_leading_dimensions_and_status():
    """spanqr_borth_f32 through the C ABI with X a column slice of a wider matrix (ldx > r) and Q written into a wider
    buffer (ldq > r): the same bits as the contiguous call, the columns outside Q's slice untouched, and the
    workspace's status word 0 afterwards"""
    import ctypes
    from spanqr_b200 import _lib
    L = _lib.lib()
    K, r = 2048, 768
    X = torch.from_numpy(_mixed(K, r, 1e3, 21).astype(np.float32)).cuda()
    want = orth(X)
    wide = torch.randn(K, r + 256, device="cuda")
    wide[:, 128:128 + r] = X
    Xs = wide[:, 128:128 + r]
    Qw = torch.full((K, r + 64), 7.0, device="cuda")
    n = ctypes.c_size_t()
    assert L.spanqr_workspace_bytes_borth(K, r, ctypes.byref(n)) == 0
    ws = torch.empty(n.value, dtype=torch.uint8, device="cuda")
    Z = zdust(K, r, "cuda")
    st = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        rc = L.spanqr_borth_f32(Xs.data_ptr(), r + 256, Qw.data_ptr(), r + 64, K, r, Z.data_ptr(), ws.data_ptr(),
                                n.value, st)
        assert rc == 0, _lib.lib().spanqr_strerror(rc)
        status = ctypes.c_int(-1)
        assert L.spanqr_read_status(ws.data_ptr(), st, ctypes.byref(status)) == 0 and status.value == 0
        assert torch.equal(Qw[:, :r].contiguous().view(torch.int32), want.view(torch.int32))
        assert torch.all(Qw[:, r:] == 7.0)
