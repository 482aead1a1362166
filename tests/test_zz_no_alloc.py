"""The orth entry point that allocates nothing (spanqr_orth_noalloc_f32).

It exists for callers that cannot allocate device memory: code inside a CUDA stream capture that must not add
allocations, memory-capped sandboxes, real-time loops that forbid cudaMalloc.  It keeps its scratch in a fixed 16 MiB
array of the library's device image instead of a caller workspace, so it must give exactly what the workspace entry
point (spanqr_orth_f32) gives, call after call, even though the array keeps the previous call's contents.
This file is collected last so that a run stopping at the first failure has already run every other test.
"""
import ctypes

import pytest
import torch

from spanqr_b200 import _lib, zdust
from tests import cases

NOALLOC_BYTES = 16 << 20


def test_ttf_shapes_fit_the_fixed_scratch():
    for K, r in cases.SHAPES:
        assert _lib.workspace_bytes(K, r, 1) <= NOALLOC_BYTES, (K, r)


def test_rejects_bad_shapes_before_touching_the_device():
    L = _lib.lib()
    assert L.spanqr_orth_noalloc_f32(None, 100, None, 100, 768, 100, None, None) == 1   # SPANQR_ERR_SHAPE
    assert "16 MiB" in _lib.strerror(6)                                                  # SPANQR_ERR_TOO_LARGE


def test_rejects_shapes_beyond_the_array_before_touching_the_device():
    """a valid shape whose workspace exceeds the fixed array returns SPANQR_ERR_TOO_LARGE with null pointers (no GPU
    needed: the size check comes before any CUDA call), and the largest TTF shape stays inside it"""
    L = _lib.lib()
    assert _lib.workspace_bytes(65536, 512, 1) > NOALLOC_BYTES
    assert L.spanqr_orth_noalloc_f32(None, 512, None, 512, 65536, 512, None, None) == 6
    big = max(cases.SHAPES, key=lambda s: _lib.workspace_bytes(*s, 1))
    assert _lib.workspace_bytes(*big, 1) <= NOALLOC_BYTES


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_on_two_calls():
    L = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    for K, r, name in [(768, 512, "ttf_cu4_t1e-2"), (2048, 256, "mixed_c6")]:     # two calls in a row, two shapes
        X = cases.make_case(K, r, name).cuda()
        Z = zdust(K, r, X.device)
        ws = torch.empty(_lib.workspace_bytes(K, r, 1), dtype=torch.uint8, device=X.device)
        want = torch.empty_like(X)
        _lib.check(L.spanqr_orth_f32(X.data_ptr(), r, want.data_ptr(), r, K, r, Z.data_ptr(), ws.data_ptr(),
                                     ws.numel(), stream), "orth")
        got = torch.full_like(X, float("nan"))
        _lib.check(L.spanqr_orth_noalloc_f32(X.data_ptr(), r, got.data_ptr(), r, K, r, Z.data_ptr(), stream),
                   "orth_noalloc")
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int32), want.view(torch.int32)), (K, r, name)
        st = ctypes.c_int(-1)
        assert L.spanqr_noalloc_read_status(stream, ctypes.byref(st)) == 0 and st.value == 0


@pytest.mark.gpu
def test_noalloc_second_call_ignores_what_the_first_left_behind():
    """two calls in a row at one r > 256 shape, the first on a different matrix: the array still holds the first
    call's Gram partials, update scratch (r > 256) and status words, and the second result must not depend on them"""
    L = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    K, r = 2048, 512
    X1 = cases.make_case(K, r, "mixed_c6").cuda()
    X2 = cases.make_case(K, r, "ttf_cu4_t1e-2").cuda()
    Z = zdust(K, r, X2.device)
    ws = torch.empty(_lib.workspace_bytes(K, r, 1), dtype=torch.uint8, device=X2.device)
    want = torch.empty_like(X2)
    _lib.check(L.spanqr_orth_f32(X2.data_ptr(), r, want.data_ptr(), r, K, r, Z.data_ptr(), ws.data_ptr(), ws.numel(),
                                 stream), "orth")
    first = torch.empty_like(X1)
    _lib.check(L.spanqr_orth_noalloc_f32(X1.data_ptr(), r, first.data_ptr(), r, K, r, Z.data_ptr(), stream), "first")
    got = torch.full_like(X2, float("nan"))
    _lib.check(L.spanqr_orth_noalloc_f32(X2.data_ptr(), r, got.data_ptr(), r, K, r, Z.data_ptr(), stream), "second")
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int32), want.view(torch.int32))
    assert not torch.equal(first.view(torch.int32), got.view(torch.int32))
    st = ctypes.c_int(-1)
    assert L.spanqr_noalloc_read_status(stream, ctypes.byref(st)) == 0 and st.value == 0
