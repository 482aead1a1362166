"""The C ABI without a GPU: libspanqr.so loads, exports every entry point include/spanqr.h declares, and rejects bad
arguments with the documented status codes before touching the device."""
import ctypes
import re
from pathlib import Path

import pytest

from spanqr_b200 import _lib

HDR = Path(__file__).resolve().parent.parent / "include" / "spanqr.h"
OK, SHAPE, ARG, WS = 0, 1, 2, 3


def declared():
    text = re.sub(r"/\*.*?\*/", "", HDR.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(spanqr_[a-z0-9_]+)\s*\(", text)))


def test_exports_every_declared_symbol():
    L = _lib.lib()
    names = declared()
    assert len(names) >= 12
    for n in names:
        assert hasattr(L, n), n
    assert set(names) == set(_lib.SIGNATURES), "the ctypes table must bind exactly the declared entry points"


def test_version_and_strerror():
    L = _lib.lib()
    assert L.spanqr_version() >= 100
    for c in range(6):
        assert L.spanqr_strerror(c)
    assert L.spanqr_last_cuda_error() is not None


@pytest.mark.parametrize("K,r,B,rc", [(768, 512, 1, OK), (17408, 256, 1, OK), (3584, 256, 96, OK), (100, 96, 1, OK),
                                      (768, 100, 1, SHAPE), (768, 544, 1, SHAPE), (100, 128, 1, SHAPE),
                                      (768, 0, 1, SHAPE), (768, 512, 0, SHAPE)])
def test_workspace_bytes(K, r, B, rc):
    n = ctypes.c_size_t(0)
    assert _lib.lib().spanqr_workspace_bytes(K, r, B, ctypes.byref(n)) == rc
    if rc == OK:
        assert n.value > 4 * r * r * B


def test_argument_checks_before_any_device_work():
    L = _lib.lib()
    ws_need = _lib.workspace_bytes(256, 64, 1)
    fake = 1 << 20                 # never dereferenced: every call below fails its checks first
    al = fake * 256
    assert L.spanqr_orth_f32(al, 64, al, 64, 256, 100, al, al, ws_need, None) == SHAPE
    assert L.spanqr_orth_f32(None, 64, al, 64, 256, 64, al, al, ws_need, None) == ARG
    assert L.spanqr_orth_f32(al + 4, 64, al, 64, 256, 64, al, al, ws_need, None) == ARG     # misaligned X
    assert L.spanqr_orth_f32(al, 62, al, 64, 256, 64, al, al, ws_need, None) == ARG         # ldx < r
    assert L.spanqr_orth_f32(al, 64, al, 64, 256, 64, al, al, ws_need - 1, None) == WS      # workspace too small
    assert L.spanqr_orth_f32(al, 64, al, 64, 256, 64, al, al + 16, ws_need, None) == WS     # workspace misaligned
    assert L.spanqr_orth_strided_f32(al, 64, 64 * 256, al, 64, 10, 256, 64, 2, al, al, 10 ** 9, None) == ARG  # overlap
    assert L.spanqr_chol_f32(al, 100, al, al, al, al, 10 ** 9, None) == SHAPE
    assert L.spanqr_trsm_f32(al, 64, None, None, 0.0, al, al, 256, 64, al, 60, al, 10 ** 9, None) == ARG
    assert L.spanqr_gram_f32(al, 64, 32, 64, None, al, al, 10 ** 9, None) == SHAPE           # K < n
    assert L.spanqr_gram_mode_f32(al, 64, 256, 64, None, 3, al, al, 10 ** 9, None) == ARG      # no such mode
    assert L.spanqr_gram_mode_f32(al, 64, 32, 64, None, 1, al, al, 10 ** 9, None) == SHAPE     # K < n
    assert L.spanqr_gram_mode_f32(al, 64, 256, 64, None, 2, al, al, ws_need - 1, None) == WS   # workspace too small
    Ks = (ctypes.c_int * 3)(512, 256, 512)
    n = ctypes.c_size_t(0)
    assert L.spanqr_workspace_bytes_mixed(ctypes.cast(Ks, ctypes.c_void_p), 64, 3, ctypes.byref(n)) == OK
    assert n.value >= _lib.workspace_bytes(512, 64, 2) + _lib.workspace_bytes(256, 64, 1)
    assert L.spanqr_workspace_bytes_mixed(ctypes.cast(Ks, ctypes.c_void_p), 1024, 3, ctypes.byref(n)) == SHAPE
    zs = (ctypes.c_void_p * 3)(al, al, al + 256)        # two dust pointers for the height 512
    ps = (ctypes.c_void_p * 3)(al, al, al)
    assert L.spanqr_orth_mixed_f32(ctypes.cast(ps, ctypes.c_void_p), ctypes.cast(ps, ctypes.c_void_p),
                                   ctypes.cast(Ks, ctypes.c_void_p), 64, 3, ctypes.cast(zs, ctypes.c_void_p), al,
                                   10 ** 9, None) == ARG
    h = ctypes.c_void_p()
    assert L.spanqr_orth_graph_create(256, 100, 100, 100, al, al, 10 ** 9, ctypes.byref(h)) == SHAPE
    assert L.spanqr_orth_graph_create(256, 64, 64, 64, al + 4, al, 10 ** 9, ctypes.byref(h)) == ARG   # misaligned Z
    assert L.spanqr_orth_graph_create(256, 64, 64, 64, al, al, ws_need - 1, ctypes.byref(h)) == WS
    assert L.spanqr_orth_graph_create(256, 64, 64, 64, al, al, ws_need, None) == ARG
    assert L.spanqr_orth_graph_launch(None, al, 64, al, 64, None) == ARG
    assert L.spanqr_orth_graph_destroy(None) == OK
    st = ctypes.c_int(7)
    assert L.spanqr_read_status(None, None, ctypes.byref(st)) == ARG
    assert L.spanqr_noalloc_read_status(None, None) == ARG
    assert L.spanqr_timing_enable(3) == ARG and L.spanqr_timing_enable(-1) == ARG
    assert L.spanqr_timing_enable(2) == OK and L.spanqr_timing_enable(0) == OK
    assert L.spanqr_selftest_timeout(None, 256, 1000, 0, None) == WS
    assert L.spanqr_selftest_timeout(al + 16, 256, 1000, 0, None) == WS                     # misaligned
    assert L.spanqr_selftest_timeout(al, 255, 1000, 0, None) == WS                          # too small
    assert L.spanqr_selftest_timeout(al, 256, 0, 0, None) == ARG                            # no limit
    assert L.spanqr_selftest_timeout(al, 256, 3 * 10 ** 9, 0, None) == ARG                  # above 2 s


@pytest.mark.parametrize("K,r,rc", [(2048, 768, OK), (5120, 1024, OK), (1024, 256, OK), (2048, 640, SHAPE),
                                    (700, 768, SHAPE), (2048, 16640, SHAPE), (1 << 24, 768, SHAPE)])
def test_borth_workspace_bytes(K, r, rc):
    n = ctypes.c_size_t(0)
    assert _lib.lib().spanqr_workspace_bytes_borth(K, r, ctypes.byref(n)) == rc
    if rc == OK:
        assert n.value >= _lib.workspace_bytes(K, 256, 1) + 8 * 256 * (r - 256)


def test_borth_argument_checks_before_any_device_work():
    L = _lib.lib()
    n = ctypes.c_size_t(0)
    assert L.spanqr_workspace_bytes_borth(2048, 768, ctypes.byref(n)) == OK
    need = n.value
    al = (1 << 20) * 256
    far = al + (1 << 34)          # a Q that does not overlap X
    assert L.spanqr_borth_f32(al, 768, far, 768, 2048, 640, al, al, need, None) == SHAPE
    assert L.spanqr_borth_f32(None, 768, far, 768, 2048, 768, al, al, need, None) == ARG
    assert L.spanqr_borth_f32(al, 768, far, 768, 2048, 768, None, al, need, None) == ARG     # no dust
    assert L.spanqr_borth_f32(al + 4, 768, far, 768, 2048, 768, al, al, need, None) == ARG   # misaligned X
    assert L.spanqr_borth_f32(al, 700, far, 768, 2048, 768, al, al, need, None) == ARG       # ldx < r
    assert L.spanqr_borth_f32(al, 768, al + 4096, 768, 2048, 768, al, al, need, None) == ARG  # Q overlaps X
    assert L.spanqr_borth_f32(al, 768, far, 768, 2048, 768, al, al, need - 1, None) == WS    # workspace too small
    assert L.spanqr_borth_f32(al, 768, far, 768, 2048, 768, al, al + 16, need, None) == WS   # workspace misaligned


def test_peer_slab_argument_checks_before_any_device_work():
    """the exchange-slab entry points reject null or empty arguments without a CUDA call; an empty copy is a no-op"""
    L = _lib.lib()
    p = ctypes.c_void_p()
    h = ctypes.create_string_buffer(64)
    assert L.spanqr_peer_slab_alloc(0, ctypes.byref(p), h) == ARG
    assert L.spanqr_peer_slab_alloc(1 << 20, None, h) == ARG
    assert L.spanqr_peer_slab_alloc(1 << 20, ctypes.byref(p), None) == ARG
    assert L.spanqr_peer_slab_open(None, ctypes.byref(p)) == ARG
    assert L.spanqr_peer_slab_open(h, None) == ARG
    assert L.spanqr_peer_slab_close(None) == ARG
    assert L.spanqr_peer_slab_free(None) == ARG
    assert L.spanqr_peer_copy(None, None, 0, None) == OK
    assert L.spanqr_peer_copy(None, 1 << 20, 256, None) == ARG


def test_error_type_names_the_code():
    with pytest.raises(_lib.SpanqrError, match="unsupported shape"):
        _lib.check(SHAPE, "orth")
