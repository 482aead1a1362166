"""ctypes binding of libspanqr.so (include/spanqr.h).  Loading fails loudly when the library is missing: there is no
fallback implementation anywhere in this package."""
import ctypes
import threading
from pathlib import Path

_DIR = Path(__file__).resolve().parent
LIB_PATH = _DIR / "libspanqr.so"

# every entry point include/spanqr.h declares, with its argument types
_P, _I, _LL, _F, _SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_float, ctypes.c_size_t
SIGNATURES = {
    "spanqr_version": (_I, []),
    "spanqr_strerror": (ctypes.c_char_p, [_I]),
    "spanqr_last_cuda_error": (ctypes.c_char_p, []),
    "spanqr_workspace_bytes": (_I, [_I, _I, _I, ctypes.POINTER(_SZ)]),
    "spanqr_orth_f32": (_I, [_P, _LL, _P, _LL, _I, _I, _P, _P, _SZ, _P]),
    "spanqr_orth_strided_f32": (_I, [_P, _LL, _LL, _P, _LL, _LL, _I, _I, _I, _P, _P, _SZ, _P]),
    "spanqr_orth_batched_f32": (_I, [_P, _P, _I, _I, _I, _P, _P, _SZ, _P]),
    "spanqr_orth_ptrs_f32": (_I, [_P, _P, _I, _I, _I, _P, _P, _SZ, _P]),
    "spanqr_gram_f32": (_I, [_P, _LL, _I, _I, _P, _P, _P, _SZ, _P]),
    "spanqr_chol_f32": (_I, [_P, _I, _P, _P, _P, _P, _SZ, _P]),
    "spanqr_trsm_f32": (_I, [_P, _LL, _P, _P, _F, _P, _P, _I, _I, _P, _LL, _P, _SZ, _P]),
    "spanqr_read_status": (_I, [_P, _P, ctypes.POINTER(_I)]),
    "spanqr_orth_noalloc_f32": (_I, [_P, _LL, _P, _LL, _I, _I, _P, _P]),
    "spanqr_noalloc_read_status": (_I, [_P, ctypes.POINTER(_I)]),
    "spanqr_workspace_bytes_mixed": (_I, [_P, _I, _I, ctypes.POINTER(_SZ)]),
    "spanqr_orth_mixed_f32": (_I, [_P, _P, _P, _I, _I, _P, _P, _SZ, _P]),
    "spanqr_workspace_bytes_borth": (_I, [_I, _I, ctypes.POINTER(_SZ)]),
    "spanqr_borth_f32": (_I, [_P, _LL, _P, _LL, _I, _I, _P, _P, _SZ, _P]),
    "spanqr_orth_graph_create": (_I, [_I, _I, _LL, _LL, _P, _P, _SZ, ctypes.POINTER(_P)]),
    "spanqr_orth_graph_launch": (_I, [_P, _P, _LL, _P, _LL, _P]),
    "spanqr_orth_graph_destroy": (_I, [_P]),
    "spanqr_gram_mode_f32": (_I, [_P, _LL, _I, _I, _P, _I, _P, _P, _SZ, _P]),
    "spanqr_timing_enable": (_I, [_I]),
    "spanqr_selftest_timeout": (_I, [_P, _SZ, _LL, _I, _P]),
    "spanqr_timing_collect": (_I, [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(_LL), _I]),
    "spanqr_kernel_kinds": (_I, []),
    "spanqr_kernel_kind_name": (ctypes.c_char_p, [_I]),
    "spanqr_peer_slab_alloc": (_I, [_SZ, ctypes.POINTER(_P), _P]),
    "spanqr_peer_slab_open": (_I, [_P, ctypes.POINTER(_P)]),
    "spanqr_peer_slab_close": (_I, [_P]),
    "spanqr_peer_slab_free": (_I, [_P]),
    "spanqr_peer_copy": (_I, [_P, _P, _SZ, _P]),
}

_lib = None
_lock = threading.Lock()


class SpanqrError(RuntimeError):
    """an error status returned by libspanqr"""

    def __init__(self, code, what):
        self.code = code
        msg = f"{what}: {strerror(code)}"
        if code == 4:   # SPANQR_ERR_CUDA
            msg += f" ({lib().spanqr_last_cuda_error().decode()})"
        super().__init__(msg)


def lib():
    """the loaded library (built in-tree by spanqr_b200.build / __graft_entry__.build)"""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise ImportError(f"{LIB_PATH} is missing: build it with `python -m spanqr_b200.build`")
                L = ctypes.CDLL(str(LIB_PATH))
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = L
    return _lib


def strerror(code):
    return lib().spanqr_strerror(int(code)).decode()


def check(code, what):
    if code != 0:
        raise SpanqrError(code, what)


def workspace_bytes(K, r, batch=1):
    n = ctypes.c_size_t(0)
    check(lib().spanqr_workspace_bytes(int(K), int(r), int(batch), ctypes.byref(n)), f"workspace_bytes({K}, {r}, {batch})")
    return n.value


class KernelTimer:
    """per-kernel-kind device time of the orth calls made on this thread while active (CUDA events around every
    launch; see spanqr_timing_enable); with count_only=True, launch counts alone (no events on the streams, times 0)"""

    def __init__(self, count_only=False):
        self.mode = 2 if count_only else 1

    def __enter__(self):
        L = lib()
        self.n = L.spanqr_kernel_kinds()
        self.names = [L.spanqr_kernel_kind_name(i).decode() for i in range(self.n)]
        self.ms = (ctypes.c_double * self.n)()
        self.launches = (ctypes.c_longlong * self.n)()
        L.spanqr_timing_collect(self.ms, self.launches, 0)   # drop anything pending
        check(L.spanqr_timing_enable(self.mode), "timing_enable")
        return self

    def __exit__(self, *exc):
        lib().spanqr_timing_enable(0)

    def collect(self):
        check(lib().spanqr_timing_collect(self.ms, self.launches, self.n), "timing_collect")
        return {nm: (self.ms[i], self.launches[i]) for i, nm in enumerate(self.names) if self.launches[i]}
