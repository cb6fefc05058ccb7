"""ctypes binding of the qrb200 C ABI (``include/qrb200.h``).

The shared library is loaded from this package directory only. If it is missing the import
of the operator fails loudly: there is no CPU or library fallback on the product path.
"""

from __future__ import annotations

import ctypes
import os
import threading

from .build import LIB_PATH

QRB200_OK = 0
QRB200_ERR_ARG = 1
QRB200_ERR_WORKSPACE = 2
QRB200_ERR_CUDA = 3
QRB200_ERR_DEVICE = 4
QRB200_ERR_TIMEOUT = 5
QRB200_ERR_SCRATCH_LIMIT = 6
NOALLOC_SCRATCH_BYTES = 32 << 20  # QRB200_NOALLOC_SCRATCH_BYTES

class KernelStat(ctypes.Structure):
    """``qrb200_kernel_stat`` of include/qrb200.h."""

    _fields_ = [("name", ctypes.c_char * 32), ("launches", ctypes.c_int32), ("tensor_bound", ctypes.c_int32),
                ("ms", ctypes.c_double), ("flops", ctypes.c_double), ("bytes", ctypes.c_double)]


# Every symbol include/qrb200.h declares, with its ctypes signature.
SIGNATURES = {
    "qrb200_workspace_bytes": (ctypes.c_size_t, [ctypes.c_int64, ctypes.c_int64]),
    "qrb200_geqrf_f32": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                        ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                        ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "qrb200_geqrf_f32_noalloc": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                                ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                                ctypes.c_void_p]),
    "qrb200_apply_workspace_bytes": (ctypes.c_size_t, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64]),
    "qrb200_ormqr_f32": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                        ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p,
                                        ctypes.c_size_t, ctypes.c_void_p]),
    "qrb200_orgqr_f32": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                        ctypes.c_int64, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "qrb200_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "qrb200_version": (ctypes.c_int, []),
    "qrb200_device_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int)]),
    "qrb200_last_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int)]),
    "qrb200_selftest_wait_timeout": (ctypes.c_int, [ctypes.c_uint32, ctypes.c_void_p]),
    "qrb200_launch_count": (ctypes.c_longlong, []),
    "qrb200_diag_wide_update_f32": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                                   ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "qrb200_profile_geqrf_f32": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                                ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                                ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                                                ctypes.POINTER(KernelStat), ctypes.c_int,
                                                ctypes.POINTER(ctypes.c_int)]),
}

_lock = threading.Lock()
_lib = None


class QRB200Error(RuntimeError):
    """A qrb200 C-ABI call returned a non-zero status."""

    def __init__(self, status: int, what: str = ""):
        self.status = status
        msg = load().qrb200_status_string(status).decode() if _lib is not None else str(status)
        super().__init__(f"qrb200 {what} failed: status {status} ({msg})")


def load(path: str | None = None) -> ctypes.CDLL:
    """Load ``libqrb200.so`` (once) and attach the C signatures."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise ImportError(
                f"qrb200 CUDA library not found at {p}; build it with "
                "`python -m qr_v2_b200_kernel_b200.build` (no CPU fallback exists)")
        lib = ctypes.CDLL(p)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


def check(status: int, what: str) -> None:
    if status != QRB200_OK:
        raise QRB200Error(status, what)


def check_last_status(what: str = "an earlier call") -> None:
    """Raise :class:`QRB200Error` (QRB200_ERR_TIMEOUT) if a kernel on the current device has
    recorded an expired wait since the last check (the results of that call are invalid).

    Reads the library's mapped host word: no CUDA synchronisation, so it reports failures of
    work that has already executed on the device. The word is cleared by the read.
    """
    site = ctypes.c_int(0)
    st = load().qrb200_last_status(ctypes.byref(site))
    if st == QRB200_ERR_TIMEOUT:
        raise QRB200Error(st, f"{what} (device wait site {site.value})")
    check(st, "last_status")
