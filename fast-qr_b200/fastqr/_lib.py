"""ctypes binding of libfastqr.so (the C ABI in include/fastqr.h).

The library is loaded from this directory only (built in-tree by
``fastqr.build``).  There is no fallback: if the shared object is missing or
does not export the expected symbols, loading raises.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libfastqr.so"

# Every symbol include/fastqr.h declares, with its ctypes signature.
_i64 = ctypes.c_int64
_p = ctypes.c_void_p
SIGNATURES = {
    "fqr_geqrf_f32": (ctypes.c_int, [_p, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, ctypes.c_size_t, _p]),
    "fqr_geqrf_f32_profile": (ctypes.c_int, [_p, _i64, _i64, _i64, _i64, _i64, _p, _p, _p,
                                             ctypes.c_size_t, _p, _p]),
    "fqr_geqrf_f32_noalloc": (ctypes.c_int, [_p, _i64, _i64, _i64, _i64, _i64, _p, _p, _p]),
    "fqr_noalloc_check_status": (ctypes.c_int, [_p]),
    "fqr_debug_force_timeout": (ctypes.c_int, [ctypes.c_int]),
    "fqr_debug_plan": (ctypes.c_int, [ctypes.c_int]),
    "fqr_geqrf_f32_host": (ctypes.c_int, [_p, _i64, _i64, _i64, _i64, _i64, _p, _p, _p,
                                          ctypes.c_size_t, _p]),
    "fqr_host_workspace_bytes": (ctypes.c_size_t, [_i64, _i64]),
    "fqr_host_check_status": (ctypes.c_int, [_p, ctypes.c_size_t, _i64, _i64, _p]),
    "fqr_workspace_bytes": (ctypes.c_size_t, [_i64, _i64]),
    "fqr_geqrf_rect_workspace_bytes": (ctypes.c_size_t, [_i64, _i64, _i64]),
    "fqr_geqrf_rect_f32": (ctypes.c_int, [_p, _i64, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, ctypes.c_size_t,
                                          _p]),
    "fqr_orgqr_workspace_bytes": (ctypes.c_size_t, [_i64, _i64]),
    "fqr_orgqr_f32": (ctypes.c_int, [_p, _p, _i64, _i64, _p, _p, ctypes.c_size_t, _p]),
    "fqr_ormqr_f32": (ctypes.c_int, [_p, _p, _i64, _i64, _p, _i64, ctypes.c_int, _p, ctypes.c_size_t, _p]),
    "fqr_ormqr_right_f32": (ctypes.c_int, [_p, _p, _i64, _i64, _p, _i64, ctypes.c_int, _p, ctypes.c_size_t, _p]),
    "fqr_check_status": (ctypes.c_int, [_p, ctypes.c_size_t, _i64, _p]),
    "fqr_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "fqr_plan_describe": (ctypes.c_int, [_i64, _i64, ctypes.c_char_p, ctypes.c_size_t]),
    "fqr_launch_count": (ctypes.c_int, [_i64, _i64]),
    "fqr_version": (ctypes.c_int, []),
}

STAGES = ("small", "copy_in", "panel", "trailing", "inblock", "mid")

STATUS = {
    0: "FQR_OK",
    1: "FQR_EINVAL",
    2: "FQR_EUNSUPPORTED",
    3: "FQR_ELAUNCH",
    4: "FQR_ETIMEOUT",
    5: "FQR_EWORKSPACE",
    6: "FQR_ECUDA",
    7: "FQR_ENOALLOC_LIMIT",
}

_lib = None


def load(path: Path | None = None):
    """Load libfastqr.so and attach signatures (cached)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise ImportError(
            f"{p} is missing: build it with `python -m fastqr.build` (fastqr has no CPU fallback)")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)  # AttributeError if the ABI is incomplete
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


class FastQRError(RuntimeError):
    """Raised for any non-OK status from the C ABI."""

    def __init__(self, status: int, where: str = "fqr_geqrf_f32"):
        self.status = status
        msg = load().fqr_status_string(status)
        super().__init__(f"{where} failed: {STATUS.get(status, status)} ({msg.decode() if msg else '?'})")
