"""CPU oracle for batched square Householder QR -- TEST INFRASTRUCTURE ONLY.

This package is the checker, never the thing measured or shipped.  Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
import it.  The product path (``fastqr``) never imports it and has no CPU
fallback.

What it restates (third-party algorithm, pinned through the installed torch
wheel: LAPACK xGEQRF as shipped by MKL 2024.2 in torch 2.11):

* ``geqrf_f64`` / ``geqrf_f32``: unblocked Householder QR, LAPACK xGEQR2 +
  xLARFG semantics -- the arithmetic behind ``torch.geqrf``, which is the
  reference's own contract (official/reference.py:125-127 ``ref_kernel``,
  submissions/baseline_geqrf.py:5-6).  ``geqrf_rect_f64``: the same for
  m x n matrices (the reference's embedded rectangular geqrf routes,
  submissions/candidate.py:7204-7214), pinned against numpy's LAPACK.
* ``geqrf_blocked_f64``: the compact-WY blocked variant of
  tools/blocked_qr_reference.py:98-122,192-262 (the algorithm the GPU
  blocked path executes).
* ``orgqr_f32`` / ``orgqr_f64``: ``torch.linalg.householder_product``
  (LAPACK xORG2R), used by the official checker (official/reference.py:199).

Parity is pinned by tests/test_oracle.py against golden vectors produced by
running the reference's own generator and torch.geqrf in the build container
(tests/golden/make_golden.py).

Array conventions: ``A`` is ``float32[b, n, n]`` with logical (row, col)
indexing (any strides).  Returned ``H`` has the same logical indexing; its
memory is column-major per matrix, like torch.geqrf's output.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "liboracle.so"
_lib = None

_i64 = ctypes.c_int64
_p = ctypes.c_void_p


def build() -> Path:
    """Compile the C restatement with the committed Makefile."""
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < (_HERE / "geqr2.c").stat().st_mtime:
        build()
    lib = ctypes.CDLL(str(_LIB_PATH))
    for name in ("oracle_geqrf_f64", "oracle_geqrf_f32"):
        fn = getattr(lib, name)
        fn.argtypes = [_i64, _i64, _p, _i64, _i64, _i64, _p, _p]
        fn.restype = ctypes.c_int
    lib.oracle_geqrf_rect_f64.argtypes = [_i64, _i64, _i64, _p, _i64, _i64, _i64, _p, _p]
    lib.oracle_geqrf_rect_f64.restype = ctypes.c_int
    lib.oracle_geqrf_blocked_f64.argtypes = [_i64, _i64, _i64, _p, _i64, _i64, _i64, _p, _p]
    lib.oracle_geqrf_blocked_f64.restype = ctypes.c_int
    for name in ("oracle_orgqr_f64", "oracle_orgqr_f32"):
        fn = getattr(lib, name)
        fn.argtypes = [_i64, _i64, _p, _p, _p]
        fn.restype = ctypes.c_int
    lib.oracle_version.restype = ctypes.c_char_p
    _lib = lib
    return lib


def _as_input(a) -> np.ndarray:
    a = np.asarray(a)
    if a.dtype != np.float32 or a.ndim != 3 or a.shape[1] != a.shape[2]:
        raise ValueError("A must be float32 with shape (batch, n, n)")
    return a


def _strides(a: np.ndarray):
    return tuple(s // a.itemsize for s in a.strides)


def _colmajor(buf: np.ndarray) -> np.ndarray:
    # buf is [b][j][i] in memory; expose logical [b, i, j]
    return buf.transpose(0, 2, 1)


def geqrf_f64(a):
    """Householder QR in double arithmetic.  Returns (H float64, tau float64)."""
    a = _as_input(a)
    b, n, _ = a.shape
    h = np.empty((b, n, n), dtype=np.float64)
    tau = np.empty((b, n), dtype=np.float64)
    bs, rs, cs = _strides(a)
    rc = _load().oracle_geqrf_f64(b, n, a.ctypes.data, bs, rs, cs, h.ctypes.data, tau.ctypes.data)
    if rc:
        raise RuntimeError(f"oracle_geqrf_f64 failed: {rc}")
    return _colmajor(h), tau


def geqrf_f32(a):
    """Householder QR in float arithmetic (norms in double).  Returns float32 (H, tau)."""
    a = _as_input(a)
    b, n, _ = a.shape
    h = np.empty((b, n, n), dtype=np.float32)
    tau = np.empty((b, n), dtype=np.float32)
    bs, rs, cs = _strides(a)
    rc = _load().oracle_geqrf_f32(b, n, a.ctypes.data, bs, rs, cs, h.ctypes.data, tau.ctypes.data)
    if rc:
        raise RuntimeError(f"oracle_geqrf_f32 failed: {rc}")
    return _colmajor(h), tau


def geqrf_rect_f64(a):
    """Householder QR of float32[b, m, n] (any m, n) in double arithmetic.
    Returns (H float64 [b, m, n] logical view of column-major memory,
    tau float64 [b, min(m, n)])."""
    a = np.asarray(a)
    if a.dtype != np.float32 or a.ndim != 3:
        raise ValueError("A must be float32 with shape (batch, m, n)")
    b, m, n = a.shape
    h = np.empty((b, n, m), dtype=np.float64)  # [b][j][i]
    tau = np.empty((b, min(m, n)), dtype=np.float64)
    bs, rs, cs = _strides(a)
    rc = _load().oracle_geqrf_rect_f64(b, m, n, a.ctypes.data, bs, rs, cs, h.ctypes.data, tau.ctypes.data)
    if rc:
        raise RuntimeError(f"oracle_geqrf_rect_f64 failed: {rc}")
    return _colmajor(h), tau


def geqrf_blocked_f64(a, nb: int):
    """Compact-WY blocked Householder QR (panel width ``nb``) in double arithmetic."""
    a = _as_input(a)
    b, n, _ = a.shape
    h = np.empty((b, n, n), dtype=np.float64)
    tau = np.empty((b, n), dtype=np.float64)
    bs, rs, cs = _strides(a)
    rc = _load().oracle_geqrf_blocked_f64(b, n, nb, a.ctypes.data, bs, rs, cs, h.ctypes.data, tau.ctypes.data)
    if rc:
        raise RuntimeError(f"oracle_geqrf_blocked_f64 failed: {rc}")
    return _colmajor(h), tau


def _h_colmajor_f32(h) -> np.ndarray:
    h = np.asarray(h, dtype=np.float32)
    # memory layout [b][j][i]
    return np.ascontiguousarray(h.transpose(0, 2, 1))


def orgqr_f64(h, tau):
    """Q = H_0 H_1 ... H_{n-1} from compact (H, tau), accumulated in double."""
    hc = _h_colmajor_f32(h)
    t = np.ascontiguousarray(np.asarray(tau, dtype=np.float32))
    b, n, _ = hc.shape
    q = np.empty((b, n, n), dtype=np.float64)
    rc = _load().oracle_orgqr_f64(b, n, hc.ctypes.data, t.ctypes.data, q.ctypes.data)
    if rc:
        raise RuntimeError(f"oracle_orgqr_f64 failed: {rc}")
    return _colmajor(q)


def orgqr_f32(h, tau):
    """Same product accumulated in float, as torch.linalg.householder_product on float32."""
    hc = _h_colmajor_f32(h)
    t = np.ascontiguousarray(np.asarray(tau, dtype=np.float32))
    b, n, _ = hc.shape
    q = np.empty((b, n, n), dtype=np.float32)
    rc = _load().oracle_orgqr_f32(b, n, hc.ctypes.data, t.ctypes.data, q.ctypes.data)
    if rc:
        raise RuntimeError(f"oracle_orgqr_f32 failed: {rc}")
    return _colmajor(q)


def version() -> str:
    return _load().oracle_version().decode()


def cpu_count() -> int:
    return os.cpu_count() or 1
