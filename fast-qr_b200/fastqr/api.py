"""PyTorch-facing entry points.

``custom_kernel(data) -> (H, tau)`` mirrors the reference's submission entry
(official/submission.py:5-6, submissions/candidate.py:8383-8415): a CUDA
float32 tensor ``[batch, n, n]`` goes in; ``H`` (same shape, column-major per
matrix, strides ``(n*n, 1, n)`` like torch.geqrf) and ``tau`` (``[batch, n]``)
come out, with torch.geqrf's values.  ``geqrf`` is the same call with a
torch.geqrf-like name and optional preallocated outputs.

Everything runs on the caller's current CUDA stream through the C ABI
(``fqr_geqrf_f32``).  There is no CPU or torch.geqrf fallback: a CPU tensor,
a wrong dtype or a failing kernel raises.
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import FastQRError, load


def _check_input(a: torch.Tensor, square: bool = True) -> torch.Tensor:
    if not isinstance(a, torch.Tensor):
        raise TypeError("input must be a torch.Tensor")
    if a.device.type != "cuda":
        raise ValueError("fastqr runs on CUDA tensors only (no CPU fallback)")
    if a.dtype != torch.float32:
        raise ValueError(f"input dtype must be torch.float32, got {a.dtype}")
    if a.ndim == 2:
        a = a.unsqueeze(0)
    if square and (a.ndim != 3 or a.shape[-1] != a.shape[-2]):
        raise ValueError(f"input must have shape (batch, n, n), got {tuple(a.shape)}")
    if not square and a.ndim != 3:
        raise ValueError(f"input must have shape (batch, m, n), got {tuple(a.shape)}")
    return a


def workspace_bytes(batch: int, n: int, m: int | None = None) -> int:
    """Device workspace of geqrf for (batch, n, n), or for (batch, m, n) when
    ``m`` is given."""
    if m is None or m == n:
        return int(load().fqr_workspace_bytes(batch, n))
    return int(load().fqr_geqrf_rect_workspace_bytes(batch, m, n))


def plan(batch: int, n: int) -> str:
    buf = ctypes.create_string_buffer(256)
    rc = load().fqr_plan_describe(batch, n, buf, 256)
    if rc:
        raise FastQRError(rc, "fqr_plan_describe")
    return buf.value.decode()


def launch_count(batch: int, n: int) -> int:
    return int(load().fqr_launch_count(batch, n))


def empty_outputs(batch: int, n: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """Column-major H (strides (n*n, 1, n)) and contiguous tau, as torch.geqrf
    returns them (reference allocator: submissions/candidate.py:3752-3798)."""
    h = torch.empty_strided((batch, n, n), (n * n, 1, n), device=device, dtype=torch.float32)
    tau = torch.empty((batch, n), device=device, dtype=torch.float32)
    return h, tau


def geqrf(a: torch.Tensor, *, out: tuple[torch.Tensor, torch.Tensor] | None = None,
          workspace: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Batched Householder QR of float32 CUDA matrices, square (batch, n, n)
    (``fqr_geqrf_f32``), tall (batch, m, n) with m > n or wide with m < n
    (``fqr_geqrf_rect_f32``).

    Returns ``(H, tau)`` as torch.geqrf does: H (batch, m, n) column-major
    (strides (m*n, 1, m)), tau (batch, min(m, n)).  ``out`` may supply
    preallocated outputs of that layout; ``workspace`` a uint8 CUDA tensor of
    at least ``workspace_bytes(batch, n, m)`` bytes.
    """
    squeeze = a.ndim == 2
    a = _check_input(a, square=False)
    batch, m, n = a.shape
    k = min(m, n)
    lib = load()
    if out is None:
        h = torch.empty_strided((batch, m, n), (m * n, 1, m), device=a.device, dtype=torch.float32)
        tau = torch.empty((batch, k), device=a.device, dtype=torch.float32)
    else:
        h, tau = out
        if h.shape != (batch, m, n) or h.stride() != (m * n, 1, m) or h.dtype != torch.float32:
            raise ValueError("out H must be float32 (batch, m, n) with strides (m*n, 1, m)")
        if tau.shape != (batch, k) or not tau.is_contiguous() or tau.dtype != torch.float32:
            raise ValueError("out tau must be contiguous float32 (batch, min(m, n))")
        if h.device != a.device or tau.device != a.device:
            raise ValueError("outputs must be on the input's device")
    # a wide block's library call writes tau [batch][n] (the first m per row)
    tau_lib = tau if m >= n else torch.empty((batch, n), device=a.device, dtype=torch.float32)
    need = workspace_bytes(batch, n, m)
    if need:
        if workspace is None:
            workspace = torch.empty(need, dtype=torch.uint8, device=a.device)
        elif workspace.numel() * workspace.element_size() < need or workspace.device != a.device:
            raise ValueError(f"workspace needs {need} bytes on {a.device}")
        ws_ptr, ws_len = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    else:
        ws_ptr, ws_len = None, 0
    with torch.cuda.device(a.device):
        stream = torch.cuda.current_stream(a.device).cuda_stream
        bs, rs, cs = a.stride()
        if m == n:
            rc = lib.fqr_geqrf_f32(a.data_ptr(), batch, n, bs, rs, cs, h.data_ptr(), tau.data_ptr(),
                                   ws_ptr, ws_len, stream)
        else:
            rc = lib.fqr_geqrf_rect_f32(a.data_ptr(), batch, m, n, bs, rs, cs, h.data_ptr(), tau_lib.data_ptr(),
                                        ws_ptr, ws_len, stream)
    if rc:
        raise FastQRError(rc)
    if tau_lib is not tau:
        tau.copy_(tau_lib[:, :m])
    if squeeze:
        return h[0], tau[0]
    return h, tau


def _colmajor(t: torch.Tensor) -> torch.Tensor:
    """The batch with each matrix column-major (strides (rows*cols, 1, rows)), a copy if needed."""
    b, r, c = t.shape
    if t.stride() == (r * c, 1, r):
        return t
    return t.transpose(1, 2).contiguous().transpose(1, 2)


def _check_factors(h: torch.Tensor, tau: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    h = _check_input(h)
    batch, n, _ = h.shape
    if tau.device != h.device or tau.dtype != torch.float32 or tuple(tau.shape[-1:]) != (n,):
        raise ValueError("tau must be a float32 (batch, n) tensor on H's device")
    return _colmajor(h), tau.reshape(batch, n).contiguous()


def _apply_workspace(lib, batch, n, workspace, device):
    """(pointer, bytes) of the S-block workspace for orgqr/ormqr; allocated when not given."""
    need = int(lib.fqr_orgqr_workspace_bytes(batch, n))
    if not need:
        return None, 0
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=device)
    elif workspace.numel() * workspace.element_size() < need or workspace.device != device:
        raise ValueError(f"workspace needs {need} bytes on {device}")
    return workspace.data_ptr(), workspace.numel() * workspace.element_size()


def orgqr_workspace_bytes(batch: int, n: int) -> int:
    return int(load().fqr_orgqr_workspace_bytes(batch, n))


def householder_product(h: torch.Tensor, tau: torch.Tensor, *, out: torch.Tensor | None = None,
                        workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Q = H_0 H_1 ... H_{n-1} from geqrf's compact (H, tau), as
    ``torch.linalg.householder_product(H, tau)`` for square float32 CUDA
    batches (``fqr_orgqr_f32``).  Q is returned column-major per matrix
    (``out``, when given, must be such a tensor)."""
    squeeze = h.ndim == 2
    h, tau = _check_factors(h, tau)
    batch, n, _ = h.shape
    if out is None:
        q = torch.empty_strided((batch, n, n), (n * n, 1, n), device=h.device, dtype=torch.float32)
    else:
        q = out.unsqueeze(0) if out.ndim == 2 else out
        if q.shape != (batch, n, n) or q.stride() != (n * n, 1, n) or q.dtype != torch.float32 \
                or q.device != h.device:
            raise ValueError("out must be float32 (batch, n, n) with strides (n*n, 1, n) on H's device")
    lib = load()
    ws_ptr, need = _apply_workspace(lib, batch, n, workspace, h.device)
    with torch.cuda.device(h.device):
        stream = torch.cuda.current_stream(h.device).cuda_stream
        rc = lib.fqr_orgqr_f32(h.data_ptr(), tau.data_ptr(), batch, n, q.data_ptr(), ws_ptr, need, stream)
    if rc:
        raise FastQRError(rc, "fqr_orgqr_f32")
    return q[0] if squeeze else q


def ormqr(h: torch.Tensor, tau: torch.Tensor, c: torch.Tensor, *, left: bool = True, transpose: bool = False,
          out: torch.Tensor | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """op(Q) C (``left=True``) or C op(Q) (``left=False``), op(Q) = Q or Q^T
    with ``transpose=True``, for the Q of geqrf's square (H, tau), as
    ``torch.ormqr(H, tau, C, left=left, transpose=transpose)`` for float32
    CUDA batches.  Left: C (batch, n, ncols), the result column-major
    (``fqr_ormqr_f32``).  Right: C (batch, mrows, n), the result row-major,
    torch's default layout (``fqr_ormqr_right_f32``).  ``out`` when given must
    have that layout (C itself for an in-place update)."""
    squeeze = h.ndim == 2
    h, tau = _check_factors(h, tau)
    batch, n, _ = h.shape
    if c.ndim == 2:
        c = c.unsqueeze(0)
    if c.device != h.device or c.dtype != torch.float32 or c.ndim != 3 or c.shape[0] != batch:
        raise ValueError("C must be a float32 (batch, rows, cols) tensor on H's device")
    if left:
        if c.shape[1] != n:
            raise ValueError("left: C must be (batch, n, ncols)")
        other = c.shape[2]
        shape, strides = (batch, n, other), (n * other, 1, n)
    else:
        if c.shape[2] != n:
            raise ValueError("right: C must be (batch, mrows, n)")
        other = c.shape[1]
        shape, strides = (batch, other, n), (other * n, n, 1)
    if out is None:
        out = torch.empty_strided(shape, strides, device=c.device, dtype=torch.float32)
    else:
        out = out.unsqueeze(0) if out.ndim == 2 else out
        if out.shape != shape or out.stride() != strides or out.dtype != torch.float32 or out.device != c.device:
            raise ValueError(f"out must be float32 {shape} with strides {strides} on C's device")
    if out.data_ptr() != c.data_ptr():
        out.copy_(c)
    lib = load()
    ws_ptr, need = _apply_workspace(lib, batch, n, workspace, h.device)
    fn, name = (lib.fqr_ormqr_f32, "fqr_ormqr_f32") if left else (lib.fqr_ormqr_right_f32, "fqr_ormqr_right_f32")
    with torch.cuda.device(h.device):
        stream = torch.cuda.current_stream(h.device).cuda_stream
        rc = fn(h.data_ptr(), tau.data_ptr(), batch, n, out.data_ptr(), other, 1 if transpose else 0, ws_ptr, need,
                stream)
    if rc:
        raise FastQRError(rc, name)
    return out[0] if squeeze else out


def host_workspace_bytes(batch: int, n: int) -> int:
    return int(load().fqr_host_workspace_bytes(batch, n))


def geqrf_host(a: torch.Tensor, *, out: tuple[torch.Tensor, torch.Tensor] | None = None,
               workspace: torch.Tensor | None = None, device=None,
               synchronize: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """Batched QR of a HOST float32 batch ``[batch, n, n]`` on a CUDA device.

    The result ``(H, tau)`` lands in host tensors with torch.geqrf's layout
    (page-locked when allocated here).  Chunks of the batch are uploaded,
    factored and downloaded on overlapping streams (``fqr_geqrf_f32_host``).
    ``a`` must hold each matrix as one dense row- or column-major block; pin it
    (``a.pin_memory()``) for the copies to overlap.  ``workspace`` is a uint8
    tensor on ``device`` of at least ``host_workspace_bytes(batch, n)`` bytes.
    With ``synchronize=False`` the call returns once the work is enqueued on
    the device's current stream; the outputs are valid after that stream has
    passed it.
    """
    if not isinstance(a, torch.Tensor):
        raise TypeError("input must be a torch.Tensor")
    if a.device.type != "cpu":
        raise ValueError("geqrf_host takes a host (CPU) tensor; use geqrf for CUDA tensors")
    if a.dtype != torch.float32:
        raise ValueError(f"input dtype must be torch.float32, got {a.dtype}")
    squeeze = a.ndim == 2
    if squeeze:
        a = a.unsqueeze(0)
    if a.ndim != 3 or a.shape[-1] != a.shape[-2]:
        raise ValueError(f"input must have shape (batch, n, n), got {tuple(a.shape)}")
    batch, n, _ = a.shape
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    lib = load()
    if out is None:
        h = torch.empty_strided((batch, n, n), (n * n, 1, n), dtype=torch.float32, pin_memory=True)
        tau = torch.empty((batch, n), dtype=torch.float32, pin_memory=True)
    else:
        h, tau = out
        if h.device.type != "cpu" or tau.device.type != "cpu":
            raise ValueError("geqrf_host outputs must be host tensors")
        if h.shape != (batch, n, n) or h.stride() != (n * n, 1, n) or h.dtype != torch.float32:
            raise ValueError("out H must be float32 (batch, n, n) with strides (n*n, 1, n)")
        if tau.shape != (batch, n) or not tau.is_contiguous() or tau.dtype != torch.float32:
            raise ValueError("out tau must be contiguous float32 (batch, n)")
    need = int(lib.fqr_host_workspace_bytes(batch, n))
    if need:
        if workspace is None:
            workspace = torch.empty(need, dtype=torch.uint8, device=dev)
        elif workspace.numel() * workspace.element_size() < need or workspace.device != dev:
            raise ValueError(f"workspace needs {need} bytes on {dev}")
        ws_ptr, ws_len = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    else:
        ws_ptr, ws_len = None, 0
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev)
        bs, rs, cs = a.stride()
        rc = lib.fqr_geqrf_f32_host(a.data_ptr(), batch, n, bs, rs, cs, h.data_ptr(),
                                    tau.data_ptr(), ws_ptr, ws_len, stream.cuda_stream)
        if rc:
            raise FastQRError(rc, "fqr_geqrf_f32_host")
        if synchronize:
            stream.synchronize()
    if squeeze:
        return h[0], tau[0]
    return h, tau


def host_check_status(workspace: torch.Tensor, batch: int, n: int) -> None:
    """Blocks on the current stream and raises if a chunk of the last
    geqrf_host that used ``workspace`` recorded a device-side wait that gave up."""
    stream = torch.cuda.current_stream(workspace.device).cuda_stream
    rc = load().fqr_host_check_status(workspace.data_ptr(),
                                      workspace.numel() * workspace.element_size(), batch, n, stream)
    if rc:
        raise FastQRError(rc, "fqr_host_check_status")


def check_status(workspace: torch.Tensor, batch: int) -> None:
    """Blocks on the current stream and raises if the last geqrf that used
    ``workspace`` recorded a device-side wait that gave up."""
    stream = torch.cuda.current_stream(workspace.device).cuda_stream
    rc = load().fqr_check_status(workspace.data_ptr(), workspace.numel() * workspace.element_size(),
                                 batch, stream)
    if rc:
        raise FastQRError(rc, "fqr_check_status")


def geqrf_profile(a: torch.Tensor, out, workspace) -> dict:
    """Run one geqrf with a CUDA event pair around every kernel (blocking).
    Returns the summed device milliseconds per kernel class."""
    from ._lib import STAGES

    a = _check_input(a)
    batch, n, _ = a.shape
    h, tau = out
    lib = load()
    ms = (ctypes.c_float * len(STAGES))()
    ws_ptr = workspace.data_ptr() if workspace is not None else None
    ws_len = workspace.numel() * workspace.element_size() if workspace is not None else 0
    with torch.cuda.device(a.device):
        stream = torch.cuda.current_stream(a.device).cuda_stream
        bs, rs, cs = a.stride()
        rc = lib.fqr_geqrf_f32_profile(a.data_ptr(), batch, n, bs, rs, cs, h.data_ptr(),
                                       tau.data_ptr(), ws_ptr, ws_len, stream, ms)
    if rc:
        raise FastQRError(rc, "fqr_geqrf_f32_profile")
    return {name: float(ms[i]) for i, name in enumerate(STAGES)}


def custom_kernel(data: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """The reference's submission contract: ``custom_kernel(data) -> (H, tau)``."""
    return geqrf(data)
