"""The C-ABI library loads and exports every declared symbol (CPU only:
no call here reaches the GPU; argument validation returns before any CUDA
call)."""
import ctypes
import re
from pathlib import Path

import pytest

import fastqr
from fastqr import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "fastqr.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(fqr_\w+)\s*\(", text)))


def test_header_declares_the_bound_symbols():
    assert declared_symbols() == sorted(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(fastqr.LIB_PATH))
    for name in declared_symbols():
        assert hasattr(lib, name), name
    fastqr.load()


def test_status_strings_and_version():
    lib = fastqr.load()
    for code in range(8):
        assert lib.fqr_status_string(code)
    assert lib.fqr_status_string(99) == b"unknown status"
    assert lib.fqr_version() >= 100


def test_argument_validation_without_gpu():
    lib = fastqr.load()
    # null pointers
    assert lib.fqr_geqrf_f32(None, 2, 8, 64, 8, 1, None, None, None, 0, None) == 1
    # negative sizes
    assert lib.fqr_geqrf_f32(None, -1, 8, 64, 8, 1, None, None, None, 0, None) == 1
    # empty problems are a no-op
    assert lib.fqr_geqrf_f32(None, 0, 8, 64, 8, 1, None, None, None, 0, None) == 0
    assert lib.fqr_geqrf_f32(None, 4, 0, 0, 0, 1, None, None, None, 0, None) == 0
    # n outside the dispatch table
    assert lib.fqr_geqrf_f32(None, 1, 8193, 1, 1, 1, None, None, None, 0, None) == 2
    # zero strides
    dummy = ctypes.c_void_p(16)
    assert lib.fqr_geqrf_f32(dummy, 1, 8, 64, 0, 1, dummy, dummy, None, 0, None) == 1
    # blocked path without workspace
    assert lib.fqr_geqrf_f32(dummy, 1, 100, 10000, 100, 1, dummy, dummy, None, 0, None) == 5


def test_workspace_and_plan_depend_on_shape_only():
    assert fastqr.workspace_bytes(1024, 32) == 0
    assert fastqr.workspace_bytes(256, 256) == 256 * 32 * 32 * 4 + 256  # T factors + status
    assert fastqr.workspace_bytes(3, 100) % 256 == 0
    assert fastqr.plan(1024, 32).startswith("small")
    assert fastqr.plan(256, 256).startswith("blocked")
    # the one-launch mid-size kernel only under the diagnostic override
    lib = fastqr.load()
    assert lib.fqr_debug_plan(1) == 0
    try:
        assert fastqr.plan(256, 256).startswith("mid") and fastqr.launch_count(256, 256) == 1
        assert fastqr.plan(3, 176).startswith("mid") and fastqr.plan(3, 130).startswith("blocked")
        assert fastqr.plan(3, 100).startswith("blocked") and fastqr.plan(3, 260).startswith("blocked")
    finally:
        assert lib.fqr_debug_plan(0) == 1
    assert "cluster 8" in fastqr.plan(16, 4096)
    with pytest.raises(fastqr.FastQRError):
        fastqr.plan(1, 10000)
    assert fastqr.launch_count(1024, 32) == 1
    # copy-in + 8 panels + 7 trailing; a batch runs as one part up to 64
    # matrices (n < 2048), else as two parts on two streams
    assert fastqr.launch_count(256, 256) == 2 * (1 + 8 + 7)
    assert fastqr.launch_count(64, 256) == 1 + 8 + 7
    assert fastqr.launch_count(1, 256) == 1 + 8 + 7
    # n >= 2048: rank-64 blocks (panel, in-block update, panel, then Gram
    # block + trailing update for all but the last block); four parts for
    # n >= 2048 above 140M elements (one part up to that): 32 blocks each
    assert "rank 64" in fastqr.plan(16, 4096) and "rank 32" in fastqr.plan(64, 1024)
    assert fastqr.launch_count(16, 2048) == 1 + 32 * 3 + 31 * 2
    assert fastqr.launch_count(3, 2048) == 1 + 32 * 3 + 31 * 2
    assert fastqr.launch_count(40, 2048) == 4 * (1 + 32 * 3 + 31 * 2)
    assert fastqr.launch_count(64, 1024) == 2 * (1 + 32 + 31)
    # 2100 = 32 blocks of 64 + a 32- and a 20-column panel (every block has a
    # trailing update, the first rank-32 panel too)
    assert fastqr.launch_count(1, 2100) == 1 + 32 * 3 + 32 * 2 + 2 + 1
    # rows above 4096: rank-32 steps only
    assert fastqr.launch_count(1, 8192) == 1 + 256 + 255
    # a status block, then one S block per matrix (64 x 64 for rank-64 plans)
    assert fastqr.workspace_bytes(16, 4096) == 256 + 16 * 64 * 64 * 4
    assert fastqr.workspace_bytes(64, 1024) == 256 + 64 * 32 * 32 * 4
    assert fastqr.workspace_bytes(2, 8192) == 256 + 2 * 32 * 32 * 4


def test_python_api_rejects_cpu_tensors():
    import torch
    with pytest.raises(ValueError):
        fastqr.geqrf(torch.zeros(2, 8, 8))


def test_host_entry_validation_without_gpu():
    lib = fastqr.load()
    dummy = ctypes.c_void_p(16)
    # empty problems are a no-op; negative sizes and null pointers are rejected
    assert lib.fqr_geqrf_f32_host(None, 0, 8, 64, 8, 1, None, None, None, 0, None) == 0
    assert lib.fqr_geqrf_f32_host(None, -1, 8, 64, 8, 1, None, None, None, 0, None) == 1
    assert lib.fqr_geqrf_f32_host(None, 2, 8, 64, 8, 1, None, None, None, 0, None) == 1
    assert lib.fqr_geqrf_f32_host(dummy, 1, 8193, 1, 1, 1, dummy, dummy, None, 0, None) == 2
    # each host matrix must be a dense row- or column-major block
    assert lib.fqr_geqrf_f32_host(dummy, 2, 8, 64, 16, 1, dummy, dummy, None, 0, None) == 1
    assert lib.fqr_geqrf_f32_host(dummy, 2, 8, 32, 8, 1, dummy, dummy, None, 0, None) == 1
    # no (or too little) device workspace
    assert lib.fqr_geqrf_f32_host(dummy, 2, 8, 64, 8, 1, dummy, dummy, None, 0, None) == 5
    need = lib.fqr_host_workspace_bytes(2, 8)
    assert lib.fqr_geqrf_f32_host(dummy, 2, 8, 64, 8, 1, dummy, dummy, dummy, need - 1, None) == 5


def test_host_workspace_plan():
    # one staging slot per chunk, at most 16 chunks, each >= 1 MiB of input
    # or 1/16 of the batch; sizes depend on (batch, n) only
    for batch, n in [(1024, 32), (256, 256), (512, 512), (64, 1024), (16, 4096), (1, 8), (3, 100)]:
        mat = n * n * 4
        need = fastqr.host_workspace_bytes(batch, n)
        assert need % 256 == 0
        assert need >= 2 * mat  # at least one A and one H staging block
        # about the batch's own size twice (A and H staging), at most 1.5x with
        # the slots rounded per chunk, plus per-slot S blocks
        assert need <= 256 + 1.5 * batch * (2 * mat + n * 4) + 16 * (fastqr.workspace_bytes(batch, n) + 1024)
    # C2: 16 chunks of 16 matrices, one slot each of (A + H + tau + S blocks)
    slot = 2 * 16 * 256 * 256 * 4 + 16 * 256 * 4 + fastqr.workspace_bytes(16, 256)
    assert fastqr.host_workspace_bytes(256, 256) == 256 + 16 * slot
    assert fastqr.host_workspace_bytes(0, 8) == 0


def test_host_api_rejects_cuda_tensors_and_bad_dtypes():
    import torch
    with pytest.raises(ValueError):
        fastqr.geqrf_host(torch.zeros(2, 8, 8, dtype=torch.float64))


def test_orgqr_ormqr_validation_without_gpu():
    lib = fastqr.load()
    dummy = ctypes.c_void_p(256)
    assert lib.fqr_orgqr_f32(None, None, -1, 8, None, None, 0, None) == 1
    assert lib.fqr_orgqr_f32(None, None, 0, 8, None, None, 0, None) == 0
    assert lib.fqr_orgqr_f32(dummy, dummy, 1, 8193, dummy, None, 0, None) == 2
    # blocked sizes (tensor-core ones, and every n above 512) need the S
    # workspace; sizes up to 512 off the tensor-core path need none
    assert lib.fqr_orgqr_f32(dummy, dummy, 2, 256, dummy, None, 0, None) == 5
    assert lib.fqr_orgqr_f32(dummy, dummy, 2, 514, dummy, None, 0, None) == 5
    assert fastqr.orgqr_workspace_bytes(2, 514) == 2 * 17 * 32 * 32 * 4 + 256
    assert fastqr.orgqr_workspace_bytes(2, 510) == 0
    assert lib.fqr_ormqr_f32(dummy, dummy, 2, 256, dummy, 10, 1, None, 0, None) == 5
    assert lib.fqr_ormqr_f32(None, dummy, 2, 256, dummy, 10, 1, None, 0, None) == 1
    # one 32 x 32 S block per panel per matrix + a status block
    assert fastqr.orgqr_workspace_bytes(16, 4096) == 16 * 128 * 4096 + 256
    assert fastqr.orgqr_workspace_bytes(3, 100) == 0


def test_rect_entry_validation_without_gpu():
    lib = fastqr.load()
    dummy = ctypes.c_void_p(16)
    # wide blocks (m < n) take the blocked path too: a workspace is required;
    # sizes beyond the table are unsupported
    assert lib.fqr_geqrf_rect_f32(dummy, 1, 8, 16, 128, 16, 1, dummy, dummy, None, 0, None) == 5
    assert fastqr.workspace_bytes(4, 100, 20) == 4 * 32 * 32 * 4 + 256
    assert lib.fqr_geqrf_rect_f32(dummy, 1, 8193, 16, 8193 * 16, 16, 1, dummy, dummy, None, 0, None) == 2
    # null pointers, negative sizes, empty problems
    assert lib.fqr_geqrf_rect_f32(None, 2, 100, 20, 2000, 20, 1, None, None, None, 0, None) == 1
    assert lib.fqr_geqrf_rect_f32(None, 2, -1, 20, 2000, 20, 1, None, None, None, 0, None) == 1
    assert lib.fqr_geqrf_rect_f32(None, 0, 100, 20, 2000, 20, 1, None, None, None, 0, None) == 0
    # tall matrices always take the blocked path: a workspace is required,
    # even for n <= 64
    assert lib.fqr_geqrf_rect_f32(dummy, 1, 100, 20, 2000, 20, 1, dummy, dummy, None, 0, None) == 5
    assert fastqr.workspace_bytes(4, 20, 100) == 4 * 32 * 32 * 4 + 256
    assert fastqr.workspace_bytes(4, 20, 20) == 0  # square n <= 64: the small path
    assert fastqr.workspace_bytes(4, 100, 100) == fastqr.workspace_bytes(4, 100)
    assert lib.fqr_geqrf_rect_workspace_bytes(4, 10, 20) == 4 * 32 * 32 * 4 + 256  # wide: blocked path


def test_python_geqrf_rejects_wide_input():
    import torch
    with pytest.raises(ValueError):
        fastqr.geqrf(torch.zeros(2, 8, 16))  # CPU tensor: rejected before any GPU call
