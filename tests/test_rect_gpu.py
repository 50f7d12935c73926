"""GPU parity of the rectangular entry (fqr_geqrf_rect_f32, fastqr.geqrf on
(batch, m, n) with m > n) against the CPU oracle's m x n xGEQR2 restatement
in float64 (pinned to numpy's LAPACK in tests/test_oracle.py), and the QR
gates.  The reference calls torch.geqrf on such tall blocks
(submissions/candidate.py:7204-7214).

Tolerances: per-column relative error of H and tau <= 1e-3 against float64
on well-conditioned N(0,1) inputs; ||A - QR||_F / ||A||_F <= 1e-4 and
||Q^T Q - I||_F / sqrt(n) <= 1e-4 (Q the m x n thin factor).
"""
import ctypes

import numpy as np
import pytest
import torch

import fastqr
import oracle
from fastqr import inputs
from gpu_gates import column_errors, gates

pytestmark = pytest.mark.gpu

COL_TOL = 1e-3

# small m (panel rows <= 128, SIMT update), m % 4 != 0 (SIMT update),
# tensor-core update, clusters of panels (m > 1024), one panel (n <= 32)
SHAPES = [(48, 32), (64, 17), (100, 64), (130, 96), (301, 256), (300, 256), (512, 384),
          (1000, 128), (1500, 40), (2100, 96), (257, 250)]


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    fastqr.load()
    return torch.device("cuda:0")


def tall(batch, m, n, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(batch, m, n, generator=g, dtype=torch.float32)


@pytest.mark.parametrize("m,n", SHAPES)
def test_rect_matches_oracle(m, n, dev):
    a = tall(3, m, n, 1000 * m + n)
    h, t = fastqr.geqrf(a.to(dev))
    torch.cuda.synchronize()
    assert h.shape == (3, m, n) and h.stride() == (m * n, 1, m) and t.shape == (3, n)
    h64, t64 = oracle.geqrf_rect_f64(a.numpy())
    he, te = column_errors(h.cpu(), t.cpu(), torch.from_numpy(np.ascontiguousarray(h64)),
                           torch.from_numpy(t64))
    assert float(he.max()) <= COL_TOL and float(te.max()) <= COL_TOL, (float(he.max()), float(te.max()))
    g = gates(a.to(dev), h, t, chunk=3)
    assert g["ok"], g


@pytest.mark.parametrize("m,n", [(1024, 512), (4096, 256), (2304, 2080)])
def test_rect_large_gates(m, n, dev):
    """Large tall blocks; 2304 x 2080 takes the rank-64 plan (32 blocks of 64
    columns, then one 32-column panel), checked per column against float64
    geqrf too."""
    a = tall(2, m, n, 77 + n).to(dev)
    h, t = fastqr.geqrf(a)
    g = gates(a, h, t, chunk=1)
    assert g["ok"], g
    if n >= 2048:
        h64, t64 = torch.geqrf(a.double())
        he, te = column_errors(h, t, h64, t64)
        assert float(he.max()) <= COL_TOL and float(te.max()) <= COL_TOL, (float(he.max()), float(te.max()))


def test_rect_batch_split_and_strides(dev):
    """A matrix factored within a batch and on its own gives bitwise the same
    result (large batches run as parts on several streams); a column-major
    input takes the strided copy-in."""
    a = tall(5, 300, 200, 9).to(dev)
    h, t = fastqr.geqrf(a)
    h1, t1 = fastqr.geqrf(a[3:4])
    assert torch.equal(h[3:4], h1) and torch.equal(t[3:4], t1)
    acm = a.transpose(1, 2).contiguous().transpose(1, 2)  # column-major copy
    h2, t2 = fastqr.geqrf(acm)
    assert torch.equal(h, h2) and torch.equal(t, t2)


def test_rect_entry_with_square_shape_is_the_square_path(dev):
    a = tall(4, 160, 160, 5).to(dev)
    h, t = fastqr.geqrf(a)
    lib = fastqr.load()
    h2 = torch.empty_strided((4, 160, 160), (160 * 160, 1, 160), device=dev)
    t2 = torch.empty(4, 160, device=dev)
    ws = torch.empty(fastqr.workspace_bytes(4, 160, 160), dtype=torch.uint8, device=dev)
    bs, rs, cs = a.stride()
    rc = lib.fqr_geqrf_rect_f32(a.data_ptr(), 4, 160, 160, bs, rs, cs, h2.data_ptr(), t2.data_ptr(),
                                ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == 0
    assert torch.equal(h, h2) and torch.equal(t, t2)


def test_rect_embedded_route_shape(dev):
    """The reference's embedded route: geqrf of the first `cols` columns of
    square matrices (a strided view, no copy)."""
    a = tall(4, 512, 512, 3).to(dev)
    cols = 384
    h, t = fastqr.geqrf(a[:, :, :cols])
    h64, t64 = oracle.geqrf_rect_f64(a[:, :, :cols].cpu().numpy())
    he, te = column_errors(h.cpu(), t.cpu(), torch.from_numpy(np.ascontiguousarray(h64)),
                           torch.from_numpy(t64))
    assert float(he.max()) <= COL_TOL and float(te.max()) <= COL_TOL
    # the leading columns of the square factorisation are the same reflectors
    hs, ts = fastqr.geqrf(a)
    assert float((hs[:, :, :cols] - h).abs().max()) <= 1e-4 * float(hs.abs().max())


@pytest.mark.parametrize("m,n", [(20, 32), (96, 130), (128, 256), (200, 512), (256, 300)])
def test_wide_blocks_match_lapack(m, n, dev):
    """Wide blocks (m < n): LAPACK xGEQRF's result -- m reflectors from the
    first m columns, the rest of R = Q^T A[:, m:] -- against float64 geqrf
    (torch on the CPU, i.e. LAPACK): per column 1e-3 on H's reflector columns
    and tau, and ||A - Q R||_F / ||A||_F <= 1e-4 with R the m x n upper part."""
    a = inputs.generate_input(3, max(m, n), 1, 40 + m + n, device="cpu")[:, :m, :n].contiguous()
    h, tau = fastqr.geqrf(a.to(dev))
    torch.cuda.synchronize()
    assert h.shape == (3, m, n) and h.stride() == (m * n, 1, m) and tau.shape == (3, m)
    h64, t64 = torch.geqrf(a.double())
    he, te = column_errors(h[:, :, :m].cpu(), tau.cpu(), h64[:, :, :m], t64)
    assert float(he.max()) <= 1e-3 and float(te.max()) <= 1e-3, (float(he.max()), float(te.max()))
    q = torch.linalg.householder_product(h[:, :, :m].double(), tau.double())
    r = torch.triu(h.double())
    rec = ((q @ r - a.double().to(dev)).flatten(1).norm(dim=1) / a.double().flatten(1).norm(dim=1).to(dev)).max()
    assert float(rec) <= 1e-4, float(rec)
