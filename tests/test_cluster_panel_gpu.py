"""GPU tests of the cluster panels (panels taller than 1024 rows: a
thread-block cluster of 512-row CTAs whose per-column partial sums cross the
cluster through distributed shared memory between cluster barriers).

Parity per column against float64 geqrf at heights that give clusters of 3
to 8 CTAs (ragged last CTAs included), and the QR gates through the robust
path (exactly zero and repeated columns, tiny scales)."""
import pytest
import torch

import fastqr
from fastqr import inputs

from gpu_gates import column_errors, gates

pytestmark = pytest.mark.gpu
COL_TOL = 1e-3


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    fastqr.load()
    return torch.device("cuda:0")


@pytest.mark.parametrize("n,batch", [(1028, 2), (1300, 1), (1600, 3), (2052, 1), (4096, 1)])
def test_cluster_panels_against_float64(n, batch, dev):
    assert "cluster" in fastqr.plan(batch, n)
    a = inputs.generate_input(batch, n, 1, 4000 + n, device=dev)
    h, t = fastqr.geqrf(a)
    assert gates(a, h, t, chunk=1)["ok"]
    h64, t64 = torch.geqrf(a.double())
    he, te = column_errors(h, t, h64, t64)
    assert float(he.max()) <= COL_TOL and float(te.max()) <= COL_TOL, (float(he.max()), float(te.max()))


def test_cluster_panels_robust_path(dev):
    """Columns that take the LAPACK-order path inside cluster panels: an
    exactly zero block, exactly repeated columns, and a 1e-30 scale (the
    squares underflow in float32); the QR gates on each."""
    n = 1300
    g = torch.Generator().manual_seed(11)
    a = torch.randn(3, n, n, generator=g)
    a[0, :, 40:100] = 0.0
    a[1, :, 200:260] = a[1, :, 0:60]
    a[2] *= 1e-30
    a = a.to(dev)
    h, t = fastqr.geqrf(a)
    assert gates(a, h, t, chunk=1)["ok"]
