"""GPU: batches larger than a grid dimension.

CUDA caps a grid's y and z dimensions at 65,535, and the blocked path puts
the matrices of a launch there, so its launchers cut a batch into pieces of
at most 65,535 matrices.  A batch of two or more runs as two stream parts at
n < 2048, so a part passes that limit only beyond 131,070 matrices: 140,000
matrices here, at n = 100 (the SIMT update) and n = 128 (the tensor-core
update).  Matrices on both sides of every boundary (piece and part) are
checked with the official gates and against the same matrix factored alone,
and Q formed for the whole batch (fastqr.householder_product, whose
launchers cut batches the same way) against Q of the matrix alone.
"""
import pytest
import torch

import fastqr
from oracle import checker

pytestmark = pytest.mark.gpu

BATCH = 140_000


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    fastqr.load()
    return torch.device("cuda:0")


@pytest.mark.parametrize("n", [100, 128])
def test_batch_beyond_the_grid_limit(dev, n):
    g = torch.Generator(device=dev).manual_seed(n)
    a = torch.randn(BATCH, n, n, device=dev, generator=g)
    h, tau = fastqr.geqrf(a)
    torch.cuda.synchronize()
    half = BATCH // 2
    picks = [0, 1, 65_534, 65_535, 65_536, half - 1, half, half + 65_535, BATCH - 1]
    idx = torch.tensor(picks, device=dev)
    a_s, h_s, t_s = a[idx], h[idx], tau[idx]
    rep = checker.check_qr(a_s.cpu().numpy(), h_s.cpu().numpy(), t_s.cpu().numpy())
    assert rep.ok, rep.message
    for j, i in enumerate(picks):
        h1, t1 = fastqr.geqrf(a[i : i + 1])
        err = float((h1[0] - h_s[j]).abs().max() / h1[0].abs().max().clamp_min(1e-30))
        assert err <= 1e-5, (i, err)
        assert float((t1[0] - t_s[j]).abs().max()) <= 1e-5, i
    del a
    q = fastqr.householder_product(h, tau)
    torch.cuda.synchronize()
    for i in picks:
        q1 = fastqr.householder_product(h[i : i + 1], tau[i : i + 1])
        assert float((q1[0] - q[i]).abs().max()) <= 1e-5, i
