"""GPU: matrices holding NaN or Inf.

LAPACK's sgeqrf (torch.geqrf, the reference's CPU path) raises no error on
non-finite input: the values propagate into that matrix's H and tau.  fastqr
does the same, and because every matrix of a batch is factored on its own
(the plan depends only on (batch, n), never on values), a bad matrix leaves
its neighbours bitwise unchanged.  Covered: the warp-per-matrix path
(n <= 64), the rank-32 tensor-core path, the SIMT update for n % 4 != 0, and
the rank-64 plan with cluster panels (n = 2048).
"""
import pytest
import torch

import fastqr

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    fastqr.load()
    return torch.device("cuda:0")


@pytest.mark.parametrize("n,batch", [(32, 5), (64, 5), (256, 5), (600, 5), (1001, 4), (2048, 3)])
def test_nonfinite_matrix_stays_contained(dev, n, batch):
    g = torch.Generator().manual_seed(n)
    a = torch.randn(batch, n, n, generator=g)
    bad = a.clone()
    bad[1, n // 2, n // 3] = float("nan")  # one NaN inside the trailing part
    bad[2, 0, 0] = float("inf")            # an infinite first pivot
    h0, t0 = fastqr.geqrf(a.to(dev))
    h1, t1 = fastqr.geqrf(bad.to(dev))    # returns: no error for non-finite data
    torch.cuda.synchronize()
    for i in range(batch):
        if i in (1, 2):
            assert not bool(torch.isfinite(h1[i]).all()), f"matrix {i}: non-finite input gave finite H"
        else:
            assert torch.equal(h1[i], h0[i]) and torch.equal(t1[i], t0[i]), f"matrix {i} changed"
    # the clean matrices' results are themselves finite
    assert bool(torch.isfinite(h0).all()) and bool(torch.isfinite(t0).all())
