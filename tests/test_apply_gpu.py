"""GPU parity of Q formation (fqr_orgqr_f32, fastqr.householder_product) and
Q application (fqr_ormqr_f32, fastqr.ormqr) against the CPU oracle's xORG2R
restatement in float64 and against torch's own CUDA implementations, on
factors from fastqr.geqrf.

Tolerances: ||Q - Q64||_F / sqrt(n) <= 1e-5 (Q has unit columns); Q^T C and
Q C within 1e-5 relative (Frobenius) of the float64 products; orthogonality
||Q^T Q - I||_F / sqrt(n) <= 1e-4 and reconstruction ||A - Q R||_F / ||A||_F
<= 1e-4 as for geqrf.
"""
import numpy as np
import pytest
import torch

import fastqr
import oracle
from fastqr import inputs

pytestmark = pytest.mark.gpu

# small path (n % 4 != 0 or n < 128, up to 512), tensor-core path sizes, and
# the blocked SIMT path (n > 512 off the tensor-core path: 514, 601)
SIZES = [1, 8, 33, 64, 100, 130, 128, 256, 260, 384, 512, 514, 601]


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    fastqr.load()
    return torch.device("cuda:0")


def factor(batch, n, cond, seed, dev):
    a = inputs.generate_input(batch, n, cond, seed, device="cpu")
    h, tau = fastqr.geqrf(a.to(dev))
    return a, h, tau


def frob(x):
    return float(np.linalg.norm(x.reshape(x.shape[0], -1), axis=1).max())


@pytest.mark.parametrize("n", SIZES)
def test_householder_product_matches_oracle(dev, n):
    a, h, tau = factor(3, n, 2, 100 + n, dev)
    q = fastqr.householder_product(h, tau)
    torch.cuda.synchronize()
    assert q.stride() == (n * n, 1, n)
    q64 = oracle.orgqr_f64(h.cpu().numpy(), tau.cpu().numpy())
    err = frob(q.cpu().double().numpy() - q64) / np.sqrt(n)
    assert err <= 1e-5, err
    # the same product from torch's CUDA implementation
    qt = torch.linalg.householder_product(h, tau)
    assert frob((q - qt).cpu().double().numpy()) / np.sqrt(n) <= 1e-5


@pytest.mark.parametrize("n,batch", [(256, 8), (1024, 2), (1000, 2)])
def test_q_is_orthogonal_and_reconstructs(dev, n, batch):
    a, h, tau = factor(batch, n, 0, 7, dev)
    q = fastqr.householder_product(h, tau)
    r = torch.triu(h)
    eye = torch.eye(n, device=dev)
    orth = torch.linalg.matrix_norm(q.transpose(1, 2) @ q - eye) / n ** 0.5
    rec = torch.linalg.matrix_norm(a.to(dev) - q @ r) / torch.linalg.matrix_norm(a.to(dev))
    assert float(orth.max()) <= 1e-4
    assert float(rec.max()) <= 1e-4


@pytest.mark.parametrize("n,ncols", [(64, 7), (130, 1), (256, 64), (256, 300), (512, 129), (514, 200), (601, 37)])
@pytest.mark.parametrize("transpose", [True, False])
def test_ormqr_matches_oracle(dev, n, ncols, transpose):
    a, h, tau = factor(2, n, 1, 40 + n, dev)
    g = torch.Generator().manual_seed(n + ncols)
    c = torch.randn(2, n, ncols, generator=g)
    out = fastqr.ormqr(h, tau, c.to(dev), transpose=transpose)
    torch.cuda.synchronize()
    q64 = oracle.orgqr_f64(h.cpu().numpy(), tau.cpu().numpy())
    c64 = c.double().numpy()
    want = np.transpose(q64, (0, 2, 1)) @ c64 if transpose else q64 @ c64
    err = frob(out.cpu().double().numpy() - want) / frob(want)
    assert err <= 1e-5, err
    # torch's CUDA ormqr on the same factors
    ref = torch.ormqr(h, tau, c.to(dev), left=True, transpose=transpose)
    assert frob((out - ref).cpu().double().numpy()) / frob(want) <= 1e-5


def test_ormqr_round_trip(dev):
    a, h, tau = factor(4, 384, 3, 11, dev)
    c = torch.randn(4, 384, 50, device=dev)
    back = fastqr.ormqr(h, tau, fastqr.ormqr(h, tau, c, transpose=True), transpose=False)
    assert float((back - c).abs().max()) <= 1e-4


def test_qt_a_is_r(dev):
    """Q^T A equals R (upper triangle of H) -- ormqr undoes the factorisation."""
    a, h, tau = factor(2, 512, 0, 5, dev)
    qta = fastqr.ormqr(h, tau, a.to(dev), transpose=True)
    r = torch.triu(h)
    err = torch.linalg.matrix_norm(qta - r) / torch.linalg.matrix_norm(r)
    assert float(err.max()) <= 1e-5
    below = torch.tril(qta, diagonal=-1)
    assert float(below.abs().max()) <= 1e-4 * float(r.abs().max())


def test_row_major_factors_and_errors(dev):
    a, h, tau = factor(2, 128, 0, 3, dev)
    q1 = fastqr.householder_product(h, tau)
    q2 = fastqr.householder_product(h.contiguous(), tau)  # row-major copy of H
    assert torch.equal(q1, q2)
    with pytest.raises(fastqr.FastQRError):  # n above FQR_MAX_N
        hb = torch.zeros(1, 8200, 8200, device=dev)
        fastqr.householder_product(hb, torch.zeros(1, 8200, device=dev))
    with pytest.raises(ValueError):
        fastqr.ormqr(h, tau, torch.zeros(2, 127, 3, device=dev))


def test_column_range_update_leaves_other_columns(dev):
    """ormqr on a C wider than one 128-column tile but not a multiple of 32
    columns: every column is updated and none is written twice (the update
    kernel stores only the quarters of its column range)."""
    a, h, tau = factor(1, 256, 0, 21, dev)
    c = torch.randn(1, 256, 200, device=dev)
    out = fastqr.ormqr(h, tau, c, transpose=True)
    q64 = oracle.orgqr_f64(h.cpu().numpy(), tau.cpu().numpy())
    want = np.transpose(q64, (0, 2, 1)) @ c.cpu().double().numpy()
    assert frob(out.cpu().double().numpy() - want) / frob(want) <= 1e-5


@pytest.mark.parametrize("n", [64, 100, 256, 384, 601])
@pytest.mark.parametrize("mrows", [1, 50, 256])
@pytest.mark.parametrize("transpose", [False, True])
def test_ormqr_right_side_matches_torch_float64(dev, n, mrows, transpose):
    """C Q and C Q^T (torch.ormqr with left=False, the reference's tail
    projection, submissions/candidate.py:7231) against float64 products with
    Q from the same factors: 1e-5 relative (Frobenius), result row-major."""
    a, h, tau = factor(2, n, 1, 300 + n + mrows, dev)
    c = torch.randn(2, mrows, n, generator=torch.Generator().manual_seed(n + mrows)).to(dev)
    out = fastqr.ormqr(h, tau, c, left=False, transpose=transpose)
    assert out.shape == (2, mrows, n) and out.stride() == (mrows * n, n, 1)
    q = torch.linalg.householder_product(h.double(), tau.double())
    want = c.double() @ (q.transpose(1, 2) if transpose else q)
    err = ((out.double() - want).flatten(1).norm(dim=1) / want.flatten(1).norm(dim=1)).max()
    assert float(err) <= 1e-5, float(err)
    # in place, and the round trip C Q Q^T = C
    back = fastqr.ormqr(h, tau, out, left=False, transpose=not transpose, out=out)
    assert back.data_ptr() == out.data_ptr()
    rt = ((back.double() - c.double()).flatten(1).norm(dim=1) / c.double().flatten(1).norm(dim=1)).max()
    assert float(rt) <= 1e-5, float(rt)


def test_unaligned_factors_take_the_simt_blocked_path(dev):
    """n = 640 with H and C one float off 16-byte alignment: the tensor-core
    update cannot take them, so Q, Q^T C and Q C come from the blocked SIMT
    path; they agree with the aligned (tensor-core) results to 1e-5."""
    n, batch = 640, 2
    a, h, tau = factor(batch, n, 0, 17, dev)
    buf = torch.empty(batch * n * n + 1, device=dev)
    hs = buf[1:].as_strided((batch, n, n), (n * n, 1, n))
    hs.copy_(h)
    assert hs.data_ptr() % 16 != 0
    q = fastqr.householder_product(h, tau)
    qs = fastqr.householder_product(hs, tau)
    assert float((qs - q).abs().max()) <= 1e-5
    c = torch.randn(batch, n, 70, device=dev)
    cbuf = torch.empty(batch * n * 70 + 1, device=dev)
    cs = cbuf[1:].as_strided((batch, n, 70), (n * 70, 1, n))
    for transpose in (True, False):
        want = fastqr.ormqr(h, tau, c, transpose=transpose)
        cs.copy_(c)
        got = fastqr.ormqr(hs, tau, cs, transpose=transpose, out=cs)
        assert got.data_ptr() % 16 != 0
        err = torch.linalg.matrix_norm(got - want) / torch.linalg.matrix_norm(want)
        assert float(err.max()) <= 1e-5, float(err.max())
