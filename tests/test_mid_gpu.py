"""GPU tests of the one-launch mid-size kernel (128 <= n <= 256, n % 4 == 0):
one CTA per matrix runs the copy-in, every panel and every tensor-core
trailing update of its matrix.  The static plan takes the blocked path for
these sizes (measured faster); the module selects the kernel with the
diagnostic override fqr_debug_plan(1) and restores the plan afterwards.

Parity against the CPU oracle per column (1e-3 of float64 on well-conditioned
inputs, the north star's tolerance) and the QR gates, at every n the path takes
(including partial last panels and row blocks), at batch sizes around the
two-CTAs-per-SM residency (296 on 148 SMs), with strided inputs, and through
the bounded-wait failure path, which a test hook drives without any fault.
"""
import pytest
import torch

import fastqr
import oracle
from fastqr import inputs
from oracle import checker

from gpu_gates import column_errors, gates

pytestmark = pytest.mark.gpu
COL_TOL = 1e-3
FQR_ETIMEOUT = 4


@pytest.fixture(scope="module", autouse=True)
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    lib = fastqr.load()
    lib.fqr_debug_plan(1)
    yield torch.device("cuda:0")
    lib.fqr_debug_plan(0)


@pytest.mark.parametrize("n", [128, 132, 144, 160, 172, 176, 192, 196, 224, 228, 252, 256])
def test_mid_sizes_against_oracle(n, dev):
    assert fastqr.plan(3, n).startswith("mid")
    a = inputs.generate_input(3, n, 1, 3000 + n, device="cpu")
    h, t = fastqr.geqrf(a.to(dev))
    torch.cuda.synchronize()
    hn, tn = h.cpu().numpy(), t.cpu().numpy()
    h64, t64 = oracle.geqrf_f64(a.numpy())
    ok, msg = checker.check_columns(hn, tn, h64, t64, COL_TOL)
    assert ok, (n, msg)
    rep = checker.check_qr(a.numpy(), hn, tn)
    assert rep.ok, (n, rep.message)
    assert (tn[:, -1] == 0.0).all()


@pytest.mark.parametrize("case", list(inputs.CASES))
def test_mid_every_conditioning_profile(case, dev):
    # the reference generator's profiles (graded, near rank, ...) at n = 256;
    # residual gates for all, per column for the well-conditioned ones
    n = 256
    cond = 0 if case in ("rankdef", "clustered", "nearrank", "band", "rowscale", "nearcollinear") else 2
    a = inputs.generate_input(4, n, cond, 77, case=case, device=dev)
    h, t = fastqr.geqrf(a)
    g = gates(a, h, t)
    assert g["ok"], (case, g)


@pytest.mark.parametrize("batch", [1, 2, 295, 296, 297, 600])
def test_mid_batch_sizes(batch, dev):
    # one CTA per matrix, two per SM: batches below, at and above one wave
    n = 256
    a = inputs.generate_input(batch, n, 0, 11 + batch, device=dev)
    h, t = fastqr.geqrf(a)
    pick = sorted({0, batch // 2, batch - 1})
    h64, t64 = torch.geqrf(a[pick].double())
    he, te = column_errors(h[pick], t[pick], h64, t64)
    assert float(he.max()) <= COL_TOL and float(te.max()) <= COL_TOL
    assert gates(a[pick], h[pick], t[pick])["ok"]


def test_mid_strided_and_column_major_inputs(dev):
    n = 192
    base = inputs.generate_input(5, n, 1, 5, device=dev)
    h0, t0 = fastqr.geqrf(base)
    # column-major input and a batch-strided view give the same bits
    cm = base.transpose(1, 2).contiguous().transpose(1, 2)
    h1, t1 = fastqr.geqrf(cm)
    wide = torch.zeros(5, n, n + 8, device=dev)
    wide[:, :, :n] = base
    h2, t2 = fastqr.geqrf(wide[:, :, :n])
    assert torch.equal(h0, h1) and torch.equal(t0, t1)
    assert torch.equal(h0, h2) and torch.equal(t0, t2)


def test_mid_is_deterministic(dev):
    a = inputs.generate_input(8, 256, 1, 9, device=dev)
    h0, t0 = fastqr.geqrf(a)
    h1, t1 = fastqr.geqrf(a)
    assert torch.equal(h0, h1) and torch.equal(t0, t1)


def test_mid_special_matrices(dev):
    n = 256
    eye = torch.eye(n, device=dev).expand(2, n, n).contiguous()
    zero = torch.zeros(2, n, n, device=dev)
    diag = torch.diag_embed(torch.linspace(-3, 5, n, device=dev)).expand(2, n, n).contiguous()
    for a in (eye, zero, diag):
        # exactly zero tails: tau = 0 and H = A (LAPACK)
        h, t = fastqr.geqrf(a)
        assert torch.equal(h, a) and torch.count_nonzero(t) == 0


@pytest.mark.parametrize("scale", [1e-30, 1e-12, 1e12, 1e30])
def test_mid_extreme_scales(scale, dev):
    # outside the fast envelope every column takes the LAPACK-order path
    a = inputs.generate_input(2, 256, 0, 21, device=dev) * scale
    h, t = fastqr.geqrf(a)
    h64, t64 = torch.geqrf(a.double())
    he, te = column_errors(h, t, h64, t64)
    assert float(he.max()) <= COL_TOL and float(te.max()) <= COL_TOL, (scale, float(he.max()))


def test_mid_profile_reports_one_kernel(dev):
    a = inputs.generate_input(16, 256, 0, 1, device=dev)
    h, t = fastqr.empty_outputs(16, 256, dev)
    ws = torch.empty(fastqr.workspace_bytes(16, 256), dtype=torch.uint8, device=dev)
    st = fastqr.geqrf_profile(a, (h, t), ws)
    assert st["mid"] > 0 and st["panel"] == 0 and st["trailing"] == 0 and st["copy_in"] == 0


@pytest.mark.parametrize("plan", [1, 0])
def test_bounded_wait_gives_up_and_reports_timeout(plan, dev):
    """The failure path, without a fault: the test hook makes the first
    tensor-core wait of every CTA use a barrier that nothing completes (2 ms
    limit).  The CTA then lets its copies in flight land, frees its tensor
    memory and exits; fqr_check_status reports FQR_ETIMEOUT.  The next normal
    call clears the status and is correct.  plan 1: the one-launch kernel;
    plan 0: the static plan (the blocked path's rank-32 tcgen05 update)."""
    lib = fastqr.load()
    assert lib.fqr_debug_plan(plan) == 1
    try:
        _timeout_then_recover(lib, dev)
    finally:
        lib.fqr_debug_plan(1)


def _timeout_then_recover(lib, dev):
    n, batch = 256, 4
    a = inputs.generate_input(batch, n, 0, 3, device=dev)
    h, t = fastqr.empty_outputs(batch, n, dev)
    ws = torch.empty(fastqr.workspace_bytes(batch, n), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    assert lib.fqr_debug_force_timeout(1) == 0
    try:
        fastqr.geqrf(a, out=(h, t), workspace=ws)
        rc = lib.fqr_check_status(ws.data_ptr(), ws.numel(), batch, stream)
    finally:
        assert lib.fqr_debug_force_timeout(0) == 1
    assert rc == FQR_ETIMEOUT
    fastqr.geqrf(a, out=(h, t), workspace=ws)
    assert lib.fqr_check_status(ws.data_ptr(), ws.numel(), batch, stream) == 0
    h64, t64 = torch.geqrf(a.double())
    he, te = column_errors(h, t, h64, t64)
    assert float(he.max()) <= COL_TOL and float(te.max()) <= COL_TOL
