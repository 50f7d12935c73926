"""GPU: the host-buffer entry point (fqr_geqrf_f32_host) gives bitwise the
same H and tau as the device entry point on the same matrices up to n = 1024
-- both run the same kernels and plans, chunked over the batch -- for every
layout it accepts, with page-locked and pageable buffers, and composes with
the caller's stream.  For the rank-64 plan (n >= 2048) the two entries agree
to rounding (the last test)."""
import pytest
import torch

import fastqr
import oracle
from fastqr import inputs
from oracle import checker

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    fastqr.load()
    return torch.device("cuda:0")


def device_result(a_cpu, dev):
    h, t = fastqr.geqrf(a_cpu.to(dev))
    return h.cpu(), t.cpu()


@pytest.mark.parametrize("batch,n", [(1, 8), (5, 32), (300, 32), (7, 64), (9, 96), (33, 256),
                                      (4, 520), (3, 1024)])
def test_host_matches_device_entry(dev, batch, n):
    a = inputs.generate_input(batch, n, 2, 1234 + n, device="cpu").contiguous().pin_memory()
    h, t = fastqr.geqrf_host(a, device=dev)
    assert h.device.type == "cpu" and h.stride() == (n * n, 1, n)
    hd, td = device_result(a, dev)
    assert torch.equal(h, hd) and torch.equal(t, td)
    rep = checker.check_qr(a.numpy(), h.numpy(), t.numpy())
    assert rep.ok, rep.message


def test_host_column_major_and_gapped_batches(dev):
    n, batch = 128, 6
    base = inputs.generate_input(batch, n, 0, 77, device="cpu")
    want_h, want_t = device_result(base, dev)
    # column-major matrices
    cm = base.transpose(1, 2).contiguous().transpose(1, 2)
    assert cm.stride() == (n * n, 1, n)
    h, t = fastqr.geqrf_host(cm.pin_memory(), device=dev)
    assert torch.equal(h, want_h) and torch.equal(t, want_t)
    # a gap between matrices (batch stride > n*n)
    big = torch.zeros(batch, n * n + 40)
    big[:, : n * n] = base.reshape(batch, n * n)
    gapped = big.as_strided((batch, n, n), (n * n + 40, n, 1))
    h, t = fastqr.geqrf_host(gapped, device=dev)
    assert torch.equal(h, want_h) and torch.equal(t, want_t)


def test_host_pageable_buffers_and_preallocated_outputs(dev):
    n, batch = 256, 20
    a = inputs.generate_input(batch, n, 6, 5, device="cpu")  # pageable
    h = torch.empty_strided((batch, n, n), (n * n, 1, n))
    t = torch.empty(batch, n)
    ws = torch.empty(fastqr.host_workspace_bytes(batch, n), dtype=torch.uint8, device=dev)
    fastqr.geqrf_host(a, out=(h, t), workspace=ws, device=dev)
    hd, td = device_result(a, dev)
    assert torch.equal(h, hd) and torch.equal(t, td)
    fastqr.host_check_status(ws, batch, n)


def test_host_call_orders_with_caller_stream(dev):
    """Two asynchronous calls in a row on a side stream share one workspace:
    the second call's chunks wait for the first call's on the caller's stream,
    so both results come out right."""
    n, batch = 192, 40
    a1 = inputs.generate_input(batch, n, 0, 1, device="cpu").pin_memory()
    a2 = inputs.generate_input(batch, n, 3, 2, device="cpu").pin_memory()
    ws = torch.empty(fastqr.host_workspace_bytes(batch, n), dtype=torch.uint8, device=dev)
    outs = []
    side = torch.cuda.Stream(dev)
    with torch.cuda.stream(side):
        for a in (a1, a2):
            h = torch.empty_strided((batch, n, n), (n * n, 1, n), pin_memory=True)
            t = torch.empty(batch, n, pin_memory=True)
            fastqr.geqrf_host(a, out=(h, t), workspace=ws, device=dev, synchronize=False)
            outs.append((h, t))
    side.synchronize()
    for a, (h, t) in zip((a1, a2), outs):
        hd, td = device_result(a, dev)
        assert torch.equal(h, hd) and torch.equal(t, td)


def test_host_matches_oracle_small(dev):
    a = inputs.generate_input(12, 48, 0, 9, device="cpu")
    h, t = fastqr.geqrf_host(a, device=dev)
    h64, t64 = oracle.geqrf_f64(a.numpy())
    ok, msg = checker.check_columns(h.numpy(), t.numpy(), h64, t64, 1e-3)
    assert ok, msg


def test_host_replayed_call_sees_new_data(dev):
    """Repeated calls with the same buffers replay one captured graph: each
    call must read the host input as it is at that call (bitwise equal to the
    device entry on that data), with page-locked and with pageable buffers
    (which do not capture and are enqueued directly)."""
    batch, n = 24, 256
    for pinned in (True, False):
        a = torch.empty(batch, n, n)
        h = torch.empty_strided((batch, n, n), (n * n, 1, n))
        t = torch.empty(batch, n)
        if pinned:
            a, h, t = a.pin_memory(), h.pin_memory(), t.pin_memory()
        ws = torch.empty(fastqr.host_workspace_bytes(batch, n), dtype=torch.uint8, device=dev)
        for seed in (1, 2, 3):
            a.copy_(inputs.generate_input(batch, n, 1, seed, device="cpu"))
            fastqr.geqrf_host(a, out=(h, t), workspace=ws, device=dev)
            hd, td = device_result(a, dev)
            assert torch.equal(h, hd) and torch.equal(t, td), (pinned, seed)
            fastqr.host_check_status(ws, batch, n)  # raises if a bounded wait gave up


def test_host_large_chunks_planned_for_the_batch(dev):
    """10 x 4096^2: n >= 3584 and the call's trailing tiles fill two CTAs per
    SM, so the one-matrix chunks are planned for the whole batch (unsplit
    rank-64 tiles), as the device entry plans its parts.  The in-block steps
    size their clusters by each launch's own batch (one matrix per chunk here,
    two or three per part there), so the two entries agree to rounding, within
    the per-column 1e-3 that the parity tests allow against float64."""
    n, batch = 4096, 10
    a = torch.randn(batch, n, n, generator=torch.Generator().manual_seed(11)).pin_memory()
    h, t = fastqr.geqrf_host(a, device=dev)
    hd, td = device_result(a, dev)
    col = (h - hd).abs().amax(dim=1) / hd.abs().amax(dim=1).clamp_min(1e-30)  # per column of H
    assert col.max().item() <= 1e-3
    assert ((t - td).abs() <= 1e-3 * td.abs() + 1e-6).all()
