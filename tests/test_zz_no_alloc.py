"""fqr_geqrf_f32_noalloc, the entry point for callers that cannot allocate
device memory (for example a host that owns the whole device pool, or a
language binding with no clean way to create a scratch buffer per call).

It must give the same factorisation as fqr_geqrf_f32 -- within the per-column
tolerance the parity tests use -- on two calls in a row (the static scratch
keeps the previous call's contents), and reject batches its fixed scratch
cannot hold.  Collected last on purpose; it does not depend on other tests.
"""
import ctypes

import pytest
import torch

import fastqr
from fastqr import inputs

from gpu_gates import column_errors

pytestmark = pytest.mark.gpu
COL_TOL = 1e-3
FQR_ENOALLOC_LIMIT = 7
MAX_BATCH = 1024


def _noalloc(lib, a, h, t):
    batch, n, _ = a.shape
    bs, rs, cs = a.stride()
    stream = torch.cuda.current_stream(a.device).cuda_stream
    return lib.fqr_geqrf_f32_noalloc(a.data_ptr(), batch, n, bs, rs, cs, h.data_ptr(),
                                     t.data_ptr(), stream)


# (2, 2048) runs the rank-64 plan, whose 64 x 64 S blocks set the scratch size
@pytest.mark.parametrize("batch,n", [(64, 32), (16, 256), (5, 100), (3, 512), (2, 1100), (2, 2048)])
def test_noalloc_matches_the_allocating_entry_point(batch, n):
    assert torch.cuda.is_available()
    dev = torch.device("cuda:0")
    lib = fastqr.load()
    for call in range(2):
        a = inputs.generate_input(batch, n, 1, 900 + 10 * n + call, device=dev)
        h_ref, t_ref = fastqr.geqrf(a)
        h, t = fastqr.empty_outputs(batch, n, dev)
        rc = _noalloc(lib, a, h, t)
        assert rc == 0, fastqr.FastQRError(rc)
        stream = torch.cuda.current_stream(dev).cuda_stream
        assert lib.fqr_noalloc_check_status(stream) == 0
        torch.cuda.synchronize()
        he, te = column_errors(h, t, h_ref, t_ref)
        assert float(he.max()) <= COL_TOL and float(te.max()) <= COL_TOL, (call, float(he.max()))


def test_noalloc_rejects_batches_beyond_its_scratch():
    dev = torch.device("cuda:0")
    lib = fastqr.load()
    n = 100
    a = torch.zeros(MAX_BATCH + 1, n, n, device=dev)
    h, t = fastqr.empty_outputs(MAX_BATCH + 1, n, dev)
    assert _noalloc(lib, a, h, t) == FQR_ENOALLOC_LIMIT
    # the largest accepted batch at n > 64
    a = inputs.generate_input(MAX_BATCH, n, 1, 77, device=dev)
    h, t = fastqr.empty_outputs(MAX_BATCH, n, dev)
    assert _noalloc(lib, a, h, t) == 0
    h_ref, t_ref = fastqr.geqrf(a)
    torch.cuda.synchronize()
    he, te = column_errors(h, t, h_ref, t_ref)
    assert float(he.max()) <= COL_TOL and float(te.max()) <= COL_TOL
    # the small path needs no scratch and has no such limit
    a32 = inputs.generate_input(MAX_BATCH + 1, 32, 0, 5, device=dev)
    h32, t32 = fastqr.empty_outputs(MAX_BATCH + 1, 32, dev)
    assert _noalloc(lib, a32, h32, t32) == 0
    h_ref, t_ref = fastqr.geqrf(a32)
    torch.cuda.synchronize()
    he, te = column_errors(h32, t32, h_ref, t_ref)
    assert float(he.max()) <= COL_TOL and float(te.max()) <= COL_TOL
