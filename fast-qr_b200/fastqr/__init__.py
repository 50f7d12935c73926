"""fastqr: batched square Householder QR (geqrf) on B200 (sm_100a).

Drop-in for the reference's ``custom_kernel(data) -> (H, tau)`` and for
``torch.geqrf`` on CUDA float32 batches of square matrices.  The compute runs
in hand-written CUDA kernels behind the C ABI of ``libfastqr.so``
(include/fastqr.h); this package is the thin host side.
"""
from .api import (check_status, custom_kernel, empty_outputs, geqrf, geqrf_host, geqrf_profile,
                  host_check_status, host_workspace_bytes, householder_product, launch_count, orgqr_workspace_bytes,
                  ormqr, plan, workspace_bytes)
from ._lib import FastQRError, LIB_PATH, load

__all__ = ["check_status", "custom_kernel", "geqrf", "geqrf_host", "geqrf_profile", "empty_outputs",
           "host_check_status", "host_workspace_bytes", "householder_product", "ormqr",
           "orgqr_workspace_bytes", "workspace_bytes", "plan", "launch_count",
           "FastQRError", "LIB_PATH", "load"]
__version__ = "0.1.0"
