"""Test configuration.

Markers: ``gpu`` tests need a CUDA device (a B200 on the GPU box); everything
else runs on CPU.  The ``fastqr`` package lives in ``fast-qr_b200/`` and the
CPU oracle in ``oracle/``; both are put on sys.path here.
"""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "fast-qr_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


@pytest.fixture(scope="session")
def golden():
    import json

    import numpy as np

    data = np.load(ROOT / "tests" / "golden" / "golden.npz")
    meta = json.loads((ROOT / "tests" / "golden" / "golden.json").read_text())
    return data, meta
