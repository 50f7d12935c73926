"""The one-file submission (fastqr.stage) run the way the reference's
evaluator runs a submission (official/eval.py:125-132): a spawned worker
imports ``custom_kernel`` from the file, calls it on a clone of a generated
input and the result goes through the official checker's gates
(official/reference.py:182-244, restated in oracle/checker.py).  Inputs come
from the reference generator's restatement (fastqr.inputs, bit-exact) with
this suite's own seeds, covering the upstream shapes (32, 176, 352, 512,
1024) and conditioning profiles.  The worker uses the in-tree library
($FASTQR_LIB) so the test does not wait for nvcc; test_submission.py builds
the library from the file's own sources."""
import multiprocessing as mp
import os
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

CASES = [
    {"batch": 20, "n": 32, "cond": 1, "seed": 911},
    {"batch": 40, "n": 176, "cond": 1, "seed": 912},
    {"batch": 24, "n": 352, "cond": 1, "seed": 913},
    {"batch": 8, "n": 512, "cond": 2, "seed": 914},
    {"batch": 8, "n": 512, "cond": 0, "seed": 915, "case": "rankdef"},
    {"batch": 4, "n": 512, "cond": 2, "seed": 916, "case": "mixed"},
    {"batch": 2, "n": 1024, "cond": 0, "seed": 917, "case": "nearrank"},
]


def _run_case(path, spec):
    import importlib.util

    import torch

    from fastqr import inputs
    from oracle import checker

    s = importlib.util.spec_from_file_location("submission", path)
    sub = importlib.util.module_from_spec(s)
    s.loader.exec_module(sub)
    data = inputs.generate_input(spec["batch"], spec["n"], spec["cond"], spec["seed"],
                                 case=spec.get("case", "dense"), device="cuda")
    torch.cuda.synchronize()
    h, tau = sub.custom_kernel(data.clone())
    torch.cuda.synchronize()
    n = spec["n"]
    layout = h.shape == data.shape and h.stride() == (n * n, 1, n) and tau.shape == (spec["batch"], n)
    rep = checker.check_qr(data.cpu().numpy(), h.cpu().numpy(), tau.cpu().numpy())
    return bool(layout), bool(rep.ok), rep.message


def test_submission_file_passes_the_official_gates(tmp_path):
    from fastqr import stage
    from fastqr._lib import LIB_PATH

    path = str(stage.stage(tmp_path / "submission.py"))
    os.environ["FASTQR_LIB"] = str(LIB_PATH)
    try:
        ctx = mp.get_context("spawn")
        with ctx.Pool(1) as pool:
            for spec in CASES:
                layout, ok, msg = pool.apply(_run_case, (path, spec))
                assert layout, spec
                assert ok, (spec, msg)
    finally:
        os.environ.pop("FASTQR_LIB", None)
