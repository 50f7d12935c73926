"""bench.py's launch and work model against the library (CPU only: no
kernel runs).  The per-class launch counts feed the roofline's per-launch
figures and the bench line's gpu_launches claim, so they must match what
fqr_launch_count reports for the same plan."""
import argparse
import importlib.util
from pathlib import Path

import pytest

import fastqr

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("n", [96, 256, 512, 600, 1024, 2048, 2100, 4096])
def test_stage_launches_match_the_library(bench, n):
    # one matrix: a single part, so every launch of the plan runs once
    counts = bench.stage_launches(n)
    total = counts["copy_in"] + counts["panel"] + counts["inblock"] + counts["trailing"] + counts["mid"]
    assert (counts["mid"] == 1) == fastqr.plan(1, n).startswith("mid")
    assert total == fastqr.launch_count(1, n), (n, counts)
    assert ("rank 64" in fastqr.plan(1, n)) == (counts["inblock"] > 0)


def test_trailing_flops_count_each_update_once(bench):
    # rank-32 plan: sum over panels of 4 m b nc + b^2 nc, b = 32
    n = 256
    want = sum(4.0 * (n - k) * 32 * (n - k - 32) + 32 * 32 * (n - k - 32) for k in range(0, n - 32, 32))
    assert bench.trailing_flops(n) == want
    # rank-64 plan: the same count with b = 64 per block
    n = 2048
    want = sum(4.0 * (n - k) * 64 * (n - k - 64) + 64 * 64 * (n - k - 64) for k in range(0, n - 64, 64))
    assert bench.trailing_flops(n) == want


def test_strong_scaling_config_block(bench):
    weak = bench._config_block(argparse.Namespace(config="C5", strong=False), 8)
    strong = bench._config_block(argparse.Namespace(config="C5", strong=True), 8)
    assert (weak["batch_per_gpu"], weak["global_batch"]) == (16, 128)
    assert (strong["batch_per_gpu"], strong["global_batch"]) == (2, 16)


@pytest.mark.parametrize("m,n", [(512, 384), (2304, 2080), (8192, 2048)])
def test_rect_stage_launches_follow_the_plan(bench, m, n):
    # tall blocks take rank-64 blocks only for n >= 2048 with m <= 4096
    counts = bench.stage_launches(n, m)
    assert (counts["inblock"] > 0) == (n >= 2048 and m <= 4096)
    blocks, rest = bench.plan_blocks(n, m)
    assert 64 * blocks + rest == n
