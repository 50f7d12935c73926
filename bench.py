"""Benchmark: batched square QR (geqrf) throughput on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C2] [--impl fastqr|reference]

One step = one batched geqrf over the configuration's batch (per GPU), inputs
resident in HBM, L2 flushed (256 MiB write) before every step.  The headline
configuration is C2 (256 x 256^2, graded columns): BASELINE.json's configs[1].
Multi-GPU (torchrun, one process per GPU): strong scaling by default -- the
configuration's own batch is split into contiguous shards, north_star's
partition (C5 on 8 GPUs: 2 matrices per GPU); no collective on the data path;
time = max over ranks.  The line also carries the weak-scaling number (every
rank a full configuration batch); ``--weak`` makes that the value.
At N = 1 the line carries ``per_config`` (all five configurations measured in
the same run) and ``gpu_baseline`` (torch.geqrf on CUDA, same inputs).

Prints ONE JSON line on rank 0.  ``--impl reference`` times the reference's
own CPU implementation of the path -- torch.geqrf on the host (its
``ref_kernel``, official/reference.py:125-127, and baseline submission,
submissions/baseline_geqrf.py:5-6) -- on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT), str(ROOT / "fast-qr_b200")]

import torch  # noqa: E402

from fastqr import inputs  # noqa: E402
from fastqr.shard import all_ranks_ok, dist_env, max_over_ranks, rank_inputs  # noqa: E402

HBM_FALLBACK_GBS = 6650.0
BF16_FALLBACK_TFLOPS = 1590.0
L2_FLUSH_BYTES = 256 << 20
DEFAULT_STEPS = {"C1": 400, "C2": 200, "C3": 20, "C4": 10, "C5": 3}


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured (MEASURED_PEAKS.json)"}
    return {"hbm_gbs": HBM_FALLBACK_GBS, "bf16_tflops": BF16_FALLBACK_TFLOPS,
            "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def flops_per_matrix(n: int) -> float:
    return 4.0 * n ** 3 / 3.0


def bytes_per_matrix(n: int) -> float:
    return 4.0 * (2 * n * n + n)


def panel_bytes(n: int, b: int = 32) -> float:
    """Algorithmic HBM bytes of all panel launches of one matrix: per panel k
    the (n-k) x b column block is read and written back, and b tau values and
    the b x b S block are written."""
    return sum(8.0 * b * (n - k) + 4.0 * b + 4.0 * b * b for k in range(0, n, b))


def plan_blocks(n: int, m: int | None = None) -> tuple:
    """(rank-64 blocks, columns left for rank-32 steps) of the library's static
    plan for m x n (m = n by default): rank-64 blocks for n >= 2048 with
    m <= 4096 and m % 4 == 0."""
    m = n if m is None else m
    outer = n >= 2048 and m <= 4096 and m % 4 == 0
    blocks = n // 64 if outer else 0
    return blocks, n - 64 * blocks


def trailing_flops(n: int) -> float:
    """Algorithmic flops of all trailing updates of one matrix: per update at
    column k with b reflectors, 4 (n-k) b (n-k-b) + b^2 (n-k-b); b = 64 for
    the rank-64 blocks, 32 for the rank-32 steps."""
    blocks, _ = plan_blocks(n)
    steps = [(64 * i, 64) for i in range(blocks)] + [(k, 32) for k in range(64 * blocks, n, 32)]
    tot = 0.0
    for k, b in steps:
        m, nc = n - k, n - k - b
        if nc > 0:
            tot += 4.0 * m * b * nc + b * b * nc
    return tot


def inblock_bytes(n: int) -> float:
    """Algorithmic HBM bytes of the in-block steps of one matrix: per rank-64
    block at k the update reads V1 and C2 ((n-k) x 32 each) and writes C2; the
    Gram step (all but a last block with no columns right of it) reads V1 and
    V2 below row k+32."""
    blocks, rest = plan_blocks(n)
    tot = 0.0
    for i in range(blocks):
        m = n - 64 * i
        tot += 12.0 * 32 * m
        if rest > 0 or i + 1 < blocks:
            tot += 8.0 * 32 * (m - 32)
    return tot


def mid_plan(n: int, m: int | None = None) -> bool:
    """The library's one-launch mid-size kernel is not in its static plan (it
    runs only under fqr_debug_plan(1)); every square size takes the warp
    kernel (n <= 64) or the blocked path."""
    return False


def stage_launches(n: int, m: int | None = None) -> dict:
    """Launches per kernel class of one factorisation (one stream)."""
    if mid_plan(n, m):
        return {"small": 0, "copy_in": 0, "panel": 0, "inblock": 0, "trailing": 0, "mid": 1}
    blocks, rest = plan_blocks(n, m)
    rp = -(-rest // 32)
    full = blocks if rest > 0 else max(blocks - 1, 0)
    return {"small": 1, "copy_in": 1, "panel": 2 * blocks + rp, "inblock": blocks + full,
            "trailing": full + max(rp - 1, 0), "mid": 0}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.idx)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out = ""

    def summary(self) -> dict:
        rows = []
        for line in (self.out or "").strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                rows.append((float(f[1]), float(f[2]), float(f[3]), f[4], f[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        maxmhz = max(r[1] for r in rows)
        loaded = [r for r in rows if r[2] > 200.0] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in loaded for i, v in enumerate(r[4]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": maxmhz,
                "reasons": reasons, "samples": len(rows)}


def cpu_reference(cfg_name: str, seed: int, budget_s: float, reps_min: int = 3) -> dict:
    """torch.geqrf on the host cores over a bounded sample of the workload."""
    cfg = inputs.CONFIGS[cfg_name]
    n, batch = cfg["n"], cfg["batch"]
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    # sample size: the whole batch when it is cheap, else fewer matrices
    probe = inputs.baseline_input(cfg_name, seed=seed, device="cpu", batch=1)
    t0 = time.perf_counter()
    torch.geqrf(probe)
    one = max(time.perf_counter() - t0, 1e-6)
    sample = int(max(1, min(batch, (budget_s / reps_min) / one)))
    a = inputs.baseline_input(cfg_name, seed=seed, device="cpu", batch=sample)
    torch.geqrf(a)  # warm-up
    times = []
    start = time.perf_counter()
    while len(times) < reps_min or (time.perf_counter() - start) < budget_s * 0.5:
        t0 = time.perf_counter()
        torch.geqrf(a)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - start > budget_s:
            break
    per = statistics.median(times)
    return {"value": sample / per, "unit": "matrices/s", "cores": threads, "kind": "reference",
            "sample": f"torch.geqrf (host LAPACK) on {sample} of the {batch} {n}x{n} matrices, "
                      f"median of {len(times)} reps",
            "tflops": sample * flops_per_matrix(n) / per / 1e12,
            "cpu_model": _cpu_model()}


def _cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(args) -> int:
    """The reference arm: torch.geqrf on the host cores (rank 0 only).  Each
    step factors a bounded sample of the configuration's batch, sized so the
    whole W + K run stays within a few minutes."""
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    cfg = inputs.CONFIGS[args.config]
    n, batch = cfg["n"], cfg["batch"]
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    probe = inputs.baseline_input(args.config, seed=args.seed, device="cpu", batch=1)
    torch.geqrf(probe)
    t0 = time.perf_counter()
    torch.geqrf(probe)
    one = max(time.perf_counter() - t0, 1e-6)
    per_step_budget = min(2.0, 150.0 / (args.warmup + args.steps))
    sample = int(max(1, min(batch, per_step_budget / one)))
    a = inputs.baseline_input(args.config, seed=args.seed, device="cpu", batch=sample)
    for _ in range(args.warmup):
        torch.geqrf(a)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        torch.geqrf(a)
        times.append(time.perf_counter() - t0)
    value = sample * len(times) / sum(times)
    desc = (f"torch.geqrf (host LAPACK, {threads} threads) on {sample} of the {batch} "
            f"{n}x{n} matrices per step")
    line = {
        "impl": "reference", "metric": f"matrices/s ({args.config} geqrf)", "value": value,
        "unit": "matrices/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * batch / value, "higher_is_better": True,
        "scaling": "strong" if args.strong else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": _config_block(args, world),
        "tflops": value * flops_per_matrix(n) / 1e12,
        "cpu_baseline": {"value": value, "unit": "matrices/s", "cores": threads,
                         "kind": "reference", "sample": desc},
        "e2e": {"value": value, "unit": "matrices/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "cpu_model": _cpu_model(),
    }
    print(json.dumps(line), flush=True)
    return 0


def _config_block(args, world) -> dict:
    cfg = inputs.CONFIGS[args.config]
    strong = getattr(args, "strong", False)
    per = -(-cfg["batch"] // world) if strong else cfg["batch"]
    return {"workload": f"{args.config}: {cfg['desc']}", "batch_per_gpu": per, "n": cfg["n"],
            "global_batch": cfg["batch"] if strong else cfg["batch"] * world,
            "l2": "flushed before every step (256 MiB write)",
            "parallelism": f"batch-sharded x{world}, no collective"}


PER_CONFIG_STEPS = {"C1": 100, "C2": 50, "C3": 10, "C4": 10, "C5": 3}


def timed_steps(step, steps, flush, stream) -> float:
    """Mean device milliseconds of `steps` calls of step() on `stream`, the L2
    flushed (a 256 MiB write, outside the events) before each."""
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        flush.fill_(float(i))
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    torch.cuda.synchronize()
    return sum(s_.elapsed_time(e_) for s_, e_ in zip(starts, ends)) / steps


def torch_cuda_geqrf(a, flush, stream, budget_s: float = 20.0) -> dict:
    """The GPU comparator: torch.geqrf on the same resident inputs on the GPU
    (cuSOLVER / MAGMA through the torch build), timed like fastqr (device
    events, L2 flushed).  A bounded sub-batch when the whole batch would take
    long; the value is matrices/s of that sample."""
    batch = a.shape[0]
    torch.geqrf(a[:1])
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    torch.geqrf(a[:1])
    torch.cuda.synchronize()
    one = max(time.perf_counter() - t0, 1e-6)
    sample = int(max(1, min(batch, (budget_s / 4.0) / one)))
    x = a[:sample]
    torch.geqrf(x)
    ms = timed_steps(lambda: torch.geqrf(x), 3, flush, stream)
    return {"value": sample / (ms / 1e3), "unit": "matrices/s", "impl": "torch.geqrf (CUDA)",
            "ms_per_call": ms, "sample": f"{sample} of the {batch} matrices per call, mean of 3 calls"}


def per_config_block(args, dev, flush, stream) -> dict:
    """Every BASELINE configuration (C1..C5) measured in this run: device ms
    per step (L2 flushed), matrices/s, TFLOP/s at 4n^3/3 flops per matrix,
    the dominant kernel's roofline fraction, the QR gates on a few matrices,
    and the torch.geqrf-on-CUDA comparator on the same inputs."""
    import fastqr
    from gpu_gates import gates

    out = {}
    for name in ("C1", "C2", "C3", "C4", "C5"):
        cfg = inputs.CONFIGS[name]
        n, batch = cfg["n"], cfg["batch"]
        a = inputs.baseline_input(name, args.seed, dev)
        h, tau = fastqr.empty_outputs(batch, n, dev)
        ws = torch.empty(max(1, fastqr.workspace_bytes(batch, n)), dtype=torch.uint8, device=dev)

        def step():
            fastqr.geqrf(a, out=(h, tau), workspace=ws)

        for _ in range(3):
            step()
        steps = PER_CONFIG_STEPS[name]
        ms = timed_steps(step, steps, flush, stream)
        chk = 2 if n >= 4096 else 4
        g = gates(a[:chk], h[:chk], tau[:chk], chunk=chk)
        roof = kernel_roofline(name, a, h, tau, ws, flush, min(steps, 3), dev)
        mps = batch / (ms / 1e3)
        row = {"n": n, "batch": batch, "steps": steps, "ms_per_step": ms, "matrices_per_s": mps,
               "tflops": mps * flops_per_matrix(n) / 1e12, "hbm_gbs_alg": mps * bytes_per_matrix(n) / 1e9,
               "dominant_kernel": roof["kernel"], "roofline_bound": roof["bound"],
               "roofline_achieved": roof["achieved"], "roofline_unit": roof["unit"], "roofline_frac": roof["frac"],
               "gpu_launches_per_step": fastqr.launch_count(batch, n), "verified": bool(g["ok"])}
        if not args.no_gpu_baseline:
            ref = torch_cuda_geqrf(a, flush, stream)
            row["gpu_baseline"] = ref
            row["vs_gpu_baseline"] = mps / ref["value"]
        out[name] = row
        del a, h, tau, ws
        torch.cuda.empty_cache()
    return out


def run_fastqr(args) -> int:
    import torch.distributed as dist

    import fastqr

    rank, world, local = dist_env()
    if world > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)
    cfg = inputs.CONFIGS[args.config]
    n = cfg["n"]
    steps = args.steps

    # strong scaling (default): the configuration's batch split into
    # contiguous shards, north_star's partition (C5 on 8 GPUs: 2 matrices per
    # GPU); weak (--weak): every rank a full configuration batch
    a, first = rank_inputs(args.config, args.seed, world, rank, dev, weak=not args.strong)
    batch = a.shape[0]
    if batch < 1:
        raise SystemExit(f"--strong: {args.config}'s batch of {cfg['batch']} leaves rank {rank} no matrix")
    global_batch = cfg["batch"] if args.strong else world * batch
    h, tau = fastqr.empty_outputs(batch, n, dev)
    ws = torch.empty(max(1, fastqr.workspace_bytes(batch, n)), dtype=torch.uint8, device=dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        fastqr.geqrf(a, out=(h, tau), workspace=ws)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)

    # correctness of this rank's output (untimed)
    sys.path.insert(0, str(ROOT / "tests"))
    from gpu_gates import gates
    chk = min(batch, 16)
    g = gates(a[:chk], h[:chk], tau[:chk], chunk=chk)
    ok = all_ranks_ok(bool(g["ok"]), dev)

    # timed region: K steps, L2 flush before each (outside the events)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(dev.index) as clk:
        for i in range(steps):
            flush.fill_(float(i))
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    total_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    total_ms = max_over_ranks(total_ms, dev)
    ms = total_ms / steps
    value = global_batch / (ms / 1e3)

    # the other scaling mode beside it (N > 1): every rank a full batch when
    # the line is strong, the configuration's batch split when it is weak
    other = None
    if world > 1:
        a2, _ = rank_inputs(args.config, args.seed, world, rank, dev, weak=args.strong)
        b2 = a2.shape[0]
        h2, t2 = fastqr.empty_outputs(b2, n, dev)
        ws2 = torch.empty(max(1, fastqr.workspace_bytes(b2, n)), dtype=torch.uint8, device=dev)

        def step2():
            fastqr.geqrf(a2, out=(h2, t2), workspace=ws2)

        for _ in range(args.warmup):
            step2()
        dist.barrier()
        torch.cuda.synchronize(dev)
        ms2 = max_over_ranks(timed_steps(step2, steps, flush, stream), dev)
        gb2 = world * b2 if args.strong else cfg["batch"]
        other = {"scaling": "weak" if args.strong else "strong", "value": gb2 / (ms2 / 1e3),
                 "ms_per_step": ms2, "global_batch": gb2, "batch_per_gpu": b2}
        del a2, h2, t2, ws2

    # per-kernel times for the roofline: same steps again, kernels timed alone
    roof = kernel_roofline(args.config, a, h, tau, ws, flush, steps, dev)

    # end to end through the public API with host buffers
    e2e = end_to_end(a, n, batch, dev, max(3, min(steps, 50)))
    e2e_value = max_over_ranks(e2e["ms"], dev)
    e2e_mps = global_batch / (e2e_value / 1e3)

    # the GPU comparator on the same inputs, and every configuration (N = 1)
    gpu_ref = None
    per_cfg = None
    per_clk = None
    if world == 1:
        if not args.no_gpu_baseline:
            gpu_ref = torch_cuda_geqrf(a, flush, stream)
        if not args.no_per_config:
            with ClockSampler(dev.index) as pclk:
                per_cfg = per_config_block(args, dev, flush, stream)
            per_clk = pclk.summary()

    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu:
        budget = {"C1": 10.0, "C2": 10.0, "C3": 20.0, "C4": 20.0, "C5": 30.0}[args.config]
        r = cpu_reference(args.config, args.seed, budget)
        cpu = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")}
        cpu["cpu_model"] = r["cpu_model"]

    if rank == 0:
        line = {
            "metric": f"matrices/s ({args.config} geqrf)", "value": value, "unit": "matrices/s",
            "n_gpus": world, "steps": steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong" if args.strong else "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded, the reference generator's distributions)",
            "config": _config_block(args, world),
            "tflops": value * flops_per_matrix(n) / 1e12,
            "hbm_gbs_alg": value * bytes_per_matrix(n) / 1e9,
            "verified": bool(ok),
            "gate": {k: g[k] for k in ("factor_scaled", "orth_scaled", "recon_rel_f", "orth_rel_f")},
            "roofline": roof,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_mps, "unit": "matrices/s", "h2d_bytes_per_step": e2e["h2d"],
                    "d2h_bytes_per_step": e2e["d2h"]},
            "gpu_launches": steps * fastqr.launch_count(batch, n),
            "plan": fastqr.plan(batch, n),
            "clocks": clk.summary(),
        }
        if other is not None:
            line["other_scaling"] = other
        if gpu_ref is not None:
            line["gpu_baseline"] = gpu_ref
            line["vs_gpu_baseline"] = value / gpu_ref["value"]
        if per_cfg is not None:
            line["per_config"] = per_cfg
            line["per_config_clocks"] = per_clk
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def kernel_roofline(cfg_name, a, h, tau, ws, flush, steps, dev) -> dict:
    """Dominant-kernel roofline from per-kernel CUDA events.

    The same K steps are run again through ``fqr_geqrf_f32_profile``, which
    records an event pair on the launch stream around every kernel; the
    kernel class with the largest summed time is the dominant one and its
    algorithmic work per step over its time per step is ``achieved``.
    """
    import fastqr

    n = a.shape[-1]
    batch = a.shape[0]
    pk = peaks()
    tot = {}
    for i in range(steps):
        flush.fill_(float(i))
        st = fastqr.geqrf_profile(a, (h, tau), ws)
        for kname, v in st.items():
            tot[kname] = tot.get(kname, 0.0) + v
    per_step_ms = {kname: v / steps for kname, v in tot.items()}
    dom = max(per_step_ms, key=per_step_ms.get)
    t = per_step_ms[dom] / 1e3
    traffic = _traffic_from_profiles(cfg_name, dom)
    share = {kname: round(v / max(sum(per_step_ms.values()), 1e-12), 4) for kname, v in per_step_ms.items()}
    # launches of the dominant kernel class per profiled step (one stream)
    per_step = stage_launches(n)[dom]
    base = {"kernel": dom, "stage_ms_per_step": per_step_ms, "stage_share": share,
            "traffic": traffic, "launches_per_step": per_step, "peak_source": pk["source"]}
    if dom in ("small", "copy_in", "panel", "inblock", "mid"):
        # the panel does O(m b^2) flops on O(m b) data: it is framed by HBM
        # bytes, and its limiter is the column-by-column dependency chain.
        # The one-launch mid-size kernel does the whole factorisation: read A,
        # write H and tau (n / 6 flop per byte, below the tensor pipe's ridge,
        # so HBM is its roof)
        alg = batch * {"small": bytes_per_matrix(n), "copy_in": 8.0 * n * n,
                       "panel": panel_bytes(n), "inblock": inblock_bytes(n),
                       "mid": bytes_per_matrix(n)}[dom]
        ach = alg / t / 1e9
        base.update({"bound": "hbm", "achieved": ach, "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": ach / pk["hbm_gbs"], "alg_bytes_per_step": alg,
                     "alg_bytes_per_launch": alg / per_step})
        return base
    tf32 = pk["bf16_tflops"] / 2.0
    alg = batch * trailing_flops(n)
    ach = alg / t / 1e12
    base.update({"bound": "tensor", "achieved": ach, "peak": tf32, "unit": "TFLOP/s",
                 "frac": ach / tf32, "alg_flops_per_step": alg, "alg_flops_per_launch": alg / per_step,
                 "peak_source": pk["source"] + "; TF32 dense peak taken as measured bf16 / 2"})
    return base


def _traffic_from_profiles(cfg_name, kernel):
    """DRAM bytes per launch of `kernel` from the committed ncu summary
    profiles/traffic_<config>_<kernel>.txt (None when there is none)."""
    p = ROOT / "profiles" / f"traffic_{cfg_name}_{kernel}.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("dram_bytes_per_launch"):
            return float(line.split()[1])
    return None


def end_to_end(a, n, batch, dev, steps) -> dict:
    """The host-buffer entry point of the public API (fastqr.geqrf_host ->
    fqr_geqrf_f32_host) on page-locked host buffers: every step uploads A,
    factors it and downloads H and tau (chunked, the copies overlapping the
    kernels), all inside the events."""
    import fastqr

    stream = torch.cuda.current_stream(dev)
    a_host = a.cpu().pin_memory()
    h_host = torch.empty_strided((batch, n, n), (n * n, 1, n), dtype=torch.float32, pin_memory=True)
    t_host = torch.empty((batch, n), dtype=torch.float32, pin_memory=True)
    ws = torch.empty(max(fastqr.host_workspace_bytes(batch, n), 1), dtype=torch.uint8, device=dev)

    def one():
        fastqr.geqrf_host(a_host, out=(h_host, t_host), workspace=ws, device=dev, synchronize=False)

    for _ in range(2):
        one()
    torch.cuda.synchronize(dev)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for _ in range(steps):
        one()
    e.record(stream)
    torch.cuda.synchronize(dev)
    ms = s.elapsed_time(e) / steps
    return {"ms": ms, "h2d": batch * n * n * 4, "d2h": batch * (n * n + n) * 4}


def run_apply_op(args) -> int:
    """--op orgqr | ormqr: Q formation (householder_product) or Q^T C (ormqr,
    C = A, i.e. the n x n input batch) from factors made by fastqr.geqrf
    outside the timed region; one process, N=1 only."""
    import fastqr

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = inputs.CONFIGS[args.config]
    n, batch = cfg["n"], cfg["batch"]
    steps = args.steps
    a = inputs.baseline_input(args.config, args.seed, dev)
    h, tau = fastqr.geqrf(a)
    ws = torch.empty(max(1, fastqr.orgqr_workspace_bytes(batch, n)), dtype=torch.uint8, device=dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    # outputs allocated once: Q, or the column-major copy of A that ormqr
    # overwrites with Q^T A (the copy is part of the op)
    res = torch.empty_strided((batch, n, n), (n * n, 1, n), device=dev, dtype=torch.float32)

    def step():
        if args.op == "orgqr":
            return fastqr.householder_product(h, tau, out=res, workspace=ws)
        return fastqr.ormqr(h, tau, a, transpose=True, out=res, workspace=ws)

    for _ in range(args.warmup):
        out = step()
    torch.cuda.synchronize(dev)
    # correctness (untimed): Q orthogonal and Q R = A, or Q^T A = R
    chk = min(batch, 8)
    r = torch.triu(h[:chk])
    if args.op == "orgqr":
        q = out[:chk]
        eye = torch.eye(n, device=dev)
        e1 = float((torch.linalg.matrix_norm(q.transpose(1, 2) @ q - eye) / n ** 0.5).max())
        e2 = float((torch.linalg.matrix_norm(a[:chk] - q @ r) / torch.linalg.matrix_norm(a[:chk])).max())
        gate = {"orth_rel_f": e1, "recon_rel_f": e2}
        ok = e1 <= 1e-4 and e2 <= 1e-4
    else:
        e1 = float((torch.linalg.matrix_norm(out[:chk] - r) / torch.linalg.matrix_norm(r)).max())
        gate = {"qta_minus_r_rel_f": e1}
        ok = e1 <= 1e-4
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    stream = torch.cuda.current_stream(dev)
    torch.cuda.synchronize(dev)
    with ClockSampler(0) as clk:
        for i in range(steps):
            flush.fill_(float(i))
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        torch.cuda.synchronize(dev)
    clocks = clk.summary()
    ms = sum(s_.elapsed_time(e_) for s_, e_ in zip(starts, ends)) / steps
    mps = batch / (ms / 1e3)
    # Householder application: 4n^3/3 flops per matrix for either op on square C
    alg = batch * flops_per_matrix(n)
    pk = peaks()
    tf32 = pk["bf16_tflops"] / 2.0
    ach = alg / (ms / 1e3) / 1e12
    cpu = None
    if not args.no_cpu:
        threads = os.cpu_count() or 1
        torch.set_num_threads(threads)
        hc, tc = h[:min(batch, 32)].cpu(), tau[:min(batch, 32)].cpu()
        ac = a[:hc.shape[0]].cpu()
        fn = (lambda: torch.linalg.householder_product(hc, tc)) if args.op == "orgqr" else \
             (lambda: torch.ormqr(hc, tc, ac, left=True, transpose=True))
        fn()
        times = []
        t_start = time.perf_counter()
        while len(times) < 3 or time.perf_counter() - t_start < 5.0:
            t0 = time.perf_counter()
            fn()
            times.append(time.perf_counter() - t0)
            if time.perf_counter() - t_start > 20.0:
                break
        per = statistics.median(times)
        name = "torch.linalg.householder_product" if args.op == "orgqr" else "torch.ormqr"
        cpu = {"value": hc.shape[0] / per, "unit": "matrices/s", "cores": threads, "kind": "reference",
               "sample": f"{name} (host LAPACK) on {hc.shape[0]} of the {batch} {n}x{n} factorisations, "
                         f"median of {len(times)} reps"}
    launches = 1 + (2 + (n + 31) // 32 if fastqr.orgqr_workspace_bytes(batch, n) else 1)
    line = {
        "metric": f"matrices/s ({args.config} {args.op})", "value": mps, "unit": "matrices/s", "n_gpus": 1,
        "steps": steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded, the reference generator's distributions); factors from fastqr.geqrf",
        "config": {"workload": f"{args.config}: {cfg['desc']}", "op": args.op, "n": n, "batch_per_gpu": batch,
                   "l2": f"flushed before every step ({L2_FLUSH_BYTES >> 20} MiB write)"},
        "verified": ok, "gate": gate,
        "roofline": {"kernel": "apply (whole op)", "bound": "tensor", "achieved": ach, "peak": tf32,
                     "unit": "TFLOP/s", "frac": ach / tf32, "traffic": None,
                     "peak_source": pk["source"] + "; TF32 dense peak taken as measured bf16 / 2"},
        "cpu_baseline": cpu, "e2e": None, "gpu_launches": steps * launches, "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    return 0 if ok else 1


def run_rect_op(args) -> int:
    """--op rect: geqrf of tall m x cols blocks, the first ``cols`` columns of
    each configuration matrix as a strided view (the reference's embedded
    rectangular route runs torch.geqrf on data[:, :, :cols]); one process,
    N=1 only.  Algorithmic work 2 m cols^2 - 2 cols^3 / 3 flops per matrix."""
    import fastqr

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = inputs.CONFIGS[args.config]
    m, batch = cfg["n"], cfg["batch"]
    cols = args.cols or (3 * m) // 4
    if not 0 < cols <= m:
        raise SystemExit(f"--cols must be in 1..{m}")
    steps = args.steps
    full = inputs.baseline_input(args.config, args.seed, dev)
    a = full[:, :, :cols]
    h = torch.empty_strided((batch, m, cols), (m * cols, 1, m), device=dev, dtype=torch.float32)
    tau = torch.empty((batch, cols), device=dev, dtype=torch.float32)
    ws = torch.empty(max(1, fastqr.workspace_bytes(batch, cols, m)), dtype=torch.uint8, device=dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    def step():
        return fastqr.geqrf(a, out=(h, tau), workspace=ws)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    chk = min(batch, 8)
    q = torch.linalg.householder_product(h[:chk], tau[:chk]).double()
    r = torch.triu(h[:chk, :cols, :].double())
    ad = a[:chk].double()
    e1 = float(((q @ r - ad).flatten(1).norm(dim=1) / ad.flatten(1).norm(dim=1)).max())
    e2 = float(((q.transpose(1, 2) @ q - torch.eye(cols, device=dev, dtype=torch.float64)).flatten(1)
                .norm(dim=1) / cols ** 0.5).max())
    gate = {"recon_rel_f": e1, "orth_rel_f": e2}
    ok = e1 <= 1e-4 and e2 <= 1e-4
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    stream = torch.cuda.current_stream(dev)
    torch.cuda.synchronize(dev)
    with ClockSampler(0) as clk:
        for i in range(steps):
            flush.fill_(float(i))
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        torch.cuda.synchronize(dev)
    clocks = clk.summary()
    ms = sum(s_.elapsed_time(e_) for s_, e_ in zip(starts, ends)) / steps
    mps = batch / (ms / 1e3)
    alg = batch * (2.0 * m * cols * cols - 2.0 * cols ** 3 / 3.0)
    pk = peaks()
    tf32 = pk["bf16_tflops"] / 2.0
    ach = alg / (ms / 1e3) / 1e12
    cpu = None
    if not args.no_cpu:
        threads = os.cpu_count() or 1
        torch.set_num_threads(threads)
        ac = a[:min(batch, 32)].cpu().contiguous()
        torch.geqrf(ac)
        times = []
        t_start = time.perf_counter()
        while len(times) < 3 or time.perf_counter() - t_start < 5.0:
            t0 = time.perf_counter()
            torch.geqrf(ac)
            times.append(time.perf_counter() - t0)
            if time.perf_counter() - t_start > 20.0:
                break
        per = statistics.median(times)
        cpu = {"value": ac.shape[0] / per, "unit": "matrices/s", "cores": threads, "kind": "reference",
               "sample": f"torch.geqrf (host LAPACK) on {ac.shape[0]} of the {batch} {m}x{cols} blocks, "
                         f"median of {len(times)} reps"}
    # blocked path: per part of the batch (two, four for 2048+ columns) a
    # copy-in and the plan's panels, in-block steps and trailing updates
    st = stage_launches(cols, m)
    parts = min(batch, 4 if cols >= 2048 else 2)
    launches = parts * (st["copy_in"] + st["panel"] + st["inblock"] + st["trailing"])
    line = {
        "metric": f"matrices/s ({args.config} rect {m}x{cols})", "value": mps, "unit": "matrices/s",
        "n_gpus": 1, "steps": steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded, the reference generator's distributions)",
        "config": {"workload": f"{args.config} first {cols} columns: {cfg['desc']}", "op": "rect", "m": m,
                   "n": cols, "batch_per_gpu": batch,
                   "l2": f"flushed before every step ({L2_FLUSH_BYTES >> 20} MiB write)"},
        "verified": ok, "gate": gate,
        "roofline": {"kernel": "geqrf (whole op)", "bound": "tensor", "achieved": ach, "peak": tf32,
                     "unit": "TFLOP/s", "frac": ach / tf32, "traffic": None,
                     "peak_source": pk["source"] + "; TF32 dense peak taken as measured bf16 / 2"},
        "cpu_baseline": cpu, "e2e": None, "gpu_launches": steps * launches, "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    return 0 if ok else 1


def run_sweep_op(args) -> int:
    """--op sweep: the small-n path (one warp per matrix, n <= 64) over a
    series of batch sizes, from C1's 1024 up to 10^6 matrices (iid N(0,1),
    n = --n, default 32): device ms per call (L2 flushed), matrices/s and the
    algorithmic HBM rate -- read A (4 n^2 bytes) and write H and tau
    (4 n^2 + 4 n) -- against the measured copy bandwidth.  One process, N = 1."""
    import fastqr

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n = args.n or 32
    if n > 64:
        raise SystemExit("--op sweep times the n <= 64 warp kernel")
    pk = peaks()
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    rows = []
    with ClockSampler(0) as clk:
        for batch in (1024, 4096, 16384, 65536, 262144, 1048576):
            a = inputs.generate_input(batch, n, 0, 17, device=dev)
            h, tau = fastqr.empty_outputs(batch, n, dev)

            def step():
                fastqr.geqrf(a, out=(h, tau))

            for _ in range(3):
                step()
            steps = max(3, min(50, int(2e6 // batch)))
            ms = timed_steps(step, steps, flush, stream)
            gbs = batch * bytes_per_matrix(n) / (ms / 1e3) / 1e9
            rows.append({"batch": batch, "ms_per_call": ms, "matrices_per_s": batch / (ms / 1e3),
                         "hbm_gbs_alg": gbs, "hbm_frac": gbs / pk["hbm_gbs"], "steps": steps})
            del a, h, tau
            torch.cuda.empty_cache()
    # the largest batch verified against the gates on a sample
    a = inputs.generate_input(64, n, 0, 19, device=dev)
    h, tau = fastqr.geqrf(a)
    sys.path.insert(0, str(ROOT / "tests"))
    from gpu_gates import gates
    g = gates(a, h, tau, chunk=64)
    best = max(rows, key=lambda r: r["hbm_frac"])
    line = {
        "metric": f"matrices/s (n={n} geqrf batch sweep)", "value": best["matrices_per_s"], "unit": "matrices/s",
        "n_gpus": 1, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic iid N(0,1) (seeded)",
        "config": {"workload": f"batched {n}x{n} geqrf, batch 1024 .. 1048576", "n": n,
                   "l2": f"flushed before every call ({L2_FLUSH_BYTES >> 20} MiB write)"},
        "verified": bool(g["ok"]), "sweep": rows,
        "roofline": {"kernel": "small", "bound": "hbm", "achieved": best["hbm_gbs_alg"], "peak": pk["hbm_gbs"],
                     "unit": "GB/s", "frac": best["hbm_frac"], "traffic": None, "peak_source": pk["source"]},
        "plan": fastqr.plan(1048576, n), "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)
    return 0 if g["ok"] else 1


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="C2", choices=sorted(inputs.CONFIGS))
    ap.add_argument("--impl", default="fastqr", choices=["fastqr", "reference"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--strong", action="store_true",
                    help="strong scaling (the default): split the configuration's batch over the ranks")
    ap.add_argument("--weak", action="store_true",
                    help="weak scaling: every rank factors a full configuration batch")
    ap.add_argument("--no-per-config", action="store_true",
                    help="skip the per_config block (all five configurations, N = 1)")
    ap.add_argument("--no-gpu-baseline", action="store_true",
                    help="skip the torch.geqrf-on-CUDA comparator")
    ap.add_argument("--cols", type=int, default=None,
                    help="--op rect: columns of the tall blocks (default 3/4 of n)")
    ap.add_argument("--n", type=int, default=None, help="--op sweep: matrix size (default 32)")
    ap.add_argument("--op", default="geqrf", choices=["geqrf", "orgqr", "ormqr", "rect", "sweep"],
                    help="geqrf (the headline); orgqr / ormqr time Q formation / Q^T A from geqrf's factors; "
                         "rect times geqrf of the tall blocks A[:, :, :cols]")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = DEFAULT_STEPS[args.config]
    args.warmup = max(args.warmup, 3)
    args.strong = not args.weak
    if args.impl == "reference":
        return run_reference(args)
    if args.op == "rect":
        return run_rect_op(args)
    if args.op == "sweep":
        return run_sweep_op(args)
    if args.op != "geqrf":
        return run_apply_op(args)
    return run_fastqr(args)


if __name__ == "__main__":
    raise SystemExit(main())
