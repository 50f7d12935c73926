"""Seeded synthetic inputs for batched square QR.

``generate_input`` reproduces the reference task's input generator
(official/reference.py:30-142): a seeded ``torch.Generator`` on the target
device draws an N(0, 1) base batch, then one conditioning profile is applied.
The draw order is part of the contract (it decides every value), so the steps
below follow the same sequence; the code is our own.

``baseline_input`` builds the five configurations of the benchmark plan
(C1..C5).  C1, C2 and C5 are plain ``generate_input`` calls; C3 (mixed
structure) and C4 (near rank deficient) have no counterpart in the reference
generator and are written from their textual definitions.
"""
from __future__ import annotations

import torch

# Conditioning profiles of the "mixed" case and their relative weights
# (official/reference.py:25-28): dense is the weighted majority.
MIXED_PROFILES = ("dense", "rankdef", "nearrank", "clustered", "band", "rowscale", "nearcollinear")
MIXED_WEIGHTS = (6.0, 1.0, 1.0, 1.0, 1.0, 1.0, 1.0)
CASES = ("dense", "upper", "diagonal", "rankdef", "nearrank", "clustered", "band",
         "nearcollinear", "rowscale", "mixed")


def _column_scale(x: torch.Tensor, cond: int) -> torch.Tensor:
    # columns multiplied by logspace(0, -cond, n) (official/reference.py:9-15)
    if not cond:
        return x.contiguous()
    n = x.shape[-1]
    return x * torch.logspace(0.0, -float(cond), n, device=x.device, dtype=torch.float32)


def _profile(x: torch.Tensor, case: str, cond: int, gen: torch.Generator) -> torch.Tensor:
    """One conditioning profile applied to a drawn base batch (official/reference.py:30-90)."""
    cnt, n = x.shape[0], x.shape[-1]
    dev = x.device
    f32 = torch.float32
    if case == "dense":
        return _column_scale(x, cond)
    if case == "upper":
        y = torch.triu(x)
        y.diagonal(dim1=-2, dim2=-1).add_(torch.linspace(1.0, 0.25, n, device=dev, dtype=f32))
        return _column_scale(y, cond)
    if case == "diagonal":
        d = torch.randn((cnt, n), device=dev, dtype=f32, generator=gen)
        signs = d.sign().clamp(min=0.0).mul(2.0).sub(1.0)
        mags = torch.logspace(0.0, -float(max(cond, 2)), n, device=dev, dtype=f32)
        return torch.diag_embed(signs * mags)
    if case == "rankdef":
        keep = max(1, (3 * n) // 4)
        x[:, :, keep:] = 0.0
        return _column_scale(x, cond)
    if case == "nearrank":
        keep = max(1, (3 * n) // 4)
        extra = n - keep
        if extra > 0:
            eps_noise = torch.randn((cnt, n, extra), device=dev, dtype=f32, generator=gen)
            x[:, :, keep:] = x[:, :, :extra] + 1.0e-5 * eps_noise
        return _column_scale(x, cond)
    if case == "clustered":
        s = torch.ones((n,), device=dev, dtype=f32)
        s[n // 2:] = 4.0 * torch.finfo(f32).eps
        if n >= 8:
            s[max(0, n // 2 - 2):min(n, n // 2 + 2)] = torch.sqrt(
                torch.tensor(torch.finfo(f32).eps, device=dev))
        return x * s
    if case == "band":
        bw = max(2, min(32, n // 32))
        idx = torch.arange(n, device=dev)
        y = x * ((idx[:, None] - idx[None, :]).abs() <= bw)
        y.diagonal(dim1=-2, dim2=-1).add_(torch.linspace(1.0, 0.5, n, device=dev, dtype=f32))
        return _column_scale(y, cond)
    if case == "nearcollinear":
        base = torch.randn((cnt, n, 1), device=dev, dtype=f32, generator=gen)
        noise = torch.randn((cnt, n, n), device=dev, dtype=f32, generator=gen)
        return _column_scale(base.expand(cnt, n, n) + 1.0e-4 * noise, cond)
    if case == "rowscale":
        rs = torch.logspace(0.0, -float(max(cond, 4)), n, device=dev, dtype=f32)
        return rs.reshape(1, n, 1) * x
    raise ValueError(f"unknown QR test case: {case}")


def _mixed(x: torch.Tensor, cond: int, gen: torch.Generator) -> torch.Tensor:
    """Per-matrix profiles at seeded random positions (official/reference.py:93-122)."""
    cnt = x.shape[0]
    dev = x.device
    w = torch.tensor(MIXED_WEIGHTS, dtype=torch.float32, device=dev)
    labels = torch.multinomial(w, cnt, replacement=True, generator=gen)
    if cnt >= 2:
        dense = labels == 0
        if not bool(dense.any()):
            labels[int(torch.randint(0, cnt, (1,), device=dev, generator=gen))] = 0
        elif bool(dense.all()):
            where = int(torch.randint(0, cnt, (1,), device=dev, generator=gen))
            labels[where] = int(torch.randint(1, len(MIXED_PROFILES), (1,), device=dev, generator=gen))
    for code, name in enumerate(MIXED_PROFILES):
        sel = labels == code
        if bool(sel.any()):
            x[sel] = _profile(x[sel], name, cond, gen)
    return x


def generate_input(batch: int, n: int, cond: int, seed: int, case: str = "dense",
                   device=None) -> torch.Tensor:
    """Seeded float32 batch [batch, n, n], row-major contiguous
    (official/reference.py:125-142).  ``device`` defaults to CUDA when present."""
    if batch <= 0 or n <= 0 or cond < 0:
        raise ValueError("batch and n must be positive, cond non-negative")
    if device is None:
        device = "cuda" if torch.cuda.is_available() else "cpu"
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    case = case.lower()
    x = torch.randn((batch, n, n), device=device, dtype=torch.float32, generator=gen)
    x = _mixed(x, cond, gen) if case == "mixed" else _profile(x, case, cond, gen)
    return x.contiguous()


# ---------------------------------------------------------------------------
# Benchmark configurations (C1..C5)
# ---------------------------------------------------------------------------

CONFIGS = {
    "C1": {"batch": 1024, "n": 32, "desc": "1024 x 32^2 iid N(0,1)"},
    "C2": {"batch": 256, "n": 256, "desc": "256 x 256^2 graded: column j scaled by 10^(-6j/255)"},
    "C3": {"batch": 512, "n": 512, "desc": "512 x 512^2 mixed: 50% N(0,1), 25% rank-256 UV^T, 25% upper-tri (diag N(0,1)+5)"},
    "C4": {"batch": 64, "n": 1024, "desc": "64 x 1024^2 near rank deficient: last 256 columns = X C/sqrt(768) + 1e-6 noise"},
    "C5": {"batch": 16, "n": 4096, "desc": "16 x 4096^2 iid N(0,1)"},
}

# C3 structure labels
C3_DENSE, C3_LOWRANK, C3_UPPER = 0, 1, 2


def c3_labels(batch: int, seed: int) -> torch.Tensor:
    """Structure label per matrix for C3: the first half dense, the next
    quarter rank-256, the last quarter upper triangular, then the positions are
    shuffled with the seed so no contiguous shard is homogeneous."""
    lab = torch.empty(batch, dtype=torch.int64)
    h = batch // 2
    q = batch // 4
    lab[:h] = C3_DENSE
    lab[h:h + q] = C3_LOWRANK
    lab[h + q:] = C3_UPPER
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    return lab[torch.randperm(batch, generator=g)]


def _c3_matrix(label: int, n: int, seed: int, device) -> torch.Tensor:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    if label == C3_DENSE:
        return torch.randn((n, n), device=device, dtype=torch.float32, generator=g)
    if label == C3_LOWRANK:
        r = n // 2
        u = torch.randn((n, r), device=device, dtype=torch.float32, generator=g) / (r ** 0.5)
        v = torch.randn((n, r), device=device, dtype=torch.float32, generator=g) / (r ** 0.5)
        return u @ v.T
    m = torch.triu(torch.randn((n, n), device=device, dtype=torch.float32, generator=g))
    m.diagonal().copy_(torch.randn((n,), device=device, dtype=torch.float32, generator=g) + 5.0)
    return m


def _c4_batch(batch: int, n: int, seed: int, device) -> torch.Tensor:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    keep = (3 * n) // 4
    x = torch.randn((batch, n, n), device=device, dtype=torch.float32, generator=g)
    comb = torch.randn((batch, keep, n - keep), device=device, dtype=torch.float32, generator=g)
    noise = torch.randn((batch, n, n - keep), device=device, dtype=torch.float32, generator=g)
    x[:, :, keep:] = (x[:, :, :keep] @ comb) / (keep ** 0.5) + 1.0e-6 * noise
    return x.contiguous()


def baseline_input(name: str, seed: int = 0, device=None, batch: int | None = None,
                   first: int = 0) -> torch.Tensor:
    """Input batch of configuration ``name`` (C1..C5).

    ``batch`` overrides the configured batch (tests use small batches of the
    same distribution); ``first`` is the global index of the first matrix, so a
    rank that owns matrices [first, first+batch) of C3 builds exactly its
    share of the global batch."""
    if name not in CONFIGS:
        raise ValueError(f"unknown config {name}")
    cfg = CONFIGS[name]
    n = cfg["n"]
    b = cfg["batch"] if batch is None else batch
    if device is None:
        device = "cuda" if torch.cuda.is_available() else "cpu"
    if name == "C1":
        return generate_input(b, n, 0, seed, device=device)
    if name == "C2":
        return generate_input(b, n, 6, seed, device=device)
    if name == "C5":
        return generate_input(b, n, 0, seed, device=device)
    if name == "C4":
        return _c4_batch(b, n, seed, device)
    total = max(cfg["batch"], first + b)
    labels = c3_labels(total, seed)
    out = torch.empty((b, n, n), device=device, dtype=torch.float32)
    for i in range(b):
        gi = first + i
        out[i] = _c3_matrix(int(labels[gi]), n, seed * 1_000_003 + gi, device)
    return out


def well_conditioned_mask(name: str, batch: int, seed: int = 0, first: int = 0) -> torch.Tensor:
    """Matrices on which the per-column H/tau parity gate applies: all of C1
    and C5, the dense half of C3; none of C2 (graded, cond ~1e6) or C4."""
    if name in ("C1", "C5"):
        return torch.ones(batch, dtype=torch.bool)
    if name == "C3":
        total = max(CONFIGS["C3"]["batch"], first + batch)
        return c3_labels(total, seed)[first:first + batch] == C3_DENSE
    return torch.zeros(batch, dtype=torch.bool)
