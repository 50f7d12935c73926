"""QR gates evaluated on the GPU, for sizes where the CPU oracle is too slow.

The same gates as oracle/checker.py (the official ones from
official/reference.py:182-244 plus the north star's Frobenius gates), with Q
materialised by torch.linalg.householder_product in float32 exactly as the
official checker does (official/reference.py:199) and the residuals formed in
float64.  Test infrastructure only.
"""
from __future__ import annotations

import math

import torch

EPS32 = torch.finfo(torch.float32).eps


@torch.no_grad()
def gates(a: torch.Tensor, h: torch.Tensor, tau: torch.Tensor, chunk: int = 8) -> dict:
    """Square (batch, n, n) or tall (batch, m, n) inputs: Q is the m x n thin
    factor, R the leading n x n upper triangle of H, and the official scales
    use m (= n for the square case)."""
    batch, m, n = a.shape
    worst = {"factor_scaled": 0.0, "orth_scaled": 0.0, "recon_rel_f": 0.0, "orth_rel_f": 0.0,
             "factor_ok": True, "finite": True}
    eye = torch.eye(n, device=a.device, dtype=torch.float64)
    for s in range(0, batch, chunk):
        e = min(batch, s + chunk)
        hs, ts, as_ = h[s:e], tau[s:e], a[s:e].double()
        worst["finite"] &= bool(torch.isfinite(hs).all()) and bool(torch.isfinite(ts).all())
        q = torch.linalg.householder_product(hs, ts).double()
        r = torch.triu(hs.double()[:, :n, :])
        proj = q.transpose(-1, -2) @ as_
        l1 = lambda x: torch.linalg.matrix_norm(x, ord=1, dim=(-2, -1))
        fres = l1(r - proj)
        fscale = l1(as_)
        fscaled = fres / (EPS32 * m * fscale.clamp_min(1e-30))
        worst["factor_ok"] &= bool((fres <= 20.0 * m * EPS32 * fscale).all())
        worst["factor_scaled"] = max(worst["factor_scaled"], float(fscaled.max()))
        qtq = q.transpose(-1, -2) @ q - eye
        worst["orth_scaled"] = max(worst["orth_scaled"], float(l1(qtq).max()) / (EPS32 * m))
        recon = (q @ r - as_).flatten(1).norm(dim=1) / as_.flatten(1).norm(dim=1).clamp_min(1e-300)
        worst["recon_rel_f"] = max(worst["recon_rel_f"], float(recon.max()))
        worst["orth_rel_f"] = max(worst["orth_rel_f"],
                                  float(qtq.flatten(1).norm(dim=1).max()) / math.sqrt(n))
    worst["orth_ok"] = worst["orth_scaled"] <= 100.0
    worst["ok"] = (worst["finite"] and worst["factor_ok"] and worst["orth_ok"]
                   and worst["recon_rel_f"] <= 1e-4 and worst["orth_rel_f"] <= 1e-4)
    return worst


@torch.no_grad()
def column_errors(h, tau, h64, tau64):
    """Per-column relative errors (see oracle.checker.column_errors), on device."""
    h = h.double()
    h64 = h64.double()
    num = (h - h64).norm(dim=-2)
    den = h64.norm(dim=-2)
    h_err = torch.where(den > 0, num / den.clamp_min(1e-300), num)
    tau_err = (tau.double() - tau64.double()).abs() / tau64.double().abs().clamp_min(1e-30)
    return h_err, tau_err
