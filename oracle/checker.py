"""Correctness gates for compact Householder QR -- TEST INFRASTRUCTURE ONLY.

Restates the reference's official checker (official/reference.py:150-266,
``check_implementation``) in numpy float64, plus the gates BASELINE.json's
north star adds:

* official factor gate: ||R - Q^T A||_1 <= 20 * n * eps32 * ||A||_1 per matrix
  (official/reference.py:5,185,213-227);
* official orthogonality gate: max_b ||Q^T Q - I||_1 <= 100 * n * eps32
  (official/reference.py:6,186,229-244);
* relative reconstruction ||A - QR||_F / ||A||_F <= 1e-4 and
  ||Q^T Q - I||_F / sqrt(n) <= 1e-4 (north star);
* per-column parity with float64 geqrf:
  ||h_j - h64_j|| / ||h64_j|| <= 1e-3 and
  |tau_j - tau64_j| / max(|tau64_j|, tiny) <= 1e-3 (north star, on
  well-conditioned inputs only; reflectors of rank-deficient columns are not
  unique in any useful sense).

Q is materialised from (H, tau) by the oracle's float32 Householder product,
mirroring ``torch.linalg.householder_product`` on float32 inputs
(official/reference.py:199); the residuals are then formed in float64
(official/reference.py:205-207).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from . import orgqr_f32

EPS32 = float(np.finfo(np.float32).eps)
FACTOR_RTOL_FACTOR = 20.0  # official/reference.py:5
ORTH_RTOL_FACTOR = 100.0  # official/reference.py:6
RECON_TOL = 1e-4  # north star
ORTH_F_TOL = 1e-4  # north star
COLUMN_TOL = 1e-3  # north star


def _l1(x: np.ndarray) -> np.ndarray:
    """Matrix 1-norm (max column abs sum) per batch entry, like
    torch.linalg.matrix_norm(ord=1) (official/reference.py:163-164)."""
    return np.abs(x).sum(axis=-2).max(axis=-1)


@dataclass
class QRReport:
    ok: bool
    message: str
    factor_scaled: np.ndarray = field(default_factory=lambda: np.zeros(0))
    orth_scaled: float = 0.0
    recon_rel_f: float = 0.0
    orth_rel_f: float = 0.0
    tri_scaled: float = 0.0


def check_qr(a, h, tau) -> QRReport:
    """Official gates plus the north star's Frobenius gates.

    ``a``: float32 [b, n, n]; ``h``: float32 [b, n, n] (logical indexing);
    ``tau``: float32 [b, n].
    """
    a = np.asarray(a, dtype=np.float32)
    h = np.asarray(h)
    tau = np.asarray(tau)
    if a.ndim != 3 or a.shape[1] != a.shape[2]:
        return QRReport(False, "A must have shape (batch, n, n)")
    batch, n, _ = a.shape
    if h.shape != (batch, n, n):
        return QRReport(False, f"H shape must be {(batch, n, n)}, got {h.shape}")
    if tau.shape != (batch, n):
        return QRReport(False, f"tau shape must be {(batch, n)}, got {tau.shape}")
    if h.dtype != np.float32 or tau.dtype != np.float32:
        return QRReport(False, "H and tau must be float32")
    if not np.isfinite(h).all():
        return QRReport(False, "H contains NaN or Inf")
    if not np.isfinite(tau).all():
        return QRReport(False, "tau contains NaN or Inf")

    q = orgqr_f32(h, tau).astype(np.float64)
    r = np.triu(h.astype(np.float64))
    a64 = a.astype(np.float64)
    if not np.isfinite(q).all():
        return QRReport(False, "Q materialized from `(H, tau)` contains NaN or Inf")

    nn = max(n, 1)
    projected = np.swapaxes(q, -1, -2) @ a64
    factor_residual = _l1(r - projected)
    factor_scale = _l1(a64)
    factor_allowed = FACTOR_RTOL_FACTOR * nn * EPS32 * factor_scale
    factor_scaled = factor_residual / (EPS32 * nn * np.maximum(factor_scale, 1e-30))
    eye = np.eye(n)
    qtq = np.swapaxes(q, -1, -2) @ q
    orth_residual = float(_l1(qtq - eye).max()) if batch else 0.0
    orth_scaled = orth_residual / (EPS32 * nn)
    lower = np.tril(projected, -1)
    tri_scaled = float((_l1(lower) / (EPS32 * nn * np.maximum(factor_scale, 1e-30))).max()) if batch else 0.0

    recon = q @ r
    fa = np.sqrt((a64 ** 2).sum(axis=(-2, -1)))
    recon_rel = np.sqrt(((recon - a64) ** 2).sum(axis=(-2, -1))) / np.maximum(fa, 1e-300)
    orth_rel = np.sqrt(((qtq - eye) ** 2).sum(axis=(-2, -1))) / np.sqrt(nn)

    rep = QRReport(True, "", factor_scaled, orth_scaled,
                   float(recon_rel.max()) if batch else 0.0,
                   float(orth_rel.max()) if batch else 0.0, tri_scaled)
    if batch and (factor_residual > factor_allowed).any():
        worst = int(factor_scaled.argmax())
        rep.ok = False
        rep.message = (f"R - Q.T @ A is too large: matrix={worst}, "
                       f"scaled={factor_scaled[worst]:.3g}")
        return rep
    if orth_residual > ORTH_RTOL_FACTOR * nn * EPS32:
        rep.ok = False
        rep.message = f"Q is not orthogonal enough: scaled={orth_scaled:.3g}"
        return rep
    if rep.recon_rel_f > RECON_TOL:
        rep.ok = False
        rep.message = f"||A-QR||_F/||A||_F = {rep.recon_rel_f:.3g} > {RECON_TOL}"
        return rep
    if rep.orth_rel_f > ORTH_F_TOL:
        rep.ok = False
        rep.message = f"||Q^TQ-I||_F/sqrt(n) = {rep.orth_rel_f:.3g} > {ORTH_F_TOL}"
        return rep
    rep.message = (f"scaled_factor_residual={factor_scaled.max() if batch else 0:.3g}; "
                   f"scaled_orthogonality_residual={orth_scaled:.3g}; "
                   f"recon_rel_f={rep.recon_rel_f:.3g}; orth_rel_f={rep.orth_rel_f:.3g}")
    return rep


def column_errors(h, tau, h64, tau64):
    """Per-column relative errors against a float64 factorisation.

    Returns (h_err[b, n], tau_err[b, n]) with
    h_err = ||h_j - h64_j|| / ||h64_j|| and
    tau_err = |tau_j - tau64_j| / max(|tau64_j|, tiny).
    """
    h = np.asarray(h, dtype=np.float64)
    h64 = np.asarray(h64, dtype=np.float64)
    tau = np.asarray(tau, dtype=np.float64)
    tau64 = np.asarray(tau64, dtype=np.float64)
    num = np.sqrt(((h - h64) ** 2).sum(axis=-2))
    den = np.sqrt((h64 ** 2).sum(axis=-2))
    h_err = np.where(den > 0, num / np.maximum(den, 1e-300), num)
    tau_err = np.abs(tau - tau64) / np.maximum(np.abs(tau64), 1e-30)
    return h_err, tau_err


def check_columns(h, tau, h64, tau64, tol: float = COLUMN_TOL, matrices=None) -> tuple[bool, str]:
    """North-star per-column parity gate on the selected (well-conditioned) matrices."""
    h_err, tau_err = column_errors(h, tau, h64, tau64)
    if matrices is not None:
        h_err = h_err[matrices]
        tau_err = tau_err[matrices]
    if h_err.size == 0:
        return True, "no matrices selected"
    hm, tm = float(h_err.max()), float(tau_err.max())
    ok = hm <= tol and tm <= tol
    return ok, f"max column rel err H={hm:.3g} tau={tm:.3g} (tol {tol})"
