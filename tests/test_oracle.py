"""The CPU oracle pinned against the reference's golden vectors (CPU only).

Fixtures come from tests/golden/make_golden.py, which ran the reference's
own generator, checker and torch.geqrf (its contract, official/reference.py:
125-127) in the build container.
"""
import numpy as np
import pytest

import oracle
from oracle import checker

ILL_CONDITIONED = {"s8_nearrank", "s8_nearcollinear"}


def _cases(meta):
    return sorted(meta["cases"])


def test_oracle_f64_matches_float64_geqrf(golden):
    """oracle.geqrf_f64 == LAPACK dgeqrf (torch.geqrf on float64) per column.
    Same reflector sign convention, same tau, to double rounding."""
    data, meta = golden
    for name in _cases(meta):
        a = data[f"{name}.A"]
        h, t = oracle.geqrf_f64(a)
        he, te = checker.column_errors(h, t, data[f"{name}.H64"], data[f"{name}.tau64"])
        tol = 1e-9 if name in ILL_CONDITIONED else 1e-12
        assert he.max() <= tol and te.max() <= tol, (name, he.max(), te.max())


def test_oracle_f32_within_float_accuracy_of_geqrf(golden):
    data, meta = golden
    for name in _cases(meta):
        if name in ILL_CONDITIONED:
            continue
        a = data[f"{name}.A"]
        h, t = oracle.geqrf_f32(a)
        ok, msg = checker.check_columns(h, t, data[f"{name}.H64"], data[f"{name}.tau64"], tol=1e-4)
        assert ok, (name, msg)
        # and torch.geqrf's own float32 output is equally close
        ok, msg = checker.check_columns(data[f"{name}.H32"], data[f"{name}.tau32"],
                                        data[f"{name}.H64"], data[f"{name}.tau64"], tol=1e-4)
        assert ok, (name, msg)


def test_last_tau_is_zero_and_zero_columns_give_zero_tau(golden):
    data, meta = golden
    for name in _cases(meta):
        _, t = oracle.geqrf_f64(data[f"{name}.A"])
        assert np.all(t[:, -1] == 0.0)
    # rankdef: the trailing quarter of columns is exactly zero -> tau == 0 there
    _, t = oracle.geqrf_f64(data["n96_rankdef.A"])
    assert np.all(t[:, 72:] == 0.0)
    assert np.all(data["n96_rankdef.tau64"][:, 72:] == 0.0)


@pytest.mark.parametrize("nb", [1, 3, 5, 8, 32, 64])
def test_blocked_compact_wy_equals_unblocked(golden, nb):
    """The blocked compact-WY restatement (the GPU's algorithm) equals xGEQR2."""
    data, meta = golden
    for name in ("pub_20x32", "n65", "n130_mixed", "mixed_24"):
        a = data[f"{name}.A"]
        h, t = oracle.geqrf_f64(a)
        hb, tb = oracle.geqrf_blocked_f64(a, nb)
        he, te = checker.column_errors(hb, tb, h, t)
        assert he.max() < 1e-11 and te.max() < 1e-11, (name, nb, he.max())


def test_blocked_matches_reference_blocked_prototype(golden):
    """Against the reference's tools/blocked_qr_reference.py (compact-wy)."""
    data, meta = golden
    for name, m in meta["blocked"].items():
        a = data[f"{name}.A"]
        hb, tb = oracle.geqrf_blocked_f64(a, m["panel_width"])
        ok, msg = checker.check_columns(data[f"{name}.H"], data[f"{name}.tau"], hb, tb, tol=1e-4)
        assert ok, (name, msg)
        assert m["official_ok"]


def test_checker_agrees_with_official_checker(golden):
    """Our restated gates give the official verdicts and similar residuals."""
    data, meta = golden
    for name, m in meta["cases"].items():
        rep = checker.check_qr(data[f"{name}.A"], data[f"{name}.H32"], data[f"{name}.tau32"])
        assert rep.ok == m["official_ok"] == True, (name, rep.message)
        fields = dict(kv.split("=") for kv in m["official_message"].split("; "))
        off = float(fields["scaled_factor_residual"])
        ours = float(rep.factor_scaled.max())
        assert abs(ours - off) <= 0.5 * max(off, 0.05), (name, ours, off)
        off_o = float(fields["scaled_orthogonality_residual"])
        assert abs(rep.orth_scaled - off_o) <= 0.5 * max(off_o, 0.1), (name, rep.orth_scaled, off_o)


def test_checker_rejects_planted_errors(golden):
    """A mistake planted in the oracle's output must be caught."""
    data, _ = golden
    a = data["pub_20x32.A"]
    h, t = oracle.geqrf_f32(a)
    assert checker.check_qr(a, h, t).ok
    bad_tau = t.copy()
    bad_tau[3, 5] *= 1.01
    assert not checker.check_qr(a, h, bad_tau).ok
    bad_h = h.copy()
    bad_h[7, 20, 4] += 1e-3  # one Householder vector entry
    assert not checker.check_qr(a, bad_h, t).ok
    flipped = h.copy()
    flipped[2, 9, 9] *= -1.0  # sign of one R diagonal entry
    assert not checker.check_qr(a, flipped, t).ok
    nan_h = h.copy()
    nan_h[0, 0, 0] = np.nan
    assert not checker.check_qr(a, nan_h, t).ok
    h64, t64 = oracle.geqrf_f64(a)
    ok, _ = checker.check_columns(h, t, h64, t64)
    assert ok
    ok, _ = checker.check_columns(bad_h, t, h64, t64, tol=1e-5)
    assert not ok


def _tf32(x):
    m, e = np.frexp(x)
    return np.ldexp(np.round(m * 2048.0) / 2048.0, e)


def test_plain_tf32_trailing_update_fails_the_factor_gate(golden):
    """Negative control mirroring the reference's evidence
    (tests/test_qr_smoke.py:217-229): a compact-WY QR whose trailing-update
    operands are rounded to TF32 fails the official factor gate.  This is why
    the tensor-core update uses split (3xTF32) precision."""
    data, _ = golden
    a = data["s8_dense.A"]
    b, n, _ = a.shape
    work = a.astype(np.float32).copy()
    tau = np.zeros((b, n), np.float32)
    pw = 3
    for k in range(0, n, pw):
        w = min(pw, n - k)
        panel = np.ascontiguousarray(work[:, k:, k:k + w])
        ph, pt = oracle.geqrf_f32(np.pad(panel, ((0, 0), (0, 0), (0, panel.shape[1] - w))))
        ph = ph[:, :, :w]
        pt = pt[:, :w]
        work[:, k:, k:k + w] = ph
        tau[:, k:k + w] = pt
        if k + w >= n:
            continue
        m = n - k
        v = np.zeros((b, m, w), np.float32)
        for j in range(w):
            v[:, j, j] = 1.0
            v[:, j + 1:, j] = ph[:, j + 1:, j]
        t = np.zeros((b, w, w), np.float32)
        for j in range(w):
            t[:, j, j] = pt[:, j]
            if j:
                y = -pt[:, j, None] * np.einsum("bri,br->bi", v[:, :, :j], v[:, :, j])
                t[:, :j, j] = np.einsum("bil,bl->bi", t[:, :j, :j], y)
        c = work[:, k:, k + w:]
        proj = _tf32(np.swapaxes(v, 1, 2)) @ _tf32(c)
        mid = _tf32(np.swapaxes(t, 1, 2)) @ _tf32(proj)
        work[:, k:, k + w:] = c - (_tf32(v) @ _tf32(mid)).astype(np.float32)
    rep = checker.check_qr(a, work.astype(np.float32), tau)
    assert not rep.ok
    assert "R - Q.T @ A is too large" in rep.message


@pytest.mark.parametrize("b,m,n", [(3, 50, 20), (2, 129, 64), (2, 33, 33), (1, 300, 31), (2, 5, 9)])
def test_rect_oracle_matches_numpy_lapack(b, m, n):
    """The m x n restatement (xGEQR2 steps, min(m, n) reflectors) against
    numpy's LAPACK dgeqrf (np.linalg.qr mode='raw'), and against the square
    oracle bitwise when m == n."""
    rng = np.random.default_rng(m * 1000 + n)
    a = rng.standard_normal((b, m, n)).astype(np.float32)
    h, t = oracle.geqrf_rect_f64(a)
    assert h.shape == (b, m, n) and t.shape == (b, min(m, n))
    for i in range(b):
        hr, tr = np.linalg.qr(a[i].astype(np.float64), mode="raw")
        assert np.abs(hr.T - h[i]).max() <= 1e-12 * max(1.0, np.abs(h[i]).max())
        assert np.abs(tr[:min(m, n)] - t[i]).max() <= 1e-12
    if m == n:
        h2, t2 = oracle.geqrf_f64(a)
        assert np.array_equal(h2, h) and np.array_equal(t2, t)


def test_rank64_block_update_algebra():
    """The rank-64 plan's algebra restated in float64. With S =
    strict_upper(V^T V) assembled from the two panels' S11, S22 and the Gram
    block S12 = V1^T V2, the update C - V Y with (I + D S^T) Y = D V^T C
    (forward substitution, D = diag(tau)) equals applying the 64 reflectors
    one by one; the in-block step (the first panel's 32 reflectors, S11) does
    likewise; and S12 needs only the rows below the first panel, the Gram
    step's row range (V2 is zero above them)."""
    rng = np.random.default_rng(3)
    m = 200
    a = rng.standard_normal((1, m, 64)).astype(np.float32)
    h, tau = oracle.geqrf_rect_f64(a)
    h, tau = h[0], tau[0]
    v = np.tril(h, -1)
    v[np.arange(64), np.arange(64)] = 1.0
    c = rng.standard_normal((m, 20))

    def one_by_one(vs, taus, x):
        x = x.copy()
        for j in range(vs.shape[1]):
            x -= taus[j] * np.outer(vs[:, j], vs[:, j] @ x)
        return x

    def block_update(vs, taus, s, x):
        w = vs.T @ x
        y = np.zeros_like(w)
        for l in range(len(taus)):
            y[l] = taus[l] * (w[l] - s[:l, l] @ y[:l])
        return x - vs @ y

    v1, v2 = v[:, :32], v[:, 32:]
    s11, s22 = np.triu(v1.T @ v1, 1), np.triu(v2.T @ v2, 1)
    s12 = v1[32:].T @ v2[32:]
    assert np.allclose(s12, v1.T @ v2, rtol=0, atol=1e-12)
    s = np.zeros((64, 64))
    s[:32, :32], s[32:, 32:], s[:32, 32:] = s11, s22, s12
    assert np.allclose(block_update(v, tau, s, c), one_by_one(v, tau, c), rtol=0, atol=1e-11)
    assert np.allclose(block_update(v1, tau[:32], s11, c), one_by_one(v1, tau[:32], c), rtol=0, atol=1e-11)
