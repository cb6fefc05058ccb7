"""The CPU oracle against the reference's own outputs (tests/golden, made by make_golden.py).

Pins oracle.householder before it is trusted as the checker of the CUDA path:
* its factorisation passes the reference gate on every golden case;
* its numpy gate reproduces the reference gate's verdicts and residual magnitudes;
* on well-conditioned cases its H matches the reference CPU path and LAPACK elementwise;
* |diag R| matches LAPACK on every case.
"""

import numpy as np
import pytest

import oracle

WELL_CONDITIONED = {"dense", "band", "upper", "diagonal", "rowscale", "clustered"}


def _cases(meta):
    return [c for c in meta["cases"]]


def test_golden_cases_present(golden):
    z, meta = golden
    assert len(meta["cases"]) >= 15
    for c in meta["cases"]:
        for s in ("A", "H_ref", "tau_ref", "H_lapack", "tau_lapack"):
            assert f"{c['key']}_{s}" in z.files
        assert c["ref_ok"] and c["lapack_ok"]


def test_oracle_passes_reference_gate(golden):
    z, meta = golden
    for c in _cases(meta):
        A = z[c["key"] + "_A"]
        H, tau = oracle.geqrf_blocked(A)
        ok, info = oracle.check(A, H, tau)
        assert ok, (c["args"], info)
        assert info["scaled_factor_residual"] < 2.0


def test_numpy_gate_matches_reference_gate(golden):
    """oracle.check on the reference's own outputs agrees with the reference checker."""
    z, meta = golden
    for c in _cases(meta):
        k = c["key"]
        ok, info = oracle.check(z[k + "_A"], z[k + "_H_ref"], z[k + "_tau_ref"])
        assert ok == c["ref_ok"]
        ref = c["ref_check"].get("scaled_factor_residual")
        if ref is not None and ref > 1e-3:
            # Q is rebuilt by a different FP32 ORGQR here, so only the magnitude must agree.
            assert 0.25 * ref <= info["scaled_factor_residual"] <= 4.0 * ref + 1e-3, (c["args"], info, ref)


def test_oracle_matches_reference_elementwise_when_well_conditioned(golden):
    z, meta = golden
    for c in _cases(meta):
        if c["args"].get("case", "dense") not in WELL_CONDITIONED:
            continue
        k = c["key"]
        A = z[k + "_A"]
        n = A.shape[-1]
        H, tau = oracle.geqrf_blocked(A)
        scale = np.abs(A).sum(axis=-2).max(axis=-1)[:, None, None]
        tol = 20.0 * n * oracle.EPS32
        for ref in ("_H_ref", "_H_lapack"):
            d = np.abs(H - z[k + ref]) / np.maximum(scale, 1e-30)
            assert d.max() <= tol, (c["args"], ref, d.max(), tol)
        assert np.abs(tau - z[k + "_tau_lapack"]).max() <= 1e-4, c["args"]


def test_oracle_diag_r_matches_lapack(golden):
    z, meta = golden
    for c in _cases(meta):
        k = c["key"]
        A = z[k + "_A"]
        n = A.shape[-1]
        H, _ = oracle.geqrf_blocked(A)
        d = np.abs(np.abs(np.diagonal(H, axis1=1, axis2=2)) - np.abs(np.diagonal(z[k + "_H_lapack"], axis1=1, axis2=2)))
        scale = np.abs(A).sum(axis=-2).max(axis=-1)[:, None] * n * oracle.EPS32
        assert (d / np.maximum(scale, 1e-30)).max() <= 20.0, c["args"]


@pytest.mark.parametrize("nb", [1, 3, 8, 16, 32])
def test_oracle_block_width_invariance(nb):
    rng = np.random.default_rng(nb)
    A = rng.standard_normal((2, 37, 37)).astype(np.float32)
    H, tau = oracle.geqrf_blocked(A, nb=nb)
    H1, tau1 = oracle.geqrf_blocked(A, nb=37)
    assert np.abs(H - H1).max() < 1e-4 and np.abs(tau - tau1).max() < 1e-5
    ok, _ = oracle.check(A, H, tau)
    assert ok


def test_oracle_gate_rejects_planted_error():
    """A mistake planted in the oracle's output must fail the gate (the gate is live)."""
    rng = np.random.default_rng(7)
    A = rng.standard_normal((2, 24, 24)).astype(np.float32)
    H, tau = oracle.geqrf_blocked(A)
    H_bad = H.copy()
    H_bad[1, 3, 7] += 1e-2  # perturb one R entry
    ok, info = oracle.check(A, H_bad, tau)
    assert not ok
    tau_bad = tau.copy()
    tau_bad[0, 5] *= 1.01  # perturb one reflector coefficient -> Q loses orthogonality
    ok, info = oracle.check(A, H, tau_bad)
    assert not ok


def test_larfg_conventions():
    # x == 0: identity reflector, diagonal keeps alpha (reference submission.py:97-105).
    d, t, v = oracle.larfg(np.array([-3.0], np.float32), np.zeros((1, 4), np.float32))
    assert d[0] == -3.0 and t[0] == 0.0 and not v.any()
    # sign convention: beta = -sign(alpha) * norm.
    d, t, v = oracle.larfg(np.array([3.0], np.float32), np.array([[4.0]], np.float32))
    assert d[0] == pytest.approx(-5.0) and t[0] == pytest.approx(1.6) and v[0, 0] == pytest.approx(0.5)
