"""Pins the CPU oracle to the reference's own known-answer self-check.

The reference's SH consumer ships a self-check main() (SHGradientConsumer.cu:
436-624, same in controls/ManualSH.cu:464-652): a deterministic 257-Gaussian
fixture with clamped channels, invisible Gaussians (some sitting on the camera),
zero and non-unit seeds, nonzero incoming position adjoints and nonzero moments,
checked for degrees 0-3 and every update mode against a double-precision
central-difference gradient of the SH colour loss plus the closed-form Adam
equations, with fixed tolerances. The same fixture, expectations and tolerances
applied to the oracle pin it to the reference's semantics.
"""

import numpy as np
import pytest

import oracle

MODES = [("sgd", False), ("adam", False), ("split_adam", True),
         ("split_torch_adam", True), ("split_torch_adam", False)]


@pytest.fixture(scope="module")
def fixture():
    return oracle.reference_fixture()


def _close(got, expected, atol, rtol, what):
    got = np.asarray(got, np.float64)
    bad = ~np.isfinite(got) | (np.abs(got - expected) > atol + rtol * np.abs(expected))
    assert not bad.any(), (
        f"{what}: {int(bad.sum())} components outside {atol}+{rtol}|ref|; first "
        f"got={got[bad][:3]} ref={expected[bad][:3]}")


@pytest.mark.parametrize("degree", [0, 1, 2, 3])
@pytest.mark.parametrize("mode,snapshot", MODES)
def test_oracle_matches_reference_self_check(fixture, degree, mode, snapshot):
    dm, coeff, first, second = oracle.run_fixture_mode(fixture, degree, mode, snapshot)
    e_dm, e_coeff, e_first, e_second = oracle.fixture_expectations(fixture, degree, mode)
    tol = oracle.FIXTURE_TOLERANCES
    _close(dm, e_dm, *tol["dm"], what="position adjoint")
    _close(coeff, e_coeff, *tol["coeff"], what="coefficients")
    if e_first is not None:
        _close(first, e_first, *tol["first"], what="first moment")
        _close(second, e_second, *tol["second"], what="second moment")


def test_sgd_leaves_invisible_gaussians_alone(fixture):
    dm, coeff, _, _ = oracle.run_fixture_mode(fixture, 3, "sgd")
    invisible = fixture["radii"] == 0
    assert np.array_equal(coeff[invisible], fixture["coeff"][invisible])
    assert np.array_equal(dm[invisible], fixture["initial"][invisible])


def test_adam_updates_invisible_and_inactive_terms(fixture):
    """Zero gradients still advance Adam (SHGradientConsumer.cu:200-202)."""
    _, coeff, first, _ = oracle.run_fixture_mode(fixture, 0, "split_torch_adam")
    # Degree 0: terms 1..15 have zero gradient, but their nonzero moments decay.
    changed = first[:, 3:] != fixture["first"][:, 3:]
    nonzero = fixture["first"][:, 3:] != 0
    assert np.array_equal(changed, nonzero)


def test_direct_and_snapshot_reads_agree(fixture):
    """A snapshot equal to dc/rest gives bit-identical results."""
    a = oracle.run_fixture_mode(fixture, 3, "split_torch_adam", snapshot=True)
    b = oracle.run_fixture_mode(fixture, 3, "split_torch_adam", snapshot=False)
    for x, y in zip(a, b):
        assert np.array_equal(x, y)


def test_quaternion_oracle_against_finite_differences():
    """Quaternion VJP vs central differences of normalize(q).seed, the check of
    the reference's check.py:72-85 (rtol 2e-5, atol 2e-6)."""
    rng = np.random.default_rng(42)
    q = (rng.standard_normal((35, 4)) + 0.2).astype(np.float32)
    seed = rng.standard_normal((35, 4)).astype(np.float32)
    norms = np.linalg.norm(q.astype(np.float64), axis=1, keepdims=True).astype(np.float32)
    got = oracle.quaternion_backward(q, seed, norms).astype(np.float64)
    qd, sd = q.astype(np.float64), seed.astype(np.float64)
    fd = np.empty_like(got)
    for j in range(4):
        plus, minus = qd.copy(), qd.copy()
        plus[:, j] += 1e-5
        minus[:, j] -= 1e-5
        f = lambda x: ((x / np.linalg.norm(x, axis=1, keepdims=True)) * sd).sum(1)
        fd[:, j] = (f(plus) - f(minus)) / 2e-5
    np.testing.assert_allclose(got, fd, rtol=2e-5, atol=2e-6)


def test_quaternion_clamp_branch():
    """Saved norm below 1e-12 selects seed / 1e-12 (normalization.cu:25-27)."""
    q = np.zeros((3, 4), np.float32)
    q[:, 0] = [np.nextafter(np.float32(1e-12), np.float32(0)), np.float32(1e-12),
               np.nextafter(np.float32(1e-12), np.float32(1))]
    seed = np.ones_like(q)
    norms = np.abs(q[:, :1]).copy()
    out = oracle.quaternion_backward(q, seed, norms)
    assert np.array_equal(out[0], seed[0] / np.float32(1e-12))
    assert np.isfinite(out).all()
    assert not np.array_equal(out[1], seed[1] / np.float32(1e-12))


def test_activation_oracle_against_closed_form_adam():
    """Scale/opacity VJPs and torch-style Adam vs a float64 restatement."""
    rng = np.random.default_rng(7)
    n = 257
    raw = [rng.standard_normal((n, 4)).astype(np.float32),
           rng.uniform(-6, -2, (n, 3)).astype(np.float32),
           rng.normal(-2, 1, (n, 1)).astype(np.float32)]
    seeds = [(rng.standard_normal(r.shape) * 1e-3).astype(np.float32) for r in raw]
    saved = [np.linalg.norm(raw[0], axis=1).astype(np.float32),
             np.exp(raw[1]).astype(np.float32),
             (1 / (1 + np.exp(-raw[2].astype(np.float64)))).astype(np.float32).reshape(n)]
    first = [(rng.standard_normal(r.shape) * 0.02).astype(np.float32) for r in raw]
    second = [(rng.random(r.shape) * 0.03).astype(np.float32) for r in raw]
    counters = [99, 102, 106]
    rates = [0.001, 0.005, 0.025]
    bias1 = [float(np.float32(1 - 0.9 ** (c + 1))) for c in counters]
    bias2 = [float(np.float32(np.sqrt(1 - 0.999 ** (c + 1)))) for c in counters]
    params = [r.copy() for r in raw]
    m = [f.copy() for f in first]
    v = [s.copy() for s in second]
    oracle.activation_consume(params, seeds, saved, m, v, rates, bias1, bias2)
    g_scale = saved[1].astype(np.float64) * seeds[1]
    a = saved[2].astype(np.float64).reshape(n, 1)
    g_opacity = a * (1 - a) * seeds[2]
    for k, g in ((1, g_scale), (2, g_opacity)):
        em = 0.9 * first[k] + 0.1 * g
        ev = 0.999 * second[k] + 0.001 * g * g
        ep = raw[k] - (rates[k] / bias1[k]) * em / (np.sqrt(ev) / bias2[k] + 1e-15)
        np.testing.assert_allclose(m[k], em, rtol=3e-6, atol=2e-9)
        np.testing.assert_allclose(v[k], ev, rtol=3e-6, atol=2e-11)
        np.testing.assert_allclose(params[k], ep, rtol=3e-6, atol=2e-7)
