"""SH consumer kernel (fused SH VJP + Adam) vs the CPU oracle, through the C ABI.

The kernels are compiled without FMA contraction and evaluate every operation
in the oracle's order, so every output (parameters, both moments, the position
adjoint) must be bit-identical to the oracle. Cases cover degrees 0-3, direct
and snapshot coefficient reads, tile tails, misaligned buffers (generic path),
invisible Gaussians, clamped channels, nonzero moments, multi-step runs, all
four reference update modes, the reference's own self-check fixture with its
tolerances, invalid degrees, empty launches, and the 1.1M-Gaussian size.
"""

import ctypes

import numpy as np
import pytest
import torch

import cases
import oracle

pytestmark = pytest.mark.gpu


def _dev(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def _misaligned(a, device):
    """A 4-byte-aligned but not 16-byte-aligned device copy of a."""
    flat = torch.empty(a.size + 1, dtype=torch.from_numpy(a[:0]).dtype, device=device)
    view = flat[1:].view(a.shape)
    view.copy_(torch.from_numpy(np.ascontiguousarray(a)))
    return view


def run_kernel(p, degree, step, device, *, snapshot=False, misaligned=False):
    import consume

    put = (lambda a: _misaligned(a, device)) if misaligned else (lambda a: _dev(a, device))
    t = {k: put(p[k]) for k in ("means", "radii", "seed") + cases.SH_KEYS}
    t["clamped"] = put(p["clamped"])
    t["camera"] = _dev(p["camera"], device)
    coefficient = None
    if snapshot:
        coefficient = put(np.concatenate([p["dc"], p["rest"]], 1))
    b1, b2 = cases.bias(step)
    consume.sh_consume_split_torch_adam(
        t["means"], t["radii"], t["clamped"], t["camera"], t["seed"], t["dm"], t["dc"],
        t["rest"], t["dc_first"], t["dc_second"], t["rest_first"], t["rest_second"],
        bias1=b1, bias2_sqrt=b2, degree=degree, coefficient=coefficient)
    torch.cuda.synchronize()
    return {k: t[k].cpu().numpy() for k in cases.SH_KEYS}


def run_oracle(p, degree, step, *, snapshot=False):
    out = {k: p[k].copy() for k in cases.SH_KEYS}
    b1, b2 = cases.bias(step)
    oracle.sh_consume(
        "split_torch_adam", degree, p["means"], p["radii"], p["clamped"], p["camera"],
        p["seed"], out["dm"],
        coefficient=np.concatenate([p["dc"], p["rest"]], 1) if snapshot else None,
        dc=out["dc"], rest=out["rest"], dc_first=out["dc_first"],
        dc_second=out["dc_second"], rest_first=out["rest_first"],
        rest_second=out["rest_second"], bias1=b1, bias2_sqrt=b2)
    return out


def assert_identical(got, want, what=""):
    for k in want:
        g, w = got[k], want[k]
        same = (g.view(np.uint32) == w.view(np.uint32)) | (np.isnan(g) & np.isnan(w))
        assert same.all(), (
            f"{what} {k}: {int((~same).sum())} of {same.size} differ; first at "
            f"{np.argwhere(~same)[0]}: got {g[~same][:3]} want {w[~same][:3]}")


@pytest.mark.parametrize("n", [1, 63, 64, 65, 257, 4097, 64 * 300 + 17])
@pytest.mark.parametrize("degree", [0, 1, 2, 3])
def test_split_torch_adam_bit_exact(cuda, n, degree):
    p = cases.sh_problem(n, seed=n + degree, moments=degree % 2 == 1)
    step = 1 if degree % 2 == 0 else 37
    assert_identical(run_kernel(p, degree, step, cuda), run_oracle(p, degree, step))


@pytest.mark.parametrize("n", [65, 4097])
def test_snapshot_reads_bit_exact(cuda, n):
    p = cases.sh_problem(n, seed=5, moments=True)
    got = run_kernel(p, 3, 12, cuda, snapshot=True)
    assert_identical(got, run_oracle(p, 3, 12, snapshot=True))
    # A snapshot equal to dc/rest gives the same bits as direct reads.
    assert_identical(got, run_kernel(p, 3, 12, cuda))


@pytest.mark.parametrize("n", [1, 64, 1000])
def test_misaligned_buffers_take_generic_path(cuda, n):
    p = cases.sh_problem(n, seed=11, moments=True)
    assert_identical(run_kernel(p, 3, 4, cuda, misaligned=True), run_oracle(p, 3, 4))


def test_consecutive_steps_carry_moments(cuda):
    import consume

    n = 3000
    p = cases.sh_problem(n, seed=3)
    t = {k: _dev(p[k], cuda) for k in ("means", "radii", "clamped", "seed", "camera")
         + cases.SH_KEYS}
    ref = {k: p[k].copy() for k in cases.SH_KEYS}
    for step in range(1, 31):
        b1, b2 = cases.bias(step)
        consume.sh_consume_split_torch_adam(
            t["means"], t["radii"], t["clamped"], t["camera"], t["seed"], t["dm"],
            t["dc"], t["rest"], t["dc_first"], t["dc_second"], t["rest_first"],
            t["rest_second"], bias1=b1, bias2_sqrt=b2, degree=3)
        oracle.sh_consume("split_torch_adam", 3, p["means"], p["radii"], p["clamped"],
                          p["camera"], p["seed"], ref["dm"], dc=ref["dc"],
                          rest=ref["rest"], dc_first=ref["dc_first"],
                          dc_second=ref["dc_second"], rest_first=ref["rest_first"],
                          rest_second=ref["rest_second"], bias1=b1, bias2_sqrt=b2)
    torch.cuda.synchronize()
    assert_identical({k: t[k].cpu().numpy() for k in cases.SH_KEYS}, ref, "30 steps")


@pytest.mark.parametrize("mode", ["sgd", "adam", "split_adam"])
@pytest.mark.parametrize("n", [65, 4097])
def test_reference_variants_bit_exact(cuda, mode, n):
    import consume

    p = cases.sh_problem(n, seed=17, moments=True)
    packed = lambda a, b: np.ascontiguousarray(np.concatenate([a, b], 1))
    inv1, inv2 = float(np.float32(1 / (1 - 0.9 ** 9))), float(np.float32(1 / (1 - 0.999 ** 9)))
    dev = {k: _dev(p[k], cuda) for k in ("means", "radii", "clamped", "seed", "camera", "dm")}
    ref_dm = p["dm"].copy()
    if mode == "split_adam":
        t = {k: _dev(p[k], cuda) for k in cases.SH_KEYS[1:]}
        consume.sh_consume_variant(mode, dev["means"], dev["radii"], dev["clamped"],
                                   dev["camera"], dev["seed"], dev["dm"], degree=3,
                                   inv_bias1=inv1, inv_bias2=inv2, dc=t["dc"],
                                   rest=t["rest"], dc_first=t["dc_first"],
                                   dc_second=t["dc_second"], rest_first=t["rest_first"],
                                   rest_second=t["rest_second"])
        ref = {k: p[k].copy() for k in cases.SH_KEYS[1:]}
        oracle.sh_consume(mode, 3, p["means"], p["radii"], p["clamped"], p["camera"],
                          p["seed"], ref_dm, dc=ref["dc"], rest=ref["rest"],
                          dc_first=ref["dc_first"], dc_second=ref["dc_second"],
                          rest_first=ref["rest_first"], rest_second=ref["rest_second"],
                          inv_bias1=inv1, inv_bias2=inv2)
    else:
        arrays = dict(coeff=packed(p["dc"], p["rest"]),
                      first=packed(p["dc_first"], p["rest_first"]),
                      second=packed(p["dc_second"], p["rest_second"]))
        t = {k: _dev(v, cuda) for k, v in arrays.items()}
        ref = {k: v.copy() for k, v in arrays.items()}
        adam = mode == "adam"
        consume.sh_consume_variant(mode, dev["means"], dev["radii"], dev["clamped"],
                                   dev["camera"], dev["seed"], dev["dm"], degree=3,
                                   inv_bias1=inv1, inv_bias2=inv2, coeff=t["coeff"],
                                   first=t["first"] if adam else None,
                                   second=t["second"] if adam else None)
        oracle.sh_consume(mode, 3, p["means"], p["radii"], p["clamped"], p["camera"],
                          p["seed"], ref_dm, coeff=ref["coeff"],
                          first=ref["first"] if adam else None,
                          second=ref["second"] if adam else None,
                          inv_bias1=inv1, inv_bias2=inv2)
    torch.cuda.synchronize()
    got = {k: v.cpu().numpy() for k, v in t.items()}
    got["dm"] = dev["dm"].cpu().numpy()
    ref["dm"] = ref_dm
    assert_identical(got, ref, mode)


@pytest.mark.parametrize("degree", [0, 1, 2, 3])
def test_reference_self_check_fixture_on_gpu(cuda, degree):
    """The reference's 257-Gaussian self-check (SHGradientConsumer.cu:436-608):
    product kernel vs finite differences + closed-form Adam, same tolerances."""
    import consume

    fx = oracle.reference_fixture()
    dc, rest = oracle.split(fx["coeff"])
    m_dc, m_rest = oracle.split(fx["first"])
    v_dc, v_rest = oracle.split(fx["second"])
    t = {k: _dev(v, cuda) for k, v in dict(
        means=fx["means"], radii=fx["radii"], clamped=fx["clamp"].astype(bool),
        camera=fx["camera"], seed=fx["seed"], dm=fx["initial"], dc=dc, rest=rest,
        m_dc=m_dc, v_dc=v_dc, m_rest=m_rest, v_rest=v_rest).items()}
    consume.sh_consume_split_torch_adam(
        t["means"], t["radii"], t["clamped"], t["camera"], t["seed"], t["dm"], t["dc"],
        t["rest"], t["m_dc"], t["v_dc"], t["m_rest"], t["v_rest"],
        bias1=fx["torch"][0], bias2_sqrt=fx["torch"][1], degree=degree,
        coefficient=_dev(fx["coeff"], cuda))
    torch.cuda.synchronize()
    e_dm, e_coeff, e_first, e_second = oracle.fixture_expectations(fx, degree,
                                                                   "split_torch_adam")
    join = lambda a, b: np.concatenate([a.cpu().numpy(), b.cpu().numpy()], 1)
    tol = oracle.FIXTURE_TOLERANCES
    for got, want, key in ((t["dm"].cpu().numpy(), e_dm, "dm"),
                           (join(t["dc"], t["rest"]), e_coeff, "coeff"),
                           (join(t["m_dc"], t["m_rest"]), e_first, "first"),
                           (join(t["v_dc"], t["v_rest"]), e_second, "second")):
        atol, rtol = tol[key]
        assert np.isfinite(got).all()
        assert (np.abs(got - want) <= atol + rtol * np.abs(want)).all(), key


def test_invalid_degree_rejected_without_writes(cuda):
    import _native as native

    p = cases.sh_problem(100, seed=1)
    t = {k: _dev(p[k], cuda) for k in ("means", "radii", "clamped", "seed", "camera")
         + cases.SH_KEYS}
    before = {k: t[k].clone() for k in cases.SH_KEYS}
    lib = native.library()
    status = lib.clad3dgs_sh_consume_split_torch_adam(
        100, 4, *[t[k].data_ptr() for k in ("means", "radii")], None,
        t["clamped"].data_ptr(), t["camera"].data_ptr(), t["seed"].data_ptr(),
        *[t[k].data_ptr() for k in cases.SH_KEYS], native.TorchAdamConfig(0.1, 0.03), 0)
    assert status == native.INVALID_ARGUMENT
    assert b"degree" in lib.clad3dgs_last_error()
    torch.cuda.synchronize()
    for k in cases.SH_KEYS:
        assert torch.equal(t[k], before[k])
    # Empty launches are no-ops, even with null pointers (SHGradientConsumer.cu:468-478).
    lib.sh_consumer_split_torch_adam(0, 0, *([None] * 13), native.TorchAdamConfig(1, 1))
    lib.sh_consumer_sgd(0, 7, *([None] * 7))
    assert lib.clad3dgs_sh_consume_split_torch_adam(
        0, 9, *([None] * 13), native.TorchAdamConfig(1, 1), 0) == native.OK
    torch.cuda.synchronize()
    assert native.fault_status() == 0


def test_full_size_bit_exact(cuda):
    """1.1M Gaussians (the fused-step benchmark size) against the oracle."""
    n = 1_100_000
    p = cases.sh_problem(n, seed=42, moments=True)
    assert_identical(run_kernel(p, 3, 7, cuda), run_oracle(p, 3, 7), "1.1M")
    import _native as native
    assert native.fault_status() == 0


def test_adam_ratio_threshold_bit_exact(cuda):
    """sqrt(v)/bias2 swept densely across 2^-25, where the kernel skips the
    double-precision epsilon add that cannot change the float result; zero
    gradients (invisible Gaussians) keep v under control."""
    n = 8192
    p = cases.sh_problem(n, seed=99, invisible=1.0, moments=True)
    b1, b2 = cases.bias(3)
    rng = np.random.default_rng(5)
    # v_new = 0.999 v; pick v so sqrt(v_new)/b2 covers [2^-27, 2^-23].
    exponent = rng.uniform(-27.0, -23.0, (n, 45))
    ratio = np.exp2(exponent)
    v = ((ratio * b2) ** 2 / 0.999).astype(np.float32)
    # also hit exact float neighbours of the threshold
    edge = np.float32(2.0 ** -25)
    around = np.array([np.nextafter(edge, np.float32(0)), edge, np.nextafter(edge, np.float32(1))],
                      np.float32)
    v[:3, :3] = ((around.astype(np.float64)[None, :] * b2) ** 2 / 0.999).astype(np.float32)
    p["rest_second"] = v
    p["dc_second"] = v[:, :3].copy()
    assert_identical(run_kernel(p, 3, 3, cuda), run_oracle(p, 3, 3), "ratio sweep")
