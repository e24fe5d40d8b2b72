"""Pins the rasterizer oracle: its analytic backward against central finite
differences of its own forward loss sum(dL/dpix * colour) + sum(dL/dinvdepth *
inverse depth), in double precision, for every input the renderer
differentiates (means, scales, rotations, opacities, SH coefficients), with and
without the antialiasing opacity compensation.

The renderer the reference patches is not vendored (parity with it is
unpinned); this fixes the oracle to the mathematics the renderer implements.
"""

import numpy as np
import pytest

import oracle

FIELDS = [("means", "dmeans"), ("scales", "dscales"), ("rotations", "drots"),
          ("opacities", "dopacity"), ("sh", "dsh")]


@pytest.mark.parametrize("antialiasing", [False, True])
@pytest.mark.parametrize("degree", [0, 3])
def test_raster_oracle_gradients_match_finite_differences(antialiasing, degree):
    scene = oracle.raster_scene(6, 24, 40, seed=3 + degree, degree=degree,
                                antialiasing=antialiasing, scale=(0.04, 0.1))
    rng = np.random.default_rng(11)
    dpix = rng.standard_normal((3, 24, 40))
    dinv = rng.standard_normal((24, 40)) * 0.1
    grads = oracle.raster_backward(scene, dpix, dinv)
    h = 1e-6
    checked = 0
    for field, gkey in FIELDS:
        base = np.array(scene[field], dtype=np.float64)
        flat = base.reshape(-1)
        n = flat.size if field != "sh" else 3 * (degree + 1) ** 2 * 6
        idx = range(flat.size) if field != "sh" else [
            48 * i + k for i in range(6) for k in range(3 * (degree + 1) ** 2)]
        for k in list(idx)[:n]:
            plus, minus = flat.copy(), flat.copy()
            plus[k] += h
            minus[k] -= h
            lp = oracle.raster_loss({**scene, field: plus.reshape(base.shape)}, dpix, dinv)
            lm = oracle.raster_loss({**scene, field: minus.reshape(base.shape)}, dpix, dinv)
            fd = (lp - lm) / (2 * h)
            got = grads[gkey].reshape(-1)[k]
            assert abs(got - fd) <= 2e-5 + 1e-4 * abs(fd), (field, k, got, fd)
            checked += 1
    assert checked >= 84


def test_raster_oracle_empty_scene_is_background():
    scene = oracle.raster_scene(3, 17, 31, seed=1)
    scene["means"] = scene["means"] * 0 - 5.0  # behind the camera: culled
    color, inv, radii = oracle.raster_forward(scene)
    assert (radii == 0).all()
    for ch in range(3):
        assert np.allclose(color[ch], scene["bg"][ch])
    assert np.allclose(inv, 0)


def test_geometry_map_reproduces_the_backward():
    """The per-Gaussian geometry map (used to carry the pixel stage's
    tolerance to the geometry adjoints) applied to the pixel-stage adjoints
    gives the oracle's full backward."""
    scene = oracle.raster_scene(120, 40, 56, seed=9, antialiasing=True)
    rng = np.random.default_rng(4)
    dpix = rng.standard_normal((3, 40, 56)) * 0.1
    dinv = rng.standard_normal((40, 56)) * 0.01
    full = oracle.raster_backward(scene, dpix, dinv)
    sized = oracle.raster_backward_sized(scene, dpix, dinv)
    np.testing.assert_allclose(sized["x_mean2d"], full["dmean2d"], rtol=1e-12, atol=1e-15)
    np.testing.assert_allclose(sized["x_color"], full["dcolor"], rtol=1e-12, atol=1e-15)
    y = np.einsum("prk,pk->pr", sized["jac"], oracle.geometry_inputs(sized))
    for name, rows in oracle.GEOMETRY_ROWS.items():
        ref = full[name].reshape(len(y), -1)
        np.testing.assert_allclose(y[:, rows], ref, rtol=1e-9, atol=1e-12 * np.abs(ref).max())
    sizes = oracle.geometry_input_sizes(sized)
    x = oracle.geometry_inputs(sized)
    assert (sizes >= np.abs(x) * (1 - 1e-12)).all()
