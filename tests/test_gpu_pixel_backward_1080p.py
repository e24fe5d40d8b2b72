"""Pixel backward at the pixel-backward configuration (1920x1080, 16x16 tiles,
3,000,000 depth-sorted 2D Gaussians, radii lognormal(1.5, 0.7) px, opacity
U(0.05, 0.99), dL/dpixel N(0, 1e-3)) against the double-precision oracle on
a seeded sample of 64 whole tiles.

The CUDA pass runs over the full image with dL/dpixel kept on the sampled
tiles only (zero elsewhere: a pixel with a zero adjoint adds exactly zero to
every Gaussian), so each Gaussian's adjoints are the sums over the sampled
tiles' pixels, which the oracle computes with its own tile lists (3-sigma
rectangles, depth order) and stored transmittances. Compared elementwise
with |got - ref| <= 1e-4 |ref| + 3e-5 x (sum of |terms| of that element),
the floor being the float error of a sum relative to the size of its terms
(see test_gpu_rasterizer.py). A contribution decision within rounding of its
threshold can go either way in float: where a transmittance stop lies
within 1e-4 of 1e-4, the oracle adds to each affected Gaussian's tolerance
the most that decision can change (its allow_* arrays); Gaussians with an
alpha within rounding of 1/255 or an exponent within rounding of 0 are left
out, and their count is bounded (0.5% of those compared). Every Gaussian outside the
sampled tiles must come out exactly zero. All three accumulation modes are
checked, and the sampled pixels' colours match within 1e-5.
"""

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

W, H, P = 1920, 1080, 3_000_000
TILES = 64
FLOOR = 3e-5


@pytest.fixture(scope="module")
def scene_1080p(cuda):
    import rasterizer
    from bench import make_2d_scene

    scene = make_2d_scene(P, W, H, cuda, seed=4)
    bg = torch.tensor([0.1, 0.2, 0.3], device=cuda)
    num, color, _, state = rasterizer.forward_2d(
        scene["mean2d"], scene["conic_opacity"], scene["rgb"], scene["depth"],
        scene["radii"], W, H, bg)
    gx, gy = (W + 15) // 16, (H + 15) // 16
    tiles = np.sort(np.random.default_rng(11).choice(gx * gy, TILES, replace=False))
    dpix = (np.random.default_rng(5).standard_normal((3, H, W)) * 1e-3).astype(np.float32)
    mask = np.zeros((H, W), bool)
    for t in tiles:
        ty, tx = divmod(int(t), gx)
        mask[ty * 16:(ty + 1) * 16, tx * 16:(tx + 1) * 16] = True
    dpix[:, ~mask] = 0.0
    host = {k: v.cpu().numpy() for k, v in scene.items()}
    ref = oracle.pixel_tiles(host["mean2d"], host["conic_opacity"], host["rgb"],
                             host["depth"], host["radii"], W, H, bg.cpu().numpy(), tiles,
                             dpix.astype(np.float64))
    return dict(state=state, num=num, color=color.cpu().numpy(), mask=mask, tiles=tiles,
                dpix=torch.from_numpy(dpix).to(cuda), ref=ref)


def _run(s, mode, cuda):
    import rasterizer

    z = lambda *shape: torch.zeros(shape, device=cuda)
    grads = dict(dmean2d=z(P, 3), dconic=z(P, 4), dopacity=z(P), dcolor=z(P, 3))
    rasterizer.render_backward_2d(s["state"], s["dpix"], grads, mode)
    torch.cuda.synchronize()
    return {k: v.cpu().numpy().astype(np.float64) for k, v in grads.items()}


def test_sampled_tiles_forward_matches(scene_1080p):
    s = scene_1080p
    assert s["num"] > 20_000_000  # ~26M footprint-culled instances at this size
    got = s["color"][:, s["mask"]]
    want = s["ref"]["color"][:, s["mask"]]
    assert np.abs(got - want).max() < 1e-5


@pytest.mark.parametrize("mode", [2, 1, 0])
def test_sampled_tiles_adjoints_match_oracle(cuda, scene_1080p, mode):
    s = scene_1080p
    ref = s["ref"]
    got = _run(s, mode, cuda)
    touched = ((ref["mag_opacity"] > 0) | (ref["mag_color"].sum(1) > 0))
    ambiguous = ref["ambiguous"].astype(bool)
    compared = touched & ~ambiguous
    assert compared.sum() > 5_000, int(compared.sum())
    assert ambiguous.sum() <= 0.005 * touched.sum(), (int(ambiguous.sum()), int(touched.sum()))
    pairs = (
        ("dmean2d", got["dmean2d"][:, :2], "dmean2d", "mean2d"),
        ("dconic", got["dconic"][:, [0, 1, 3]], "dconic", "conic"),
        ("dopacity", got["dopacity"], "dopacity", "opacity"),
        ("dcolor", got["dcolor"], "dcolor", "color"),
    )
    for name, g, key, part in pairs:
        g, r = g[compared], ref[key][compared]
        m, a = ref["mag_" + part][compared], ref["allow_" + part][compared]
        tol = 1e-4 * np.abs(r) + FLOOR * m + a
        err = np.abs(g - r)
        bad = err > tol
        print(f"mode {mode} {name}: {g.size} compared, worst error/tolerance "
              f"{float((err / tol).max()):.3f}, worst relative "
              f"{float((err / np.maximum(np.abs(r), 1e-30)).max()):.2e}")
        assert not bad.any(), (name, int(bad.sum()), g[bad][:4], r[bad][:4],
                               float((err / tol).max()))
    # Nothing reaches a Gaussian the sampled tiles do not hold.
    untouched = ~touched & ~ambiguous
    for name in ("dmean2d", "dconic", "dopacity", "dcolor"):
        assert not np.any(got[name][untouched]), name
