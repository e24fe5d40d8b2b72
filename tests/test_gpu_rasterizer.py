"""CUDA rasterizer vs the double-precision oracle, warp-accumulation modes vs
each other, and the consumed SH backward vs native SH gradients + torch fused
Adam.

Tolerances. Forward colours within 1e-5 absolute. Backward adjoints
elementwise: |got - ref| <= 1e-4 |ref| + floor, where the floor follows each
adjoint's conditioning instead of the tensor's scale:

* pixel stage (dL/dmean2D, dL/dcolors, and inside the map below dL/dconic,
  the blended opacity's and inverse depth's adjoints): floor = 3e-5 x the sum
  of the absolute values of the terms summed into that element (the oracle
  reports it). A float sum of n terms is off by at most about n eps times
  that size; the walk's sums have up to a few hundred terms (eps = 6e-8);
* geometry stage (dL/dopacity, dL/dmeans3D, dL/dcov3D, dL/dsh, dL/dscales,
  dL/drotations): each Gaussian's outputs are a linear map J of its
  pixel-stage adjoints x (the oracle gives J); the pixel-stage tolerance is
  carried through |J|, plus, for the float evaluation of the map itself, 10x
  the spread of the oracle's map when all its inputs are perturbed by 4 float
  ulps (a float evaluation acts like an exact one at inputs a few ulps away;
  this covers outputs that are small or exactly zero by cancellation, such as
  the rotation adjoint of an isotropic Gaussian).

The three pixel-accumulation modes agree within the reference's own
warp-vs-native tolerance (check.py:815, rtol 5e-5, atol 2e-6) with
bit-identical forwards.
"""

import math

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def _t(a, device, dtype=torch.float32):
    return torch.as_tensor(np.ascontiguousarray(a), dtype=dtype, device=device)


def _render(scene, device, mode=2, dpix=None, dinv=None):
    import rasterizer

    rasterizer.pixel_accumulation = mode
    P, H, W = scene["P"], scene["H"], scene["W"]
    args = dict(
        bg=_t(scene["bg"], device), means=_t(scene["means"], device).reshape(P, 3),
        opacity=_t(scene["opacities"], device).reshape(P, 1),
        scales=_t(scene["scales"], device).reshape(P, 3),
        rotations=_t(scene["rotations"], device).reshape(P, 4),
        view=_t(scene["view"], device), proj=_t(scene["proj"], device),
        sh=_t(scene["sh"], device).reshape(P, 16, 3), campos=_t(scene["campos"], device))
    empty = torch.empty(0, device=device)
    out = rasterizer.rasterize_gaussians(
        args["bg"], args["means"], empty, args["opacity"], args["scales"], args["rotations"],
        scene["scale_modifier"], empty, args["view"], args["proj"], scene["tanx"],
        scene["tany"], H, W, args["sh"], scene["degree"], args["campos"], False,
        scene["antialiasing"], False)
    num, color, radii, geom, binning, image, invdepth = out
    grads = None
    if dpix is not None:
        grads = rasterizer.rasterize_gaussians_backward(
            args["bg"], args["means"], radii, empty, args["opacity"], args["scales"],
            args["rotations"], scene["scale_modifier"], empty, args["view"], args["proj"],
            scene["tanx"], scene["tany"], _t(dpix, device), _t(dinv, device).reshape(1, H, W),
            args["sh"], scene["degree"], args["campos"], geom, num, binning, image,
            scene["antialiasing"], False)
    torch.cuda.synchronize()
    return num, color, radii, invdepth, grads


PIXEL_SIZE_FLOOR = 3e-5
SPREAD_MARGIN = 10.0


def _bounded(got, ref, tol, what):
    got = np.asarray(got, np.float64).reshape(ref.shape)
    err = np.abs(got - ref)
    bad = err > tol
    worst = float((err / np.maximum(tol, 1e-300)).max()) if err.size else 0.0
    assert not bad.any(), (what, int(bad.sum()), got[bad][:4], ref[bad][:4], worst)
    return worst


def check_backward(grads, scene, dpix, dinv, label=""):
    """All eight outputs of rasterize_gaussians_backward against the oracle,
    with the conditioning-aware tolerance of the module docstring. Returns the
    worst |error| / tolerance seen."""
    P = scene["P"]
    sized = oracle.raster_backward_sized(scene, dpix, dinv)
    g2d, gcol, gop, gmean, gcov, gsh, gscale, grot = [g.cpu().numpy() for g in grads]
    worst = 0.0
    for got, key in ((g2d[:, :2], "mean2d"), (gcol, "color")):
        want = sized["x_" + key][:, :got.shape[1]]
        size = sized["size_" + key][:, :got.shape[1]]
        worst = max(worst, _bounded(got, want, 1e-4 * np.abs(want) + PIXEL_SIZE_FLOOR * size,
                                    f"{label}dL/d{key}"))
    x = oracle.geometry_inputs(sized)
    tol_x = 1e-4 * np.abs(x) + PIXEL_SIZE_FLOOR * oracle.geometry_input_sizes(sized)
    J = sized["jac"]
    y = np.einsum("prk,pk->pr", J, x)
    tol_y = (1e-4 * np.abs(y) + np.einsum("prk,pk->pr", np.abs(J), tol_x)
             + SPREAD_MARGIN * oracle.geometry_spread(scene, x))
    for name, got in (("dopacity", gop), ("dmeans", gmean), ("dcov3d", gcov), ("dsh", gsh),
                      ("dscales", gscale), ("drots", grot)):
        rows = oracle.GEOMETRY_ROWS[name]
        worst = max(worst, _bounded(got.reshape(P, -1), y[:, rows], tol_y[:, rows],
                                    f"{label}{name}"))
    return worst


@pytest.mark.parametrize("antialiasing", [False, True])
@pytest.mark.parametrize("degree", [0, 3])
@pytest.mark.parametrize("P,H,W", [(40, 48, 64), (300, 97, 131)])
def test_rasterizer_matches_oracle(cuda, P, H, W, degree, antialiasing):
    scene = oracle.raster_scene(P, H, W, seed=P + degree, degree=degree,
                                antialiasing=antialiasing)
    rng = np.random.default_rng(2)
    dpix = rng.standard_normal((3, H, W)) * 0.1
    dinv = rng.standard_normal((H, W)) * 0.01
    num, color, radii, invdepth, grads = _render(scene, cuda, 2, dpix, dinv)
    ocolor, oinv, oradii = oracle.raster_forward(scene)
    assert np.array_equal(radii.cpu().numpy(), oradii)
    assert np.abs(color.cpu().numpy() - ocolor).max() < 1e-5
    assert np.abs(invdepth.cpu().numpy()[0] - oinv).max() < 1e-5 * max(1.0, np.abs(oinv).max())
    check_backward(grads, scene, dpix, dinv)


def _rectangle_tiles(scene, radii):
    """Tile instances of the renderer's 3-sigma rectangles."""
    P, H, W = scene["P"], scene["H"], scene["W"]
    hom = np.concatenate([scene["means"], np.ones((P, 1))], 1) @ scene["proj"]
    px = ((hom[:, 0] / (hom[:, 3] + 1e-7) + 1) * W - 1) * 0.5
    py = ((hom[:, 1] / (hom[:, 3] + 1e-7) + 1) * H - 1) * 0.5
    gx, gy = (W + 15) // 16, (H + 15) // 16
    total = 0
    for x, y, r in zip(px, py, radii):
        if r <= 0:
            continue
        x0 = min(gx, max(0, int((x - r) / 16)))
        y0 = min(gy, max(0, int((y - r) / 16)))
        x1 = min(gx, max(0, int((x + r + 15) / 16)))
        y1 = min(gy, max(0, int((y + r + 15) / 16)))
        total += (x1 - x0) * (y1 - y0)
    return total


@pytest.mark.parametrize("antialiasing", [False, True])
def test_footprint_culling_keeps_every_contribution(cuda, antialiasing):
    """Needle-like, low- and high-opacity Gaussians: the instance lists hold
    only tiles the alpha >= 1/255 ellipse reaches, and every output still
    matches the oracle, which composites every Gaussian in its 3-sigma
    rectangle."""
    P, H, W = 400, 90, 150
    scene = oracle.raster_scene(P, H, W, seed=77, antialiasing=antialiasing,
                                scale=(0.004, 0.25))
    rng = np.random.default_rng(8)
    scene["opacities"] = np.concatenate([rng.uniform(0.002, 0.02, P // 2),
                                         rng.uniform(0.5, 0.999, P - P // 2)])
    dpix = rng.standard_normal((3, H, W)) * 0.1
    dinv = rng.standard_normal((H, W)) * 0.01
    num, color, radii, invdepth, grads = _render(scene, cuda, 2, dpix, dinv)
    ocolor, oinv, oradii = oracle.raster_forward(scene)
    assert np.array_equal(radii.cpu().numpy(), oradii)
    # The 3-sigma rectangles would hold far more instances than the footprints.
    assert 0 < num < 0.7 * _rectangle_tiles(scene, oradii)
    assert np.abs(color.cpu().numpy() - ocolor).max() < 1e-5
    assert np.abs(invdepth.cpu().numpy()[0] - oinv).max() < 1e-5 * max(1.0, np.abs(oinv).max())
    check_backward(grads, scene, dpix, dinv)


def _reference_fixture(name, n, H, W, scale, opacity, antialiasing):
    """The reference's raster fixtures (check.py:745-767), restated."""
    torch.manual_seed(42)
    means = (torch.randn(n, 3) * .08)
    means[:, 2] = torch.linspace(2., 3., n)
    sh = torch.randn(n, 16, 3) * .02
    proj = torch.tensor([[1., 0, 0, 0], [0, 1., 0, 0], [0, 0, 100 / 99.99, -1 / 99.99],
                         [0, 0, 1., 0]]).T.contiguous()
    rotations = torch.zeros(n, 4)
    rotations[:, 0] = 1
    return dict(P=n, degree=3, bg=np.array([.1, .2, .3]), means=means.numpy(),
                opacities=np.full(n, opacity), scales=np.full((n, 3), scale),
                scale_modifier=1.0, rotations=rotations.numpy(), view=np.eye(4),
                proj=proj.numpy(), tanx=1.0, tany=1.0, H=H, W=W,
                sh=sh.reshape(n, 48).numpy(), campos=np.zeros(3), antialiasing=antialiasing)


FIXTURES = [("full-warp", 1, 32, 32, 2., .3), ("partial-tiles", 17, 17, 31, .2, .5),
            ("occluded", 73, 32, 32, .8, .95), ("empty", 0, 17, 31, .2, .5)]


@pytest.mark.parametrize("antialiasing", [False, True])
@pytest.mark.parametrize("fixture", FIXTURES, ids=[f[0] for f in FIXTURES])
def test_accumulation_modes_agree_on_reference_fixtures(cuda, fixture, antialiasing):
    name, n, H, W, scale, opacity = fixture
    scene = _reference_fixture(name, n, H, W, scale, opacity, antialiasing)
    torch.manual_seed(7)
    dpix = (torch.randn(3, H, W) * .01).numpy()
    dinv = (torch.randn(H, W) * .01).numpy()
    runs = [_render(scene, cuda, mode, dpix, dinv) for mode in (0, 1, 2)]
    if name == "full-warp":
        assert (runs[0][3] > 0).all(), "the full-warp fixture must cover every pixel"
    base = runs[0]
    for other in runs[1:]:
        assert torch.equal(other[1], base[1]) and torch.equal(other[2], base[2])
        assert torch.equal(other[3], base[3])
        for g, b in zip(other[4], base[4]):
            assert torch.isfinite(g).all()
            torch.testing.assert_close(g, b, rtol=5e-5, atol=2e-6)
    if n:
        for run in runs:
            check_backward(run[4], scene, dpix, dinv, f"{name}: ")


@pytest.mark.parametrize("degree", [0, 1, 2, 3])
@pytest.mark.parametrize("step", [1, 100])
@pytest.mark.parametrize("direct", [False, True])
def test_consumed_backward_matches_native_plus_fused_adam(cuda, degree, step, direct):
    """check.py:980-1017: consume path vs native SH grads + torch fused Adam."""
    import rasterizer

    scene = oracle.raster_scene(64, 40, 56, seed=9 + degree, degree=degree)
    P, H, W = 64, 40, 56
    dev = cuda
    empty = torch.empty(0, device=dev)
    means = _t(scene["means"], dev)
    opacity = _t(scene["opacities"], dev).reshape(P, 1)
    scales, rots = _t(scene["scales"], dev), _t(scene["rotations"], dev)
    view, proj = _t(scene["view"], dev), _t(scene["proj"], dev)
    campos, bg = _t(scene["campos"], dev), _t(scene["bg"], dev)
    coeffs = _t(scene["sh"], dev).reshape(P, 16, 3)
    num, color, radii, geom, binning, image, inv = rasterizer.rasterize_gaussians(
        bg, means, empty, opacity, scales, rots, 1.0, empty, view, proj, scene["tanx"],
        scene["tany"], H, W, coeffs, degree, campos, False, False, False)
    torch.manual_seed(3)
    seed = torch.randn(3, H, W, device=dev) * 0.1
    dseed = torch.zeros(1, H, W, device=dev)
    common = (bg, means, radii, empty, opacity, scales, rots, 1.0, empty, view, proj,
              scene["tanx"], scene["tany"], seed, dseed)
    native = rasterizer.rasterize_gaussians_backward(*common, coeffs, degree, campos, geom,
                                                     num, binning, image, False, False)
    dc = coeffs[:, :1].contiguous().clone()
    rest = coeffs[:, 1:].contiguous().clone()
    fills = (0.002, 0.01, -0.003, 0.02) if step > 1 else (0.,) * 4
    moments = [torch.full_like(v, f) for v, f in zip((dc, dc, rest, rest), fills)]
    b1, b2 = 1 - 0.9 ** step, math.sqrt(1 - 0.999 ** step)
    if direct:
        consumed = rasterizer.rasterize_gaussians_backward_consume_direct(
            *common, empty, degree, campos, geom, num, binning, image, False, False, dc, rest,
            *moments, b1, b2)
    else:
        consumed = rasterizer.rasterize_gaussians_backward_consume(
            *common, coeffs, degree, campos, geom, num, binning, image, False, False, dc, rest,
            *moments, b1, b2)
    params = [torch.nn.Parameter(coeffs[:, :1].contiguous().clone()),
              torch.nn.Parameter(coeffs[:, 1:].contiguous().clone())]
    opt = torch.optim.Adam([dict(params=[params[0]], lr=0.0025),
                            dict(params=[params[1]], lr=0.000125)], eps=1e-15, fused=True,
                           foreach=False)
    for p_, g_, m_, v_ in zip(params, (native[5][:, :1], native[5][:, 1:]), fills[::2],
                              fills[1::2]):
        opt.state[p_] = dict(step=torch.tensor(float(step - 1), device=dev),
                             exp_avg=torch.full_like(p_, m_), exp_avg_sq=torch.full_like(p_, v_))
        p_.grad = g_.contiguous()
    opt.step()
    expected = [params[0], params[1], opt.state[params[0]]["exp_avg"],
                opt.state[params[0]]["exp_avg_sq"], opt.state[params[1]]["exp_avg"],
                opt.state[params[1]]["exp_avg_sq"]]
    actual = [dc, rest, moments[0], moments[1], moments[2], moments[3]]
    torch.cuda.synchronize()
    for a, e in zip(actual, expected):
        torch.testing.assert_close(a, e.detach(), rtol=3e-5, atol=2e-7)
    assert consumed[5].numel() == 0
    for k in (0, 1, 2, 3, 4, 6, 7):
        torch.testing.assert_close(consumed[k], native[k], rtol=3e-5, atol=2e-7)


def test_atomic_count_pass_matches_a_replay(cuda):
    """The counting pass's contributing pairs equal a float replay of the
    walk's contribution test (same exponent rounding), and its per-mode counts
    are consistent: mode 1 between pairs / 32 and pairs, mode 2 at most the
    pairs and at least pairs / 128."""
    import rasterizer

    rng = np.random.default_rng(12)
    n, W, H = 300, 80, 48
    mean2d = (rng.random((n, 2)) * [W, H]).astype(np.float32)
    s1, s2 = np.exp(1.2 + 0.5 * rng.standard_normal(n)), np.exp(1.2 + 0.5 * rng.standard_normal(n))
    th = rng.random(n) * np.pi
    c, s = np.cos(th), np.sin(th)
    a, b = c * c * s1 * s1 + s * s * s2 * s2, c * s * (s1 * s1 - s2 * s2)
    d = s * s * s1 * s1 + c * c * s2 * s2
    det = a * d - b * b
    co = np.stack([d / det, -b / det, a / det, 0.05 + 0.94 * rng.random(n)], 1).astype(np.float32)
    radii = np.ceil(3 * np.maximum(s1, s2)).astype(np.int32)
    rgb, depth = rng.random((n, 3)).astype(np.float32), (1 + 9 * rng.random(n)).astype(np.float32)
    t = lambda x: torch.from_numpy(x).to(cuda)
    num, _, _, state = rasterizer.forward_2d(t(mean2d), t(co), t(rgb), t(depth), t(radii), W, H,
                                             torch.zeros(3, device=cuda))
    counts = rasterizer.count_accumulation_2d(state)
    # Float replay: every pixel walks all Gaussians in depth order (ties by
    # index), vectorised over the pixels; the exponent is rounded like the
    # kernels' (fused multiply-adds emulated in double, exact here).
    order = np.lexsort((np.arange(n), depth))
    ys, xs = np.mgrid[0:H, 0:W]
    px, py = xs.astype(np.float32).ravel(), ys.astype(np.float32).ravel()
    T = np.ones(px.size, np.float32)
    alive = np.ones(px.size, bool)
    pairs = 0
    f32 = np.float32
    for i in order:
        if radii[i] <= 0:
            continue
        dx, dy = (mean2d[i, 0] - px).astype(f32), (mean2d[i, 1] - py).astype(f32)
        c0 = (f32(-0.5) * ((co[i, 0] * dx).astype(f32) * dx).astype(f32)).astype(f32)
        c1 = -(co[i, 1] * dx).astype(f32)
        c2 = f32(-0.5) * co[i, 2]
        inner = (np.float64(c2) * dy.astype(np.float64) + c1.astype(np.float64)).astype(f32)
        p = (inner.astype(np.float64) * dy + c0.astype(np.float64)).astype(f32)
        alpha = np.minimum(f32(0.99), (co[i, 3] * np.exp(p.astype(np.float64)).astype(f32)).astype(f32))
        live = alive & (p <= 0) & (alpha >= f32(1 / 255))
        tt = (T * (f32(1) - alpha)).astype(f32)
        stop = live & (tt < f32(1e-4))
        alive &= ~stop
        take = live & ~stop
        pairs += int(take.sum())
        T = np.where(take, tt, T)
    # The kernels' fast exponential and the replay's exact one can decide a
    # pair within rounding of the 1/255 alpha floor or the 1e-4 stop the other
    # way (about 2 in 10,000 pairs here).
    assert abs(counts["pairs"] - pairs) <= max(2, pairs // 2000), (counts, pairs)
    assert pairs / 32 <= counts["mode1_per_field"] <= pairs
    assert pairs / 128 <= counts["mode2_reductions"] <= pairs
