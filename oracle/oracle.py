"""CPU oracle of the per-Gaussian backward-and-update path (numpy + ctypes).

TEST INFRASTRUCTURE ONLY: tests/, the smoke check and bench.py's CPU-baseline
leg import this module as the checker. The product never imports it.

The arithmetic lives in oracle.c (see its header for the reference file:line
each function restates). This module builds liboracle.so on first use, wraps
it for numpy arrays, and restates the reference's deterministic 257-Gaussian
self-check fixture (SHGradientConsumer.cu:436-467) and its expectations
(SHGradientConsumer.cu:498-608).
"""

from __future__ import annotations

import ctypes
import math
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIBRARY = HERE / "liboracle.so"

_f32 = np.float32
_lib = None


def build() -> Path:
    """Builds liboracle.so (and the reference controls when mounted)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIBRARY


def lib():
    global _lib
    if _lib is None:
        sources = [HERE / "oracle.c", HERE / "raster_oracle.c"]
        newest = max(s.stat().st_mtime for s in sources if s.exists())
        if not LIBRARY.exists() or LIBRARY.stat().st_mtime < newest:
            subprocess.run(["make", "-s", "-C", str(HERE), "liboracle.so"], check=True)
        _lib = ctypes.CDLL(str(LIBRARY))
    return _lib


def _p(a):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


def _ptrs(arrays):
    return (ctypes.c_void_p * len(arrays))(*[a.ctypes.data for a in arrays])


MODES = {"sgd": 0, "adam": 1, "split_adam": 2, "split_torch_adam": 3}


def sh_consume(mode, degree, means, radii, clamped, camera, seed, dm, *,
               coefficient=None, coeff=None, first=None, second=None, dc=None,
               rest=None, dc_first=None, dc_second=None, rest_first=None,
               rest_second=None, bias1=1.0, bias2_sqrt=1.0, inv_bias1=1.0,
               inv_bias2=1.0):
    """SH VJP + update in place on numpy float32 arrays (reference layouts)."""
    n = int(radii.shape[0])
    lib().oracle_sh_consume(
        ctypes.c_int(MODES[mode]), ctypes.c_int64(n), ctypes.c_int(degree),
        _p(means), _p(radii), _p(clamped.view(np.uint8)), _p(camera), _p(seed),
        _p(dm), _p(coefficient), _p(coeff), _p(first), _p(second), _p(dc),
        _p(rest), _p(dc_first), _p(dc_second), _p(rest_first), _p(rest_second),
        ctypes.c_float(bias1), ctypes.c_float(bias2_sqrt),
        ctypes.c_float(inv_bias1), ctypes.c_float(inv_bias2))


def quaternion_backward(q, seed, norms):
    out = np.empty_like(q)
    lib().oracle_quaternion_backward(ctypes.c_int64(q.shape[0]), _p(q), _p(seed),
                                     _p(norms), _p(out))
    return out


def activation_consume(params, seeds, saved, first, second, rates, bias1, bias2):
    """Activation VJPs + torch-fused Adam in place (rotation, scaling, opacity)."""
    n = int(params[0].shape[0])
    for group in (params, seeds, saved, first, second):
        for a in group:
            assert a.flags["C_CONTIGUOUS"] and a.dtype == _f32
    lib().oracle_activation_consume(
        ctypes.c_int64(n), _ptrs(params), _ptrs(seeds), _ptrs(saved),
        _ptrs(first), _ptrs(second),
        (ctypes.c_double * 3)(*[float(r) for r in rates]),
        (ctypes.c_float * 3)(*[float(b) for b in bias1]),
        (ctypes.c_float * 3)(*[float(b) for b in bias2]))


def xyz_adam(means, dm, first, second, rate, bias1, bias2):
    """Torch-fused Adam on positions in place (float32 numpy arrays)."""
    lib().oracle_xyz_adam(ctypes.c_int64(means.shape[0]), _p(means), _p(dm), _p(first),
                          _p(second), ctypes.c_double(rate), ctypes.c_float(bias1),
                          ctypes.c_float(bias2))


SHARD_WIDTHS = (3, 48, 3, 4, 1)  # xyz, sh, scaling, rotation, opacity


def shard_update(begin, end, grad_origin, grads, params, first, second, saved_scaling,
                 saved_opacity, saved_norm, rates, bias1, bias2):
    """Exchange + update in place: grads[q][g] (rank q, group g), params[g],
    first/second[g] of the share [begin, end), float32 numpy arrays."""
    flat = [grads[q][g] for q in range(len(grads)) for g in range(5)]
    lib().oracle_shard_update(
        ctypes.c_int64(begin), ctypes.c_int64(end), ctypes.c_int64(grad_origin),
        ctypes.c_int(len(grads)), _ptrs(flat), _ptrs(params), _ptrs(first), _ptrs(second),
        _p(saved_scaling), _p(saved_opacity), _p(saved_norm),
        (ctypes.c_double * 6)(*rates), ctypes.c_float(bias1), ctypes.c_float(bias2))


def sh_fd_gradient(degree, means, radii, coeff, weights, camera, h=1e-5):
    """n x 51 central differences of the reference loss (position, 48 coeffs)."""
    n = int(radii.shape[0])
    out = np.zeros((n, 51), np.float64)
    lib().oracle_sh_fd_gradient(ctypes.c_int64(n), ctypes.c_int(degree),
                                _p(means), _p(radii), _p(coeff), _p(weights),
                                _p(camera), ctypes.c_double(h), _p(out))
    return out


def torch_bias(step):
    """(bias1, bias2_sqrt) of torch fused Adam at 1-based step, as floats."""
    return float(np.float32(1 - 0.9 ** step)), float(np.float32(math.sqrt(1 - 0.999 ** step)))


# --------------------------------------------------------------------------
# The reference's self-check fixture, restated (SHGradientConsumer.cu:436-467).

def reference_fixture(n=257):
    camera = np.array([.1, -.2, .3], _f32)
    means = np.zeros((n, 3), _f32)
    coeff = np.zeros((n, 48), _f32)
    seed = np.zeros((n, 3), _f32)
    initial = np.zeros((n, 3), _f32)
    first = np.zeros((n, 48), _f32)
    second = np.zeros((n, 48), _f32)
    radii = np.zeros(n, np.int32)
    clamp = np.zeros((n, 3), np.uint8)
    for i in range(n):
        means[i, 0] = camera[0] + _f32(.03) * _f32(i % 19 - 9)
        means[i, 1] = camera[1] + _f32(.04) * _f32(i % 13 - 6)
        means[i, 2] = camera[2] + (_f32(1.2) if i % 2 else _f32(-1.4))
        radii[i] = 1 if i % 7 else 0
        for ch in range(3):
            clamp[i, ch] = (i + ch) % (5 + 2 * ch) == 0
            seed[i, ch] = _f32(.1) * _f32((i + 3 * ch) % 17 - 8) if i % 17 else 0
            initial[i, ch] = _f32(.0625) * _f32(ch - 1)
        for k in range(48):
            field = 48 * i + k
            coeff[i, k] = _f32(.03) * _f32((i + k) % 23 - 11)
            first[i, k] = _f32(1e-5) * _f32(field % 23 - 11) / _f32(11)
            second[i, k] = _f32(1e-8) * (_f32(1) + _f32(field % 17) / _f32(17))
            if field % 19 == 0 and (k < 3 or not radii[i]):
                first[i, k] = second[i, k] = 0
        if i % 14 == 0:
            means[i] = camera
    t = 123
    adam = (float(np.float32(1 / (1 - 0.9 ** t))), float(np.float32(1 / (1 - 0.999 ** t))))
    torch = (float(np.float32(1 - 0.9 ** t)), float(np.float32(math.sqrt(1 - 0.999 ** t))))
    return dict(n=n, camera=camera, means=means, coeff=coeff, seed=seed,
                initial=initial, first=first, second=second, radii=radii,
                clamp=clamp, adam=adam, torch=torch)


def split(values):
    """Packed [n][48] -> (dc [n][3], rest [n][45]) copies."""
    return np.ascontiguousarray(values[:, :3]), np.ascontiguousarray(values[:, 3:])


def fixture_expectations(fx, degree, mode):
    """Expected (dm, coeff, first, second) in double, per the reference's
    self-check (SHGradientConsumer.cu:581-607), and their tolerances."""
    weights = np.where(fx["clamp"] != 0, 0, fx["seed"]).astype(_f32)
    grad = sh_fd_gradient(degree, fx["means"], fx["radii"], fx["coeff"], weights,
                          fx["camera"])
    dm = fx["initial"].astype(np.float64) + grad[:, :3]
    g = grad[:, 3:]
    coeff = fx["coeff"].astype(np.float64)
    first = fx["first"].astype(np.float64)
    second = fx["second"].astype(np.float64)
    if mode == "sgd":
        return dm, coeff - 1e-3 * g, None, None
    a = .9 * first + .1 * g
    v = .999 * second + .001 * g * g
    rate = np.where(np.arange(48) < 3, .0025, .000125)[None, :]
    if mode == "split_torch_adam":
        b1, b2 = fx["torch"]
        expected = coeff - (rate / b1) * a / (np.sqrt(v) / b2 + 1e-15)
    else:
        inv1, inv2 = fx["adam"]
        frate = np.where(np.arange(48) < 3, float(np.float32(.0025)),
                         float(np.float32(.000125)))[None, :]
        expected = coeff - frate * (a * inv1) / (np.sqrt(v * inv2) + 1e-15)
    return dm, expected, a, v


FIXTURE_TOLERANCES = dict(  # SHGradientConsumer.cu:584, 603-606
    dm=(2e-6, 2e-4), first=(2e-9, 2e-4), second=(2e-11, 2e-4), coeff=(5e-8, 4e-7))


def run_fixture_mode(fx, degree, mode, snapshot=True):
    """Runs the oracle on the fixture; returns (dm, coeff48, first48, second48)."""
    dm = fx["initial"].copy()
    common = (degree, fx["means"], fx["radii"], fx["clamp"], fx["camera"], fx["seed"], dm)
    if mode in ("sgd", "adam"):
        coeff, first, second = fx["coeff"].copy(), fx["first"].copy(), fx["second"].copy()
        sh_consume(mode, *common, coeff=coeff, first=first if mode == "adam" else None,
                   second=second if mode == "adam" else None,
                   inv_bias1=fx["adam"][0], inv_bias2=fx["adam"][1])
        return dm, coeff, first, second
    dc, rest = split(fx["coeff"])
    m_dc, m_rest = split(fx["first"])
    v_dc, v_rest = split(fx["second"])
    sh_consume(mode, *common, coefficient=fx["coeff"] if snapshot else None, dc=dc,
               rest=rest, dc_first=m_dc, dc_second=v_dc, rest_first=m_rest,
               rest_second=v_rest, bias1=fx["torch"][0], bias2_sqrt=fx["torch"][1],
               inv_bias1=fx["adam"][0], inv_bias2=fx["adam"][1])
    join = lambda a, b: np.concatenate([a, b], axis=1)
    return dm, join(dc, rest), join(m_dc, m_rest), join(v_dc, v_rest)


# --------------------------------------------------------------------------
# Rasterizer oracle (raster_oracle.c), double precision.

def _d(a):
    return None if a is None else np.ascontiguousarray(a, np.float64)


def _dp(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _scene_args(scene):
    s = {k: _d(v) if isinstance(v, np.ndarray) else v for k, v in scene.items()}
    return s, (ctypes.c_int(s["P"]), ctypes.c_int(s["degree"]), _dp(s["bg"]), _dp(s["means"]),
               _dp(s["opacities"]), _dp(s["scales"]), ctypes.c_double(s["scale_modifier"]),
               _dp(s["rotations"]), _dp(s["view"]), _dp(s["proj"]), ctypes.c_double(s["tanx"]),
               ctypes.c_double(s["tany"]), ctypes.c_int(s["H"]), ctypes.c_int(s["W"]),
               _dp(s["sh"]), _dp(s["campos"]), ctypes.c_int(int(s["antialiasing"])))


def raster_forward(scene):
    """-> (color [3,H,W], invdepth [H,W], radii [P])."""
    s, args = _scene_args(scene)
    color = np.zeros((3, s["H"], s["W"]))
    inv = np.zeros((s["H"], s["W"]))
    radii = np.zeros(s["P"], np.int32)
    lib().oracle_raster_forward(*args, _dp(color), _dp(inv), radii.ctypes.data_as(ctypes.c_void_p))
    return color, inv, radii


def raster_backward(scene, dpix, dinv):
    s, args = _scene_args(scene)
    P = s["P"]
    out = dict(dmean2d=np.zeros((P, 3)), dconic=np.zeros((P, 4)), dopacity=np.zeros(P),
               dcolor=np.zeros((P, 3)), dinvdepth=np.zeros(P), dmeans=np.zeros((P, 3)),
               dcov3d=np.zeros((P, 6)), dsh=np.zeros((P, 48)), dscales=np.zeros((P, 3)),
               drots=np.zeros((P, 4)))
    dpix, dinv = _d(dpix), _d(dinv)
    lib().oracle_raster_backward(*args, _dp(dpix), _dp(dinv),
                                 *[_dp(out[k]) for k in ("dmean2d", "dconic", "dopacity",
                                                         "dcolor", "dinvdepth", "dmeans",
                                                         "dcov3d", "dsh", "dscales", "drots")])
    return out


def pixel_tiles(mean2d, conic_opacity, rgb, depth, radii, width, height, bg, tiles, dpix):
    """Pixel stage of projected 2D Gaussians on the listed tiles (double
    precision; see oracle_pixel_tiles in raster_oracle.c). Inputs are the
    float32 arrays the CUDA path reads. Returns a dict with colour [3,H,W]
    and final_t [H,W] (only the listed tiles' pixels are written), the
    adjoints dmean2d [P,2], dconic [P,3], dopacity [P], dcolor [P,3] from those
    pixels, the matching sizes mag_*, the allowances allow_* for stop
    decisions within rounding and the `ambiguous` flags [P]."""
    P = int(mean2d.shape[0])
    f32 = lambda a: np.ascontiguousarray(a, np.float32)
    mean2d, conic_opacity, rgb, depth = map(f32, (mean2d, conic_opacity, rgb, depth))
    radii = np.ascontiguousarray(radii, np.int32)
    tiles = np.ascontiguousarray(tiles, np.int32)
    bg, dpix = _d(bg), _d(dpix)
    out = dict(color=np.zeros((3, height, width)), final_t=np.zeros((height, width)),
               dmean2d=np.zeros((P, 2)), dconic=np.zeros((P, 3)), dopacity=np.zeros(P),
               dcolor=np.zeros((P, 3)), mag_mean2d=np.zeros((P, 2)),
               mag_conic=np.zeros((P, 3)), mag_opacity=np.zeros(P),
               mag_color=np.zeros((P, 3)), allow_mean2d=np.zeros((P, 2)),
               allow_conic=np.zeros((P, 3)), allow_opacity=np.zeros(P),
               allow_color=np.zeros((P, 3)), ambiguous=np.zeros(P, np.uint8))
    f = lib().oracle_pixel_tiles
    f.restype = ctypes.c_int
    status = f(ctypes.c_int(P), _dp(mean2d), _dp(conic_opacity), _dp(rgb), _dp(depth),
               _dp(radii), ctypes.c_int(width), ctypes.c_int(height), _dp(bg),
               ctypes.c_int(len(tiles)), _dp(tiles), _dp(dpix),
               *[_dp(out[k]) for k in ("color", "final_t", "dmean2d", "dconic", "dopacity",
                                      "dcolor", "mag_mean2d", "mag_conic", "mag_opacity",
                                      "mag_color", "allow_mean2d", "allow_conic",
                                      "allow_opacity", "allow_color", "ambiguous")])
    if status != 0:
        raise MemoryError("oracle_pixel_tiles: out of memory")
    return out


def raster_backward_sized(scene, dpix, dinv):
    """Pixel-stage adjoints with the sizes of their sums and the per-Gaussian
    geometry map (see oracle_raster_backward_sized). Returns x_* and size_*
    for mean2d [P,3], conic [P,4], opacity [P], color [P,3], invdepth [P], and
    jac [P,65,10]: rows (dL/dopacity, dL/dmeans 3, dL/dcov3D 6, dL/dsh 48,
    dL/dscales 3, dL/drotations 4), columns (dmean2D x, y, dconic a, b, c,
    blended opacity, colour r, g, b, inverse depth)."""
    s, args = _scene_args(scene)
    P = s["P"]
    shapes = dict(mean2d=(P, 3), conic=(P, 4), opacity=(P,), color=(P, 3), invdepth=(P,))
    out = {f"{p}_{k}": np.zeros(v) for p in ("x", "size") for k, v in shapes.items()}
    out["jac"] = np.zeros((P, 65, 10))
    dpix, dinv = _d(dpix), _d(dinv)
    lib().oracle_raster_backward_sized(
        *args, _dp(dpix), _dp(dinv), *[_dp(out[f"x_{k}"]) for k in shapes],
        *[_dp(out[f"size_{k}"]) for k in shapes], _dp(out["jac"]))
    return out


def geometry_spread(scene, x, rel=4 * 2.0 ** -24, draws=8):
    """[P,65] spread of the geometry map under rounding-level perturbations of
    all its inputs (see oracle_raster_geometry_spread); x is [P,10] in the
    column order of `jac`."""
    s, args = _scene_args(scene)
    out = np.zeros((s["P"], 65))
    x = _d(x)
    lib().oracle_raster_geometry_spread(*args, _dp(x), ctypes.c_double(rel),
                                        ctypes.c_int(draws), _dp(out))
    return out


GEOMETRY_ROWS = dict(dopacity=slice(0, 1), dmeans=slice(1, 4), dcov3d=slice(4, 10),
                     dsh=slice(10, 58), dscales=slice(58, 61), drots=slice(61, 65))


def geometry_inputs(sized):
    """The pixel-stage vector x [P,10] in the column order of `jac`."""
    return np.concatenate([sized["x_mean2d"][:, :2], sized["x_conic"][:, [0, 1, 3]],
                           sized["x_opacity"][:, None], sized["x_color"],
                           sized["x_invdepth"][:, None]], 1)


def geometry_input_sizes(sized):
    return np.concatenate([sized["size_mean2d"][:, :2], sized["size_conic"][:, [0, 1, 3]],
                           sized["size_opacity"][:, None], sized["size_color"],
                           sized["size_invdepth"][:, None]], 1)


def raster_loss(scene, dpix, dinv):
    s, args = _scene_args(scene)
    dpix, dinv = _d(dpix), _d(dinv)
    f = lib().oracle_raster_loss
    f.restype = ctypes.c_double
    return f(*args, _dp(dpix), _dp(dinv))


def projection_matrix(znear, zfar, tanx, tany):
    """OpenGL-style perspective (row-major) with z mapped to [0, 1] depth,
    the convention of the 3DGS renderer's camera model."""
    top, right = tany * znear, tanx * znear
    P = np.zeros((4, 4))
    P[0, 0] = 2 * znear / (2 * right)
    P[1, 1] = 2 * znear / (2 * top)
    P[3, 2] = 1.0
    P[2, 2] = zfar / (zfar - znear)
    P[2, 3] = -(zfar * znear) / (zfar - znear)
    return P


def raster_scene(P, H, W, seed=0, degree=3, antialiasing=False, spread=0.6, depth=(2.0, 4.0),
                 scale=(0.02, 0.08), rotation=None):
    """Random Gaussians in front of a camera; matrices in the renderer's
    column-major convention (viewmatrix = world-to-camera transposed,
    projmatrix = (proj @ world-to-camera) transposed)."""
    rng = np.random.default_rng(seed)
    tanx = tany = 0.5
    ang = rng.uniform(-0.1, 0.1, 3) if rotation is None else rotation
    cx, cy, cz = np.cos(ang)
    sx, sy, sz = np.sin(ang)
    Rx = np.array([[1, 0, 0], [0, cx, -sx], [0, sx, cx]])
    Ry = np.array([[cy, 0, sy], [0, 1, 0], [-sy, 0, cy]])
    Rz = np.array([[cz, -sz, 0], [sz, cz, 0], [0, 0, 1]])
    R = Rz @ Ry @ Rx
    t = rng.uniform(-0.1, 0.1, 3)
    w2c = np.eye(4)
    w2c[:3, :3] = R
    w2c[:3, 3] = t
    c2w = np.linalg.inv(w2c)
    campos = c2w[:3, 3]
    # Gaussians: place them in camera space, then map to world.
    zc = rng.uniform(*depth, P)
    xc = rng.uniform(-spread, spread, P) * zc * tanx
    yc = rng.uniform(-spread, spread, P) * zc * tany
    cam_pts = np.stack([xc, yc, zc, np.ones(P)], 1)
    means = (c2w @ cam_pts.T).T[:, :3]
    q = rng.standard_normal((P, 4))
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    proj = projection_matrix(0.01, 100.0, tanx, tany)
    return dict(P=P, degree=degree, bg=np.array([0.1, 0.2, 0.3]), means=means,
                opacities=rng.uniform(0.05, 0.99, P), scales=rng.uniform(*scale, (P, 3)),
                scale_modifier=1.0, rotations=q, view=w2c.T.copy(),
                proj=(proj @ w2c).T.copy(), tanx=tanx, tany=tany, H=H, W=W,
                sh=rng.standard_normal((P, 48)) * 0.2, campos=campos,
                antialiasing=antialiasing)
