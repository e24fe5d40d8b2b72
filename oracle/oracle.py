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
