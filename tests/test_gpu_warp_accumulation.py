"""The pixel backward's warp accumulation against the reference's own helper.

oracle/_ref/libref_warp.so wraps the reference's clad::cuda::full_warp_key /
warp_accumulate (WarpAccumulation.cuh:9-29), compiled from its source tree.
The product's clad3dgs_warp_accumulate_probe runs the pixel backward's own
accumulation helpers (mode 1: the same full-warp rule; mode 2: the
converged-warp transposing reduction; mode 0: per-lane atomics) on the same
lane streams. The streams restate the reference's self-check
(SHGradientConsumer.cu:326-386): sizes {0, 1, 33, 257} x key patterns {one
key, all distinct, groups of 8, a third of the lanes inactive, per-warp keys},
3D blocks (8, 2, 2) for the first pattern and (16, 2) otherwise, destinations
starting at 0.125 (k % 5 - 2). Sums must match the double-precision sum of
the inputs and each other within the reference's tolerance
5e-6 + 2e-5 |expected|, and the full-warp decision must be the reference's:
grouped exactly for the one-key and per-warp patterns on complete warps.
Mode 2 needs a warp converged on one key (the pixel backward's situation: all
lanes walk the same Gaussian), so it runs on the patterns whose keys agree
within each warp and reports the others as not applicable.
"""

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

REF = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libref_warp.so"
SIZES = (0, 1, 33, 257)
PATTERNS = ("one-key", "distinct", "groups-of-8", "third-inactive", "per-warp")
ROWS = 32


def _streams(n, pattern, fields, seed):
    i = np.arange(n)
    keys = {0: np.zeros(n), 1: i % 32, 2: (i % 32) // 8, 3: np.zeros(n),
            4: (i // 32) % 3}[pattern].astype(np.int32)
    active = np.ones(n, np.uint8)
    if pattern == 3:
        active[i % 3 == 0] = 0
    values = np.random.default_rng(seed).standard_normal((n, fields)).astype(np.float32)
    values *= np.float32(0.125)
    block = (8, 2, 2) if pattern == 0 else (16, 2, 1)
    return keys, active, values, block


def _initial(fields):
    k = np.arange(ROWS * fields)
    return (0.125 * (k % 5 - 2)).astype(np.float32).reshape(ROWS, fields)


def _expected(keys, active, values, fields):
    out = _initial(fields).astype(np.float64)
    for key, on, v in zip(keys, active, values):
        if on:
            out[key] += v.astype(np.float64)
    return out


def _launch(fn, device, keys, active, values, block, fields, *, probe_mode=None):
    n = len(keys)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)
    dk, da, dv = t(np.maximum(keys, 0) if n else np.zeros(1, np.int32)), \
        t(active if n else np.zeros(1, np.uint8)), t(values if n else np.zeros((1, fields),
                                                                                np.float32))
    out = t(_initial(fields))
    grouped = torch.full((max(n, 1),), 7, dtype=torch.int32, device=device)
    args = [n, fields, dk.data_ptr(), da.data_ptr(), dv.data_ptr(), out.data_ptr(), ROWS,
            grouped.data_ptr(), *block, None]
    if probe_mode is None:
        status = fn(*args)
    else:
        status = fn(probe_mode, *args)
    assert status == 0, status
    torch.cuda.synchronize()
    return out.cpu().numpy().astype(np.float64), grouped.cpu().numpy()[:n]


def _within(got, expected, what):
    bad = np.abs(got - expected) > 5e-6 + 2e-5 * np.abs(expected)
    assert not bad.any(), (what, got[bad][:4], expected[bad][:4])


@pytest.fixture(scope="module")
def reference_helper():
    if not REF.exists():
        pytest.skip(f"{REF} not built (needs the reference sources at build time)")
    lib = ctypes.CDLL(str(REF))
    lib.ref_warp_accumulate.restype = ctypes.c_int
    lib.ref_warp_accumulate.argtypes = [ctypes.c_int] * 2 + [ctypes.c_void_p] * 4 + \
        [ctypes.c_int, ctypes.c_void_p] + [ctypes.c_int] * 3 + [ctypes.c_void_p]
    return lib.ref_warp_accumulate


def _probe():
    import _native

    return _native.library().clad3dgs_warp_accumulate_probe


@pytest.mark.parametrize("fields", [3, 10])
@pytest.mark.parametrize("pattern", range(5), ids=PATTERNS)
@pytest.mark.parametrize("n", SIZES)
def test_full_warp_rule_matches_reference_helper(cuda, reference_helper, n, pattern, fields):
    keys, active, values, block = _streams(n, pattern, fields, seed=n * 7 + pattern)
    expected = _expected(keys, active, values, fields)
    ref_out, ref_grouped = _launch(reference_helper, cuda, keys, active, values, block, fields)
    _within(ref_out, expected, "reference helper")
    # The reference's own expectation of which lanes reduce as a warp.
    for i in range(n):
        if active[i]:
            full = pattern in (0, 4) and (i // 32 + 1) * 32 <= n
            assert ref_grouped[i] == full, (i, ref_grouped[i])
    out, grouped = _launch(_probe(), cuda, keys, active, values, block, fields, probe_mode=1)
    _within(out, expected, "mode 1")
    _within(out, ref_out, "mode 1 vs reference")
    assert np.array_equal(grouped[active == 1], ref_grouped[active == 1])
    plain, _ = _launch(_probe(), cuda, keys, active, values, block, fields, probe_mode=0)
    _within(plain, ref_out, "per-lane atomics vs reference")


@pytest.mark.parametrize("fields", [3, 9, 10, 16])
@pytest.mark.parametrize("pattern", [0, 3, 4], ids=["one-key", "third-inactive", "per-warp"])
@pytest.mark.parametrize("n", SIZES)
def test_converged_reduction_matches_reference_helper(cuda, reference_helper, n, pattern,
                                                      fields):
    keys, active, values, block = _streams(n, pattern, fields, seed=n * 11 + pattern)
    ref_out, _ = _launch(reference_helper, cuda, keys, active, values, block, fields)
    out, grouped = _launch(_probe(), cuda, keys, active, values, block, fields, probe_mode=2)
    _within(out, _expected(keys, active, values, fields), "mode 2")
    _within(out, ref_out, "mode 2 vs reference")
    assert (grouped == 1).all()


@pytest.mark.parametrize("pattern", [1, 2], ids=["distinct", "groups-of-8"])
def test_converged_reduction_refuses_mixed_keys(cuda, pattern):
    keys, active, values, block = _streams(257, pattern, 10, seed=3)
    out, grouped = _launch(_probe(), cuda, keys, active, values, block, 10, probe_mode=2)
    # Eight full warps of mixed keys add nothing; the last warp holds a single
    # lane (257 = 8 x 32 + 1), whose key trivially agrees.
    assert (grouped[:256] == -1).all() and grouped[256] == 1
    expected = _initial(10).astype(np.float64)
    expected[keys[256]] += values[256]
    _within(out, expected, "mode 2, single-lane warp")


def test_probe_rejects_bad_launches(cuda):
    probe = _probe()
    for mode, fields, block in ((3, 10, (32, 1, 1)), (1, 0, (32, 1, 1)), (1, 17, (32, 1, 1)),
                                (2, 10, (16, 1, 1)), (2, 10, (33, 1, 1))):
        assert probe(mode, 1, fields, None, None, None, None, ROWS, None, *block, None) != 0
