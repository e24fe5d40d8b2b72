"""Seeded synthetic inputs shared by the parity tests and the benchmark.

Distributions follow the benchmark configurations of the hot path:
SH backward + Adam (N Gaussians, features_dc ~ N(0.5, 0.1), features_rest ~
N(0, 0.05), means ~ U[-1, 1]^3, camera (0, 0, -4), dL/dcolor ~ N(0, 1e-3),
Adam lr 0.0025 / 0.000125) and activation adjoints + Adam (rotations ~ N(0, 1),
log-scales ~ U(-6, -2), opacity logits ~ N(-2, 1), seeds ~ N(0, 1e-4), lr
0.001 / 0.005 / 0.025). Visibility and clamping are drawn so every code path
(invisible, clamped channel, inactive degree) is exercised.
"""

from __future__ import annotations

import math

import numpy as np

F32 = np.float32


def sh_problem(n, seed=42, *, invisible=0.1, clamped=0.1, moments=False,
               camera=(0.0, 0.0, -4.0)):
    rng = np.random.default_rng(seed)
    p = dict(
        means=rng.uniform(-1, 1, (n, 3)).astype(F32),
        camera=np.array(camera, F32),
        radii=np.where(rng.random(n) < invisible, 0, 1 + rng.integers(0, 5, n)).astype(np.int32),
        clamped=(rng.random((n, 3)) < clamped),
        seed=(rng.standard_normal((n, 3)) * 1e-3).astype(F32),
        dm=(rng.standard_normal((n, 3)) * 1e-4).astype(F32),
        dc=rng.normal(0.5, 0.1, (n, 3)).astype(F32),
        rest=rng.normal(0.0, 0.05, (n, 45)).astype(F32),
    )
    if moments:
        p["dc_first"] = (rng.standard_normal((n, 3)) * 1e-3).astype(F32)
        p["dc_second"] = (rng.random((n, 3)) * 1e-6).astype(F32)
        p["rest_first"] = (rng.standard_normal((n, 45)) * 1e-4).astype(F32)
        p["rest_second"] = (rng.random((n, 45)) * 1e-8).astype(F32)
    else:
        for k, w in (("dc_first", 3), ("dc_second", 3), ("rest_first", 45), ("rest_second", 45)):
            p[k] = np.zeros((n, w), F32)
    return p


def activation_problem(n, seed=7, *, scale=1.0, moments=False):
    rng = np.random.default_rng(seed)
    rot = (rng.standard_normal((n, 4)) * scale).astype(F32)
    scl = rng.uniform(-6, -2, (n, 3)).astype(F32)
    opa = rng.normal(-2, 1, (n, 1)).astype(F32)
    raw = [rot, scl, opa]
    seeds = [(rng.standard_normal(r.shape) * 1e-4).astype(F32) for r in raw]
    norm = np.sqrt((rot.astype(np.float64) ** 2).sum(1, keepdims=True)).astype(F32)
    saved = [norm, np.exp(scl).astype(F32),
             (1 / (1 + np.exp(-opa.astype(np.float64)))).astype(F32)]
    if moments:
        first = [(rng.standard_normal(r.shape) * 0.02).astype(F32) for r in raw]
        second = [(rng.random(r.shape) * 0.03).astype(F32) for r in raw]
    else:
        first = [np.zeros_like(r) for r in raw]
        second = [np.zeros_like(r) for r in raw]
    return dict(params=raw, seeds=seeds, saved=saved, first=first, second=second,
                rates=[0.001, 0.005, 0.025])


def bias(step):
    """torch fused Adam bias corrections at a 1-based step, rounded to float."""
    return float(F32(1 - 0.9 ** step)), float(F32(math.sqrt(1 - 0.999 ** step)))


SH_KEYS = ("dm", "dc", "rest", "dc_first", "dc_second", "rest_first", "rest_second")
