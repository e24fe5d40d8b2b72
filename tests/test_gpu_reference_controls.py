"""Product kernels vs the reference's own kernels, run on the same GPU.

oracle/_ref/ holds the reference's handwritten controls (controls/ManualSH.cu,
controls/ManualActivations.cu) compiled from its sources for sm_100a by
oracle/Makefile, plus ManualSH.cu's own self-check main(). The reference's
Clad-generated kernels need Clang + Clad and are not built. Parity bar (the
path's stated tolerance): fp32 relative error <= 1e-5 on adjoints, parameters
and moments. Where the reference compiles with FMA contraction, a gradient that
is zero up to rounding can change sign at Adam step 1, where the update is
lr * sign(g); those elements are allowed one sign flip of the update.
"""

import ctypes
import math
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

import cases

pytestmark = pytest.mark.gpu

REF = Path(__file__).resolve().parents[1] / "oracle" / "_ref"


class TorchAdamConfig(ctypes.Structure):
    _fields_ = [("bias1", ctypes.c_float), ("bias2_sqrt", ctypes.c_float)]


def _ref_lib(name):
    path = REF / name
    if not path.exists():
        pytest.skip(f"{path} not built (needs the reference sources at build time)")
    return ctypes.CDLL(str(path))


def _dev(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def test_reference_control_self_check_passes_on_b200():
    exe = REF / "manual_sh_selfcheck"
    if not exe.exists():
        pytest.skip("reference self-check not built")
    result = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert result.returncode == 0, result.stderr
    assert "OK" in result.stdout


def _run_sh(fn, p, degree, step, device, torch_config):
    t = {k: _dev(p[k], device) for k in ("means", "radii", "clamped", "seed", "camera")
         + cases.SH_KEYS}
    args = [t["means"].data_ptr(), t["radii"].data_ptr(), None, t["clamped"].data_ptr(),
            t["camera"].data_ptr(), t["seed"].data_ptr()] + [t[k].data_ptr() for k in cases.SH_KEYS]
    fn(len(p["radii"]), degree, *args, torch_config)
    torch.cuda.synchronize()
    return {k: t[k].cpu().numpy() for k in cases.SH_KEYS}


@pytest.mark.parametrize("degree", [0, 1, 2, 3])
@pytest.mark.parametrize("step", [1, 100])
def test_sh_consume_matches_reference_control(cuda, degree, step):
    ref = _ref_lib("libref_manual_sh.so")
    ref.sh_consumer_split_torch_adam.restype = None
    ref.sh_consumer_split_torch_adam.argtypes = [ctypes.c_int, ctypes.c_int] + \
        [ctypes.c_void_p] * 13 + [TorchAdamConfig]
    import _native as native

    n = 100_000
    p = cases.sh_problem(n, seed=42 + degree, moments=step > 1)
    b1, b2 = cases.bias(step)
    ours = _run_sh(native.library().sh_consumer_split_torch_adam, p, degree, step, cuda,
                   native.TorchAdamConfig(b1, b2))
    theirs = _run_sh(ref.sh_consumer_split_torch_adam, p, degree, step, cuda,
                     TorchAdamConfig(b1, b2))
    report = {}
    for k in cases.SH_KEYS:
        a, b = ours[k].astype(np.float64), theirs[k].astype(np.float64)
        report[k] = float((ours[k].view(np.uint32) == theirs[k].view(np.uint32)).mean())
        # Relative to the operands of the last operation (old and new value):
        # an update that cancels a parameter to ~0 is judged against the
        # parameter it changed, not against the ~0 result.
        scale = np.maximum(np.abs(b), np.abs(p[k].astype(np.float64)))
        close = np.abs(a - b) <= 1e-5 * scale + 1e-30
        if k == "dm":
            # dm sums 16 term adjoints; where they cancel, relative error is
            # measured against the adjoints' scale (normwise relative 1e-5).
            close |= np.abs(a - b) <= 1e-5 * np.sqrt(np.mean(b * b))
        if k in ("dc", "rest"):
            lr = 0.0025 if k == "dc" else 0.000125
            # Step-1 sign flips of a rounding-level gradient: the update is
            # +-lr/bias1 * m/(sqrt(v)/bias2) ~ +-lr.
            m_ours, m_ref = ours[k + "_first"], theirs[k + "_first"]
            flip = np.abs(m_ours - m_ref) > 1e-5 * np.abs(m_ref) + 1e-20
            close |= flip & (np.abs(a - b) <= 2.0 * lr * 1.0001)
        elif k.endswith("first") or k.endswith("second"):
            # moments of a rounding-level gradient are rounding-level themselves
            close |= np.abs(a - b) <= (1e-9 if k.endswith("first") else 1e-15)
        assert close.all(), (k, int((~close).sum()), a[~close][:4], b[~close][:4])
    print(f"degree {degree} step {step} bit-identical fractions: {report}")


def test_activation_consume_matches_reference_control(cuda):
    ref = _ref_lib("libref_manual_activations.so")
    fn = ref.launch_activation_consume
    fn.restype = None
    PP = ctypes.POINTER(ctypes.c_void_p)
    fn.argtypes = [ctypes.c_int, PP, PP, PP, PP, PP, ctypes.POINTER(ctypes.c_double),
                   ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_float),
                   ctypes.c_void_p]
    import _native as native

    n = 1_000_000
    p = cases.activation_problem(n, seed=7, moments=True)
    counters = [41, 44, 48]
    b1 = [1 - 0.9 ** (c + 1) for c in counters]
    b2 = [math.sqrt(1 - 0.999 ** (c + 1)) for c in counters]
    results = []
    for launch in (native.library().launch_activation_consume, fn):
        dev = {k: [_dev(a, cuda) for a in p[k]] for k in
               ("params", "seeds", "saved", "first", "second")}
        arrays = [native.pointer_array([t.data_ptr() for t in dev[k]])
                  for k in ("params", "seeds", "saved", "first", "second")]
        arrays = [ctypes.cast(a, PP) for a in arrays]
        launch(n, *arrays, native.doubles(p["rates"]), native.floats(b1),
               native.floats(b2), None)
        torch.cuda.synchronize()
        results.append({k: [t.cpu().numpy() for t in dev[k]] for k in ("params", "first", "second")})
    ours, theirs = results
    for key in ("params", "first", "second"):
        for j in range(3):
            a, b = ours[key][j], theirs[key][j]
            same = (a.view(np.uint32) == b.view(np.uint32)).mean()
            np.testing.assert_allclose(a, b, rtol=1e-5, atol=1e-12, err_msg=f"{key}[{j}]")
            print(f"activation {key}[{j}] bit-identical fraction {same:.6f}")


def test_quaternion_backward_matches_reference_control(cuda):
    ref = _ref_lib("libref_manual_activations.so")
    fn = ref.launch_quaternion_backward
    fn.restype = None
    fn.argtypes = [ctypes.c_int] + [ctypes.c_void_p] * 5
    import clad_quaternion

    torch.manual_seed(3)
    q = torch.randn((100_003, 4), device=cuda)
    q[::97] *= 1e-13
    seed = torch.randn_like(q)
    norms = q.norm(2, dim=1, keepdim=True)
    out = torch.empty_like(q)
    fn(q.shape[0], q.data_ptr(), seed.data_ptr(), norms.data_ptr(), out.data_ptr(), None)
    ours = clad_quaternion.backward(q, seed, norms)
    torch.cuda.synchronize()
    assert torch.equal(ours, out)
