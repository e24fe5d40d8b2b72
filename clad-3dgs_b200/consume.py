"""Torch-tensor entry points of the per-Gaussian backward-and-update kernels.

Each function validates like the reference's C++ wrappers (TORCH_CHECK ->
RuntimeError before any write; normalization.cpp:16-31,56-104 and
direct_inputs.py:321-344) and then calls the C ABI of libclad3dgs_b200.so on
torch's current stream. There is no CPU path: inputs must be CUDA tensors and
the library must be built.
"""

from __future__ import annotations

import torch

import _native as native


def _require(condition: bool, message: str) -> None:
    if not condition:
        raise RuntimeError(message)


def _region(t: torch.Tensor):
    start = t.data_ptr()
    return start, start + t.numel() * t.element_size()


def check_disjoint(writable, readonly=(), message="buffers must be disjoint"):
    """Raises if any writable tensor shares bytes with another tensor."""
    ranges = [(_region(t), True) for t in writable if t.numel()]
    ranges += [(_region(t), False) for t in readonly if t is not None and t.numel()]
    for i in range(len(ranges)):
        (a0, a1), wa = ranges[i]
        for j in range(i + 1, len(ranges)):
            (b0, b1), wb = ranges[j]
            if (wa or wb) and a0 < b1 and b0 < a1:
                raise RuntimeError(message)


def _cuda_f32(t, device, name, contiguous=True):
    _require(t.is_cuda and t.device == device, f"{name} must be on {device}")
    _require(t.dtype == torch.float32, f"{name} must be float32")
    if contiguous:
        _require(t.is_contiguous(), f"{name} must be contiguous")


def _position_state(xyz, means, n, device):
    """Checks the optional position Adam state {first, second, rate, bias1,
    bias2_sqrt}; means is then updated in place and must be the parameter."""
    if xyz is None:
        return None
    _cuda_f32(means, device, "means")
    for key in ("first", "second"):
        _cuda_f32(xyz[key], device, "xyz " + key)
        _require(xyz[key].numel() == 3 * n, f"bad xyz {key} shape")
    return xyz


def sh_consume_split_torch_adam(means, radii, clamped, camera, seed, dm, dc, rest,
                                dc_first, dc_second, rest_first, rest_second, *,
                                bias1: float, bias2_sqrt: float, degree: int,
                                coefficient=None, xyz=None, stream=None):
    """Fused SH VJP + torch-fused Adam on split dc/rest (in place), dm += the
    position adjoint. Same contract as sh_consumer_split_torch_adam. With `xyz`
    ({first, second, rate, bias1, bias2_sqrt}) the same pass also runs
    torch-fused Adam on means in place, dm being their complete gradient."""
    n = means.shape[0]
    device = means.device
    xyz = _position_state(xyz, means, n, device)
    _require(0 <= degree <= 3, "SH degree must be between zero and three")
    _require(means.dim() == 2 and means.shape[1] == 3, "means must be [N, 3]")
    for name, t, numel in (("dc", dc, 3 * n), ("rest", rest, 45 * n),
                           ("dc_first", dc_first, 3 * n), ("dc_second", dc_second, 3 * n),
                           ("rest_first", rest_first, 45 * n),
                           ("rest_second", rest_second, 45 * n), ("dm", dm, 3 * n)):
        _cuda_f32(t, device, name)
        _require(t.numel() == numel, f"bad {name} shape")
    means = means.contiguous()
    radii = radii.contiguous()
    clamped = clamped.contiguous()
    camera = camera.contiguous()
    seed = seed.contiguous()
    _require(radii.dtype == torch.int32 and radii.numel() == n, "radii must be int32 [N]")
    _require(clamped.dtype == torch.bool and clamped.numel() == 3 * n, "clamped must be bool [N, 3]")
    _require(seed.numel() == 3 * n and seed.dtype == torch.float32, "seed must be float32 [N, 3]")
    _require(camera.numel() == 3 and camera.dtype == torch.float32, "camera must be 3 floats")
    for t in (means, radii, clamped, camera, seed):
        _require(t.is_cuda and t.device == device, "inputs must share the CUDA device")
    if coefficient is not None:
        coefficient = coefficient.contiguous()
        _require(coefficient.numel() == 48 * n and coefficient.dtype == torch.float32,
                 "coefficient snapshot must be float32 [N, 16, 3]")
    writable = [dc, rest, dc_first, dc_second, rest_first, rest_second, dm]
    if xyz is not None:
        writable += [means, xyz["first"], xyz["second"]]
    check_disjoint(writable, [clamped, seed, camera, coefficient] +
                   ([] if xyz is not None else [means]),
                   "direct SH coefficient and moment buffers must be disjoint")
    if n == 0:
        return
    if xyz is not None:
        native.check(native.library().clad3dgs_sh_consume_xyz(
            n, degree, native.ptr(means), native.ptr(radii), native.ptr(coefficient),
            native.ptr(clamped), native.ptr(camera), native.ptr(seed), native.ptr(dm),
            native.ptr(dc), native.ptr(rest), native.ptr(dc_first), native.ptr(dc_second),
            native.ptr(rest_first), native.ptr(rest_second),
            native.TorchAdamConfig(bias1, bias2_sqrt), native.ptr(xyz["first"]),
            native.ptr(xyz["second"]), float(xyz["rate"]),
            native.TorchAdamConfig(xyz["bias1"], xyz["bias2_sqrt"]),
            native.stream_handle(stream)), "SH + position consume")
        return
    native.check(native.library().clad3dgs_sh_consume_split_torch_adam(
        n, degree, native.ptr(means), native.ptr(radii), native.ptr(coefficient),
        native.ptr(clamped), native.ptr(camera), native.ptr(seed), native.ptr(dm),
        native.ptr(dc), native.ptr(rest), native.ptr(dc_first), native.ptr(dc_second),
        native.ptr(rest_first), native.ptr(rest_second),
        native.TorchAdamConfig(bias1, bias2_sqrt), native.stream_handle(stream)),
        "SH consume")


def sh_consume_variant(mode: str, means, radii, clamped, camera, seed, dm, *, degree,
                       inv_bias1=1.0, inv_bias2=1.0, coeff=None, first=None,
                       second=None, coefficient=None, dc=None, rest=None,
                       dc_first=None, dc_second=None, rest_first=None,
                       rest_second=None, stream=None):
    """The reference's test variants: 'sgd', 'adam' (packed) and 'split_adam'."""
    modes = {"sgd": 0, "adam": 1, "split_adam": 2}
    n = means.shape[0]
    if n == 0:
        return
    native.check(native.library().clad3dgs_sh_consume_variant(
        modes[mode], n, degree, native.ptr(means), native.ptr(radii),
        native.ptr(coefficient), native.ptr(clamped), native.ptr(camera),
        native.ptr(seed), native.ptr(dm), native.ptr(coeff), native.ptr(first),
        native.ptr(second), native.ptr(dc), native.ptr(rest), native.ptr(dc_first),
        native.ptr(dc_second), native.ptr(rest_first), native.ptr(rest_second),
        native.AdamConfig(inv_bias1, inv_bias2), native.stream_handle(stream)),
        f"SH consume ({mode})")


def _activation_arrays(parameters, seeds, saved, first, second):
    return [native.pointer_array([t.data_ptr() for t in group])
            for group in (parameters, seeds, saved, first, second)]


def activation_consume_raw(parameters, seeds, saved, first, second, rates, bias1,
                           bias2, stream=None):
    """Launch without validation (callers validated already)."""
    n = parameters[0].shape[0]
    if n == 0:
        return
    arrays = _activation_arrays(parameters, seeds, saved, first, second)
    native.check(native.library().clad3dgs_activation_consume(
        n, *arrays, native.doubles(rates), native.floats(bias1), native.floats(bias2),
        native.stream_handle(stream)), "activation consume")


def quaternion_backward_raw(q, seed, norms, out, stream=None):
    n = q.shape[0]
    if n == 0:
        return out
    native.check(native.library().clad3dgs_quaternion_backward(
        n, q.data_ptr(), seed.data_ptr(), norms.data_ptr(), out.data_ptr(),
        native.stream_handle(stream)), "quaternion backward")
    return out


def gaussian_step(means, radii, clamped, camera, seed, dm, dc, rest, dc_first,
                  dc_second, rest_first, rest_second, *, bias1, bias2_sqrt, degree,
                  act_parameters, act_seeds, act_saved, act_first, act_second,
                  act_rates, act_bias1, act_bias2, coefficient=None, xyz=None,
                  stream=None):
    """SH consume and activation consume fused into one pass per Gaussian (with
    `xyz`, the positions' Adam too: all 59 parameters of a Gaussian in one pass).
    Inputs are trusted to be contiguous, disjoint CUDA float32 buffers in the
    reference layouts (validate with the separate entry points' rules)."""
    n = means.shape[0]
    if n == 0:
        return
    arrays = _activation_arrays(act_parameters, act_seeds, act_saved, act_first,
                                act_second)
    if xyz is not None:
        native.check(native.library().clad3dgs_gaussian_step_xyz(
            n, degree, native.ptr(means), native.ptr(radii), native.ptr(coefficient),
            native.ptr(clamped), native.ptr(camera), native.ptr(seed), native.ptr(dm),
            native.ptr(dc), native.ptr(rest), native.ptr(dc_first), native.ptr(dc_second),
            native.ptr(rest_first), native.ptr(rest_second),
            native.TorchAdamConfig(bias1, bias2_sqrt), *arrays,
            native.doubles(act_rates), native.floats(act_bias1), native.floats(act_bias2),
            native.ptr(xyz["first"]), native.ptr(xyz["second"]), float(xyz["rate"]),
            native.TorchAdamConfig(xyz["bias1"], xyz["bias2_sqrt"]),
            native.stream_handle(stream)), "fused Gaussian step with positions")
        return
    native.check(native.library().clad3dgs_gaussian_step(
        n, degree, native.ptr(means), native.ptr(radii), native.ptr(coefficient),
        native.ptr(clamped), native.ptr(camera), native.ptr(seed), native.ptr(dm),
        native.ptr(dc), native.ptr(rest), native.ptr(dc_first), native.ptr(dc_second),
        native.ptr(rest_first), native.ptr(rest_second),
        native.TorchAdamConfig(bias1, bias2_sqrt), *arrays,
        native.doubles(act_rates), native.floats(act_bias1), native.floats(act_bias2),
        native.stream_handle(stream)), "fused Gaussian step")


def host_step_workspace(chunk: int) -> int:
    return int(native.library().clad3dgs_host_step_workspace(chunk))


def gaussian_step_host(means, radii, clamped, camera, seed, dm, dc, rest, dc_first,
                       dc_second, rest_first, rest_second, *, bias1, bias2_sqrt,
                       degree, act_parameters, act_seeds, act_saved, act_first,
                       act_second, act_rates, act_bias1, act_bias2, workspace,
                       chunk, stream=None):
    """Fused step over (pinned) host tensors; workspace is a CUDA uint8 tensor of
    host_step_workspace(chunk) bytes. Returns when results are back on the host."""
    n = means.shape[0]
    if n == 0:
        return
    arrays = _activation_arrays(act_parameters, act_seeds, act_saved, act_first,
                                act_second)
    native.check(native.library().clad3dgs_gaussian_step_host(
        n, degree, means.data_ptr(), radii.data_ptr(), clamped.data_ptr(),
        camera.data_ptr(), seed.data_ptr(), dm.data_ptr(), dc.data_ptr(),
        rest.data_ptr(), dc_first.data_ptr(), dc_second.data_ptr(),
        rest_first.data_ptr(), rest_second.data_ptr(),
        native.TorchAdamConfig(bias1, bias2_sqrt), *arrays,
        native.doubles(act_rates), native.floats(act_bias1), native.floats(act_bias2),
        workspace.data_ptr(), workspace.numel(), chunk, native.stream_handle(stream)),
        "host-buffer Gaussian step")
