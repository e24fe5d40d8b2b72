"""Quaternion normalisation whose backward runs the CUDA VJP (the
trainer-facing `normalization` module; same names and behaviour as the
reference's normalization.py:1-40).

The forward is torch's F.normalize(dim=1, eps=1e-12) arithmetic with the norm
kept; the first-order backward calls `extension.backward(raw, seed, norm)`,
whose clamp branch is chosen by that saved norm. Tensors the CUDA kernel does
not take (not CUDA, not float32, not [N, 4]) stay on torch's own path.
"""

from __future__ import annotations

from functools import wraps

import torch
import torch.nn.functional as F

_EPS = 1e-12


def _kernel_shaped(q) -> bool:
    return q.is_cuda and q.dtype == torch.float32 and q.ndim == 2 and q.shape[1] == 4


class NormalizeQuaternion(torch.autograd.Function):
    @staticmethod
    def forward(ctx, raw, extension):
        norm = raw.norm(2, dim=1, keepdim=True)
        ctx.extension = extension
        ctx.save_for_backward(raw, norm)
        return raw / norm.clamp_min(_EPS).expand_as(raw)

    @staticmethod
    def backward(ctx, seed):
        if torch.is_grad_enabled():
            raise RuntimeError("Quaternion activation supports first-order backward only")
        raw, norm = ctx.saved_tensors
        return ctx.extension.backward(raw, seed, norm), None


def normalize_quaternion(q, extension):
    if _kernel_shaped(q):
        return NormalizeQuaternion.apply(q, extension)
    return F.normalize(q, dim=1, eps=_EPS)


def enable_quaternion_backward(model_class, extension):
    """Makes every model built after this call normalise its rotations through
    `normalize_quaternion` (GaussianModel.setup_functions installs the
    activation, so the hook wraps it)."""
    install = model_class.setup_functions

    @wraps(install)
    def setup_functions(model):
        install(model)
        model.rotation_activation = lambda q: normalize_quaternion(q, extension)

    model_class.setup_functions = setup_functions
