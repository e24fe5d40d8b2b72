"""The reference's `clad_quaternion` extension surface over the C ABI.

Mirrors normalization.cpp:33-128: `backward(q, seed, norms)` and
`consume_activations(parameters, seeds, saved, first, second, rates, bias1,
bias2)`, with the same argument meaning and the same checks raising
RuntimeError before any write. Strided seeds and saved activations are packed
(normalization.cpp:222-223); writable tensors must be contiguous and disjoint
from every other argument (normalization.cpp:226-233). Kernels launch on
torch's current stream.
"""

from __future__ import annotations

import math

import torch

import consume

INT_MAX = 2**31 - 1


def _check(condition: bool, message: str) -> None:
    if not condition:
        raise RuntimeError(message)


def _validate_quaternion(q, seed, norms):
    # normalization.cpp:16-31
    _check(q.is_cuda and seed.is_cuda and norms.is_cuda and q.device == seed.device
           and q.device == norms.device, "Quaternion inputs must share a CUDA device")
    _check(q.dtype == torch.float32 and seed.dtype == torch.float32
           and norms.dtype == torch.float32, "Quaternion inputs must be float32")
    _check(q.dim() == 2 and q.shape[1] == 4 and q.shape == seed.shape
           and q.shape[0] <= INT_MAX // 4, "Quaternion inputs must have matching [N, 4] shapes")
    _check(norms.dim() == 2 and norms.shape[0] == q.shape[0] and norms.shape[1] == 1,
           "Saved quaternion norms must have shape [N, 1]")


def backward(q: torch.Tensor, seed: torch.Tensor, norms: torch.Tensor) -> torch.Tensor:
    """VJP of q / max(|q|, 1e-12) wrt q, clamp branch chosen by the saved norm."""
    _validate_quaternion(q, seed, norms)
    with torch.cuda.device(q.device):
        q, seed, norms = q.contiguous(), seed.contiguous(), norms.contiguous()
        out = torch.empty_like(q)
        return consume.quaternion_backward_raw(q, seed, norms, out)


def consume_activations(parameters, seeds, saved, first, second, rates, bias1, bias2):
    """Rotation/scaling/opacity VJPs fused with their dense Adam updates, in place.

    Lists of three: rotation [N, 4], scaling [N, 3], opacity [N, 1]; saved =
    (norm [N, 1], exp(scaling) [N, 3], sigmoid(opacity) [N, 1]); bias1 = 1-0.9^t,
    bias2 = sqrt(1-0.999^t) per group. Does not touch step counters.
    """
    _check(len(parameters) == 3 and len(seeds) == 3 and len(saved) == 3
           and len(first) == 3 and len(second) == 3 and len(rates) == 3
           and len(bias1) == 3 and len(bias2) == 3,
           "Activation consumption requires rotation, scaling and opacity")
    _validate_quaternion(parameters[0], seeds[0], saved[0])
    device = parameters[0].device
    n = parameters[0].shape[0]
    _check(n <= INT_MAX // 4, "Activation batch exceeds index range")
    seeds, saved = list(seeds), list(saved)
    writable = []
    for j, width in enumerate((4, 3, 1)):
        p = parameters[j]
        _check(p.is_cuda and p.device == device and p.dtype == torch.float32
               and p.dim() == 2 and p.shape[0] == n and p.shape[1] == width
               and p.is_contiguous(), "Unsupported activation parameter layout")
        for value in (first[j], second[j]):
            _check(value.device == device and value.dtype == torch.float32
                   and value.shape == p.shape and value.is_contiguous(),
                   "Activation moments must match their parameter")
        _check(seeds[j].device == device and seeds[j].dtype == torch.float32
               and seeds[j].shape == p.shape, "Invalid activation seed")
        _check(saved[j].device == device and saved[j].dtype == torch.float32
               and saved[j].dim() == 2 and saved[j].shape[0] == n
               and saved[j].shape[1] == (3 if j == 1 else 1), "Invalid saved activation")
        _check(math.isfinite(rates[j]) and rates[j] >= 0 and math.isfinite(bias1[j])
               and 0 < bias1[j] <= 1 and math.isfinite(bias2[j]) and 0 < bias2[j] <= 1,
               "Invalid activation Adam configuration")
        seeds[j] = seeds[j].contiguous()
        saved[j] = saved[j].contiguous()
        writable += [p, first[j], second[j]]
    try:
        consume.check_disjoint(writable, seeds + saved)
    except RuntimeError:
        raise RuntimeError("unsupported operation: some elements of the input tensor "
                           "and the written-to tensor refer to a single memory location")
    with torch.cuda.device(device):
        consume.activation_consume_raw(list(parameters), seeds, saved, list(first),
                                       list(second), rates, bias1, bias2)
