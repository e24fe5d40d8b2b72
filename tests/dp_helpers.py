"""Shared pieces of the data-parallel tests: seeded Gaussians, saved
activations computed on the host, and the oracle as the exchange's update."""

import numpy as np
import torch

import oracle

RATES = dict(xyz=0.00016, f_dc=0.0025, f_rest=0.000125, scaling=0.005, rotation=0.001,
             opacity=0.025)
GROUP_NAMES = ("xyz", "sh", "scaling", "rotation", "opacity")


def initial_values(n, seed=3, device="cpu"):
    """The 8-view configuration's distributions: means U[-1,1]^3, f_dc
    N(0.5, 0.1), f_rest N(0, 0.05), log-scales U(-6, -2), quaternions N(0, 1),
    opacity logits N(-2, 1)."""
    g = torch.Generator().manual_seed(seed)
    sh = torch.randn(n, 16, 3, generator=g) * 0.05
    sh[:, 0] = 0.5 + 0.1 * torch.randn(n, 3, generator=g)
    values = dict(xyz=torch.rand(n, 3, generator=g) * 2 - 1, sh=sh.reshape(n, 48),
                  scaling=torch.rand(n, 3, generator=g) * 4 - 6,
                  rotation=torch.randn(n, 4, generator=g),
                  opacity=torch.randn(n, 1, generator=g) - 2)
    return {k: v.to(device).contiguous() for k, v in values.items()}


def saved_from(params):
    """Saved forward values of the activations, in float32 on the host."""
    s = params["scaling"].detach().cpu().numpy().astype(np.float32)
    q = params["rotation"].detach().cpu().numpy().astype(np.float32)
    o = params["opacity"].detach().cpu().numpy().astype(np.float32).reshape(-1)
    norm = np.sqrt(((q[:, 0] * q[:, 0] + q[:, 1] * q[:, 1]) + q[:, 2] * q[:, 2])
                   + q[:, 3] * q[:, 3]).astype(np.float32)
    return dict(scaling=np.exp(s).astype(np.float32),
                opacity=(1 / (1 + np.exp(-o))).astype(np.float32),
                norm=norm)


def view_gradients(rank, step, padded, n):
    """Deterministic per-view gradients of one rank (padding rows zero)."""
    g = torch.Generator().manual_seed(1000 * step + rank)
    out = {}
    for name, k in zip(GROUP_NAMES, (3, 48, 3, 4, 1)):
        t = torch.zeros(padded, k)
        t[:n] = torch.randn(n, k, generator=g) * 1e-3
        out[name] = t
    return out


def oracle_update(s):
    """ShardStep on CPU tensors -> oracle.shard_update in place."""
    np_ = lambda t: t.numpy()
    oracle.shard_update(s.begin, s.end, s.grad_origin,
                        [[np_(t) for t in row] for row in s.grads],
                        [np_(t) for t in s.params[s.local]], [np_(t) for t in s.first],
                        [np_(t) for t in s.second], np_(s.saved_scaling),
                        np_(s.saved_opacity), np_(s.saved_norm), s.rates, s.bias1,
                        s.bias2_sqrt)
    for q, row in enumerate(s.params):
        if q != s.local:
            for dst, src in zip(row, s.params[s.local]):
                dst.copy_(src)
