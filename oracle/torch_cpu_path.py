"""The reference's PyTorch CPU path for one per-Gaussian step, restated.

TEST/BENCHMARK INFRASTRUCTURE ONLY: bench.py times this as the CPU baseline
(its `--impl reference` arm and the `cpu_baseline` field); the product never
imports it.

The reference trainer's CPU path for these parameters is: colours from the SH
coefficients with Graphdeco's `eval_sh` (degree <= 3, +0.5, clamp at 0), the
activations normalize(rotation) / exp(scaling) / sigmoid(opacity), autograd
back to the raw parameters and the position, and `torch.optim.Adam` on every
parameter group. The trainer module (graphdeco-inria/gaussian-splatting @
54c035f7, utils/sh_utils.py) is not vendored in the reference; the basis below
is the same real-SH basis as the reference's SHGradientConsumer.cu:20-76 and
the colour convention is the renderer's (+0.5, clamp_min 0). Groups and
hyperparameters follow the reference's fixed settings (adapter.py:252-285,
activation.py and check.py): SH lr 0.0025 / 0.000125, rotation 0.001, scaling
0.005, opacity 0.025, betas (0.9, 0.999), eps 1e-15.
"""

from __future__ import annotations

import os
import time

import torch

C0 = 0.28209479177387814
C1 = 0.4886025119029199
C2 = (1.0925484305920792, -1.0925484305920792, 0.31539156525252005,
      -1.0925484305920792, 0.5462742152960396)
C3 = (-0.5900435899266435, 2.890611442640554, -0.4570457994644658,
      0.3731763325901154, -0.4570457994644658, 1.445305721320277,
      -0.5900435899266435)


def eval_sh(degree: int, sh: torch.Tensor, dirs: torch.Tensor) -> torch.Tensor:
    """sh [..., 3, (degree+1)^2] (channel-major), dirs [..., 3] unit vectors."""
    result = C0 * sh[..., 0]
    if degree > 0:
        x, y, z = dirs[..., 0:1], dirs[..., 1:2], dirs[..., 2:3]
        result = result - C1 * y * sh[..., 1] + C1 * z * sh[..., 2] - C1 * x * sh[..., 3]
        if degree > 1:
            xx, yy, zz = x * x, y * y, z * z
            xy, yz, xz = x * y, y * z, x * z
            result = (result + C2[0] * xy * sh[..., 4] + C2[1] * yz * sh[..., 5]
                      + C2[2] * (2.0 * zz - xx - yy) * sh[..., 6]
                      + C2[3] * xz * sh[..., 7] + C2[4] * (xx - yy) * sh[..., 8])
            if degree > 2:
                result = (result + C3[0] * y * (3 * xx - yy) * sh[..., 9]
                          + C3[1] * xy * z * sh[..., 10]
                          + C3[2] * y * (4 * zz - xx - yy) * sh[..., 11]
                          + C3[3] * z * (2 * zz - 3 * xx - 3 * yy) * sh[..., 12]
                          + C3[4] * x * (4 * zz - xx - yy) * sh[..., 13]
                          + C3[5] * z * (xx - yy) * sh[..., 14]
                          + C3[6] * x * (xx - 3 * yy) * sh[..., 15])
    return result


class CpuGaussianStep:
    """One training step of the per-Gaussian parameters on the CPU."""

    def __init__(self, n: int, seed: int = 42, degree: int = 3, activations: bool = True):
        g = torch.Generator().manual_seed(seed)
        self.degree = degree
        self.means = torch.nn.Parameter(torch.rand((n, 3), generator=g) * 2 - 1)
        self.camera = torch.tensor([0.0, 0.0, -4.0])
        self.dc = torch.nn.Parameter(torch.randn((n, 1, 3), generator=g) * 0.1 + 0.5)
        self.rest = torch.nn.Parameter(torch.randn((n, 15, 3), generator=g) * 0.05)
        self.color_seed = torch.randn((n, 3), generator=g) * 1e-3
        # The position only receives its adjoint (dm); its Adam step is not part
        # of the consumed path.
        groups = [dict(params=[self.dc], lr=0.0025), dict(params=[self.rest], lr=0.000125)]
        self.activations = activations
        if activations:
            self.rotation = torch.nn.Parameter(torch.randn((n, 4), generator=g))
            self.scaling = torch.nn.Parameter(torch.rand((n, 3), generator=g) * 4 - 6)
            self.opacity = torch.nn.Parameter(torch.randn((n, 1), generator=g) - 2)
            self.act_seeds = [torch.randn((n, w), generator=g) * 1e-4 for w in (4, 3, 1)]
            groups += [dict(params=[self.rotation], lr=0.001),
                       dict(params=[self.scaling], lr=0.005),
                       dict(params=[self.opacity], lr=0.025)]
        self.optimizer = torch.optim.Adam(groups, betas=(0.9, 0.999), eps=1e-15)
        self.n = n

    def step(self) -> None:
        self.optimizer.zero_grad(set_to_none=True)
        shs = torch.cat((self.dc, self.rest), 1).transpose(1, 2)  # [n, 3, 16]
        dirs = self.means - self.camera
        dirs = dirs / dirs.norm(dim=1, keepdim=True)
        colors = torch.clamp_min(eval_sh(self.degree, shs, dirs) + 0.5, 0.0)
        loss = (colors * self.color_seed).sum()
        if self.activations:
            outputs = (torch.nn.functional.normalize(self.rotation, dim=1, eps=1e-12),
                       self.scaling.exp(), self.opacity.sigmoid())
            loss = loss + sum((o * s).sum() for o, s in zip(outputs, self.act_seeds))
        loss.backward()
        self.optimizer.step()


def time_cpu_path(n: int, steps: int, warmup: int = 1, threads: int | None = None,
                  activations: bool = True) -> dict:
    """Runs `steps` timed CPU steps on n Gaussians; returns Gaussians/s etc."""
    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    model = CpuGaussianStep(n, activations=activations)
    for _ in range(warmup):
        model.step()
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        model.step()
        times.append(time.perf_counter() - t0)
    total = sum(times)
    times.sort()
    return dict(gaussians_per_s=n * steps / total, median_s=times[len(times) // 2],
                total_s=total, n=n, steps=steps, threads=torch.get_num_threads())
