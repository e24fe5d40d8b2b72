"""Dense-Adam SH consumer bound to the trainer's optimizer for one step
(drop-in for the reference's adapter.py:1-389).

On an eligible step `DenseSHConsumer.render` binds features_dc /
features_rest, their Adam moments and step counters (`bind`), renders through
the rasterizer extension, and in backward calls the extension's
`rasterize_gaussians_backward_consume[_direct]`, which runs the pixel and
geometry backward and then the fused SH VJP + torch-fused Adam kernel
(sh_consumer_split_torch_adam): the SH coefficients and moments are updated
in place, no SH gradient tensor exists, and the position adjoint of the view
direction is added to dL/dmeans. The frame then advances both step counters
and the autograd versions once and leaves `.grad` unset so the trainer's
optimizer.step() skips the two SH groups. Ineligible steps return the native
rasterizer's output and record the reason in `last_reason`; any change of
ownership between forward and backward raises before a write.

The cached state is nothing: every step binds the optimizer's current
objects, so checkpoint restore, densification and pruning need no hook.

`consume_position=True` (not in the reference, whose trainer leaves xyz to
torch's Adam) also binds the optimizer's "xyz" group: once the direction
adjoint is added dL/dmeans is the positions' complete gradient, so the same
kernel runs their Adam, the backward returns no position gradient, and the
frame advances the xyz counter with the SH ones. Only valid when the means feed
nothing but this renderer; an ineligible xyz group leaves the positions to the
optimizer (`position_reason` says why) and the SH groups are still consumed.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from types import SimpleNamespace

import torch

SH_OPTIONS = ("lr", "betas", "eps", "fused", "foreach", "weight_decay",
              "amsgrad", "maximize", "capturable", "differentiable")
STATE_KEYS = ("exp_avg", "exp_avg_sq", "step")


def _forward_arguments(settings, means, opacity, scale, rotation, sh, empty):
    return (settings.bg, means, empty, opacity, scale, rotation,
            settings.scale_modifier, empty, settings.viewmatrix, settings.projmatrix,
            settings.tanfovx, settings.tanfovy, settings.image_height,
            settings.image_width, sh, settings.sh_degree, settings.campos,
            settings.prefiltered, settings.antialiasing, settings.debug)


class ConsumerRender(torch.autograd.Function):
    """Rasterizer call whose backward consumes the SH gradient (adapter.py:13-119)."""

    @staticmethod
    def forward(ctx, means, screen, dc, rest, opacity, scale, rotation, settings, owner):
        empty = torch.empty(0, device=means.device)
        direct = getattr(owner, "direct_inputs", False)
        sh = empty if direct else torch.cat((dc, rest), 1)
        args = _forward_arguments(settings, means, opacity, scale, rotation, sh, empty)
        if direct:
            args = args[:14] + (dc, rest) + args[15:]
            count, color, radii, geom, binning, image, depth = \
                owner.extension.rasterize_gaussians_direct(*args)
        else:
            count, color, radii, geom, binning, image, depth = \
                owner.extension.rasterize_gaussians(*args)
        ctx.settings, ctx.owner, ctx.count = settings, owner, count
        ctx.save_for_backward(means, opacity, scale, rotation, radii, sh, geom,
                              binning, image, dc, rest)
        return color, radii, depth

    @staticmethod
    def backward(ctx, seed, _radii_seed, depth_seed):
        owner = ctx.owner
        native_only = getattr(owner, "native_only", False)
        if native_only and torch.is_grad_enabled():
            raise RuntimeError("Direct SH inputs support first-order backward only")
        (means, opacity, scale, rotation, radii, sh, geom, binning, image, dc,
         rest) = ctx.saved_tensors
        s = ctx.settings
        empty = torch.empty(0, device=means.device)
        args = (s.bg, means, radii, empty, opacity, scale, rotation, s.scale_modifier,
                empty, s.viewmatrix, s.projmatrix, s.tanfovx, s.tanfovy,
                seed.contiguous(), depth_seed.contiguous(), sh, s.sh_degree, s.campos,
                geom, ctx.count, binning, image, s.antialiasing, s.debug)
        if native_only:
            grads = owner.extension.rasterize_gaussians_backward_direct(
                *(args[:15] + (dc, rest) + args[16:]))
            g_screen, _, g_opacity, g_means, _, g_sh, g_scale, g_rot = grads
            return (g_means, g_screen, g_sh[:, :1], g_sh[:, 1:], g_opacity, g_scale,
                    g_rot, None, None)
        m_dc, v_dc = owner.moments["dc"]
        m_rest, v_rest = owner.moments["rest"]
        step = owner.iteration
        bias1, bias2 = 1 - 0.9 ** step, math.sqrt(1 - 0.999 ** step)
        consume = (owner.extension.rasterize_gaussians_backward_consume_direct
                   if getattr(owner, "direct_inputs", False)
                   else owner.extension.rasterize_gaussians_backward_consume)
        extra = {}
        position = "xyz" in owner.params
        if position:
            m_xyz, v_xyz = owner.moments["xyz"]
            extra["xyz"] = dict(first=m_xyz, second=v_xyz, rate=owner.position_rate,
                                bias1=bias1, bias2_sqrt=bias2)
        grads = consume(*args, owner.params["dc"], owner.params["rest"], m_dc, v_dc,
                        m_rest, v_rest, bias1, bias2, **extra)
        g_screen, _, g_opacity, g_means, _, _, g_scale, g_rot = grads
        if position:
            g_means = None  # applied by the kernel
        return g_means, g_screen, None, None, g_opacity, g_scale, g_rot, None, None


def render_direct_native(extension, means, screen, dc, rest, opacity, scale, rotation,
                         settings):
    """Direct dc/rest reads with the ordinary SH backward (gradients for the
    trainer's own optimizer)."""
    owner = SimpleNamespace(extension=extension, direct_inputs=True, native_only=True)
    return ConsumerRender.apply(means, screen, dc, rest, opacity, scale, rotation,
                                settings, owner)


@dataclass(frozen=True)
class StepPolicy:
    """What the trainer does between backward and Adam on this step."""

    optimizer_step: bool = True
    topology_change: bool = False
    observation_before_step: bool = False
    single_backward: bool = True
    unscaled_gradients: bool = True
    exclusive_sh_use: bool = True

    def reason(self):
        if not self.optimizer_step:
            return "optimizer step skipped"
        if self.topology_change:
            return "topology changes before optimizer step"
        if self.observation_before_step:
            return "parameters observed before optimizer step"
        if not self.single_backward:
            return "gradient accumulation or multiple backward calls"
        if not self.unscaled_gradients:
            return "scaled gradients require native optimizer processing"
        if not self.exclusive_sh_use:
            return "SH parameters used by another loss or consumer"
        return None


class BoundStep:
    """The SH parameters, groups and Adam state of one consumed step."""

    def __init__(self, optimizer, groups, states, extension, iteration):
        self.optimizer = optimizer
        self.groups = groups
        self.states = states
        self.extension = extension
        keys = ("dc", "rest", "xyz")[:len(groups)]
        self.params = {k: g["params"][0] for k, g in zip(keys, groups)}
        self.moments = {k: (st["exp_avg"], st["exp_avg_sq"]) for k, st in zip(keys, states)}
        self.position_rate = float(groups[2]["lr"]) if len(groups) > 2 else None
        self.iteration = iteration
        self.consumed = False
        self.versions = [p._version for p in self.params.values()]
        self.options = [tuple(g.get(k) for k in SH_OPTIONS) for g in groups]
        self.values = [{k: st[k] for k in STATE_KEYS} for st in states]
        self.state_versions = [{k: v._version for k, v in row.items()} for row in self.values]

    def validate(self):
        if self.consumed:
            raise RuntimeError("SH consumption permits one backward per optimizer step")
        for group, p, version, state, values, state_versions, options in zip(
                self.groups, self.params.values(), self.versions, self.states,
                self.values, self.state_versions, self.options):
            if (len(group["params"]) != 1 or group["params"][0] is not p
                    or p._version != version or p.grad is not None or not p.requires_grad
                    or not any(g is group for g in self.optimizer.param_groups)
                    or self.optimizer.state.get(p) is not state
                    or any(state.get(k) is not v for k, v in values.items())
                    or any(values[k]._version != v for k, v in state_versions.items())
                    or tuple(group.get(k) for k in SH_OPTIONS) != options):
                raise RuntimeError("SH ownership changed between forward and backward")

    @torch.no_grad()
    def finish(self):
        for state in self.states:
            state["step"].add_(1)
        torch.autograd.graph.increment_version(
            [*self.params.values(), *[v for pair in self.moments.values() for v in pair]])
        self.consumed = True


class LifecycleRender(ConsumerRender):
    @staticmethod
    def backward(ctx, seed, radii_seed, depth_seed):
        if torch.is_grad_enabled():
            raise RuntimeError("SH consumption supports first-order backward only")
        ctx.owner.validate()
        result = ConsumerRender.backward(ctx, seed, radii_seed, depth_seed)
        ctx.owner.finish()
        return result


class DenseSHConsumer:
    def __init__(self, optimizer, *, native, extension, direct_inputs=False,
                 consume_position=False):
        if direct_inputs and not all(
                hasattr(extension, name) for name in
                ("rasterize_gaussians_direct", "rasterize_gaussians_backward_consume_direct")):
            raise ValueError("Build the extension with direct-input support first")
        self.native = native
        self.extension = extension
        self.direct_inputs = direct_inputs
        self.optimizer = optimizer
        self.consume_position = consume_position
        self.active = None
        self.last_reason = None
        self.position_reason = None

    def _fallback(self, reason):
        self.last_reason = reason
        return None

    @staticmethod
    def _group_reason(group, param, shape, what):
        """Why `group` cannot be consumed (None if it can); the rate is checked
        by the caller."""
        if len(group["params"]) != 1 or group["params"][0] is not param:
            return f"{what} parameter ownership mismatch"
        if (tuple(param.shape) != shape or not param.is_contiguous()
                or param.dtype != torch.float32 or not param.is_cuda):
            return f"unsupported {what} tensor layout"
        if not param.requires_grad or param.grad is not None:
            return f"frozen or accumulated {what} gradients"
        if group["betas"] != (0.9, 0.999) or group["eps"] != 1e-15:
            return f"unsupported {what} Adam hyperparameters"
        if group.get("fused") is not True or group.get("foreach"):
            return f"{what} consumption requires fused Adam without foreach"
        if (any(group.get(k, False) for k in
                ("amsgrad", "maximize", "differentiable", "capturable"))
                or group.get("weight_decay", 0) != 0):
            return "unsupported Adam option"
        return None

    @staticmethod
    def _state_for(optimizer, group):
        param = group["params"][0]
        state = optimizer.state.get(param)
        if not state:
            state = {"step": torch.tensor(0.0, device=param.device if group.get("fused")
                                          else "cpu"),
                     "exp_avg": torch.zeros_like(param),
                     "exp_avg_sq": torch.zeros_like(param)}
        for key in ("exp_avg", "exp_avg_sq"):
            value = state.get(key)
            if (not torch.is_tensor(value) or value.shape != param.shape
                    or value.dtype != param.dtype or value.device != param.device
                    or not value.is_contiguous()):
                return None, "moment layout"
        step = state.get("step")
        if (not torch.is_tensor(step) or step.device != param.device
                or step.dtype != torch.float32 or step.numel() != 1):
            return None, "step counter"
        return state, None

    def _position_group(self, means, count, device):
        """The xyz group and its state, or (None, reason)."""
        if means is None:
            return None, None, "positions not given"
        matches = [g for g in self.optimizer.param_groups if g.get("name") == "xyz"]
        if len(matches) != 1:
            return None, None, "missing or duplicate xyz optimizer group"
        group = matches[0]
        reason = self._group_reason(group, means, (count, 3), "position")
        rate = group.get("lr")
        if reason is None and (not isinstance(rate, (float, int)) or not math.isfinite(rate)):
            reason = "unsupported position learning rate"
        if reason is None and means.device != device:
            reason = "position device mismatch"
        if reason is not None:
            return None, None, reason
        state, bad = self._state_for(self.optimizer, group)
        if state is None:
            return None, None, f"unsupported position {bad}"
        return group, state, None

    def bind(self, dc, rest, policy, means=None):
        if self.active is not None:
            raise RuntimeError("finish the previous optimizer step first")
        reason = policy.reason()
        if not torch.is_grad_enabled():
            reason = "evaluation without gradients"
        if torch.cuda.current_stream() != torch.cuda.default_stream():
            raise RuntimeError("the pinned rasterizer requires the default CUDA stream")
        if type(self.optimizer) is not torch.optim.Adam:
            reason = "unsupported optimizer"
        if reason is not None:
            return self._fallback(reason)
        if dc.ndim != 3 or rest.ndim != 3:
            return self._fallback("unsupported SH tensor layout")
        groups = []
        for name, param, shape, rate in (("f_dc", dc, (dc.shape[0], 1, 3), 0.0025),
                                         ("f_rest", rest, (dc.shape[0], 15, 3), 0.000125)):
            matches = [g for g in self.optimizer.param_groups if g.get("name") == name]
            if len(matches) != 1:
                reason = "missing or duplicate SH optimizer group"
                break
            group = matches[0]
            groups.append(group)
            if len(group["params"]) != 1 or group["params"][0] is not param:
                reason = "SH parameter ownership mismatch"
            if (tuple(param.shape) != shape or not param.is_contiguous()
                    or param.dtype != torch.float32 or not param.is_cuda):
                reason = "unsupported SH tensor layout"
            if not param.requires_grad or param.grad is not None:
                reason = "frozen or accumulated SH gradients"
            if (not isinstance(group["lr"], (float, int)) or group["lr"] != rate
                    or group["betas"] != (0.9, 0.999) or group["eps"] != 1e-15):
                reason = "unsupported SH Adam hyperparameters"
            if group.get("fused") is not True or group.get("foreach"):
                reason = "SH consumption requires fused Adam without foreach"
            if (any(group.get(k, False) for k in
                    ("amsgrad", "maximize", "differentiable", "capturable"))
                    or group.get("weight_decay", 0) != 0):
                reason = "unsupported Adam option"
        if dc.device != rest.device:
            reason = "SH device mismatch"
        if reason is not None:
            return self._fallback(reason)
        states = []
        for group in groups:
            param = group["params"][0]
            state = self.optimizer.state.get(param)
            if not state:
                state = {"step": torch.tensor(0.0, device=param.device if group.get("fused")
                                              else "cpu"),
                         "exp_avg": torch.zeros_like(param),
                         "exp_avg_sq": torch.zeros_like(param)}
            for key in ("exp_avg", "exp_avg_sq"):
                value = state.get(key)
                if (not torch.is_tensor(value) or value.shape != param.shape
                        or value.dtype != param.dtype or value.device != param.device
                        or not value.is_contiguous()):
                    return self._fallback("unsupported SH moment layout")
            step = state.get("step")
            if (not torch.is_tensor(step) or step.device != param.device
                    or step.dtype != torch.float32 or step.numel() != 1):
                return self._fallback("unsupported SH step counter")
            states.append(state)
        writable = [dc, rest] + [st[k] for st in states for k in STATE_KEYS]
        spans = sorted((v.data_ptr(), v.data_ptr() + v.numel() * v.element_size())
                       for v in writable if v.numel())
        if any(a[1] > b[0] for a, b in zip(spans, spans[1:])):
            return self._fallback("overlapping SH parameters, moments or counters")
        counters = [st["step"].item() for st in states]
        if any(not math.isfinite(c) or c < 0 or c != int(c) or c >= 2**24 for c in counters):
            return self._fallback("invalid SH step counter")
        if counters[0] != counters[1]:
            return self._fallback("different SH Adam step counters")
        self.position_reason = None
        if self.consume_position:
            group, state, why = self._position_group(means, dc.shape[0], dc.device)
            if why is None and state["step"].item() != counters[0]:
                why = "position and SH Adam step counters differ"
            if why is None:
                extra = [means] + [state[k] for k in STATE_KEYS]
                spans = sorted((v.data_ptr(), v.data_ptr() + v.numel() * v.element_size())
                               for v in writable + extra if v.numel())
                if any(a[1] > b[0] for a, b in zip(spans, spans[1:])):
                    why = "positions overlap the SH parameters or moments"
            if why is None:
                groups.append(group)
                states.append(state)
            self.position_reason = why
        for group, state in zip(groups, states):
            self.optimizer.state[group["params"][0]] = state
        self.active = BoundStep(self.optimizer, groups, states, self.extension,
                                int(counters[0]) + 1)
        self.active.direct_inputs = self.direct_inputs
        self.last_reason = None
        return self.active

    def render(self, means, screen, dc, rest, opacity, scale, rotation, settings, policy):
        owner = self.bind(dc, rest, policy, means)
        if owner is not None:
            return LifecycleRender.apply(means, screen, dc, rest, opacity, scale, rotation,
                                         settings, owner)
        return self.native.GaussianRasterizer(settings)(
            means3D=means, means2D=screen, opacities=opacity,
            shs=torch.cat((dc, rest), 1), scales=scale, rotations=rotation)

    def end_step(self):
        if self.active is not None and not self.active.consumed:
            raise RuntimeError("consumer frame has no completed backward")
        self.active = None


def official_step_policy(iteration, options, *, white_background=False,
                         testing_iterations=(), saving_iterations=()):
    """The trainer's steps that change state between backward and Adam
    (densification, opacity reset, save/test, final iteration) fall back."""
    topology = False
    if iteration < options.densify_until_iter:
        topology = (iteration > options.densify_from_iter
                    and iteration % options.densification_interval == 0)
        topology = topology or iteration % options.opacity_reset_interval == 0
        topology = topology or (white_background and iteration == options.densify_from_iter)
    return StepPolicy(
        optimizer_step=iteration < options.iterations,
        topology_change=topology,
        observation_before_step=iteration in testing_iterations or iteration in saving_iterations)
