"""SH coefficients updated inside the rasterizer backward (the trainer-facing
`adapter` module; same public names, arguments and fallback reasons as the
reference's adapter.py:1-389).

`DenseSHConsumer.render(...)` is the trainer's render call. On a step the
policy allows, it claims the optimizer's f_dc / f_rest groups (their Adam
moments and counters) and renders through `LifecycleRender`, whose backward
calls the extension's `rasterize_gaussians_backward_consume[_direct]`: the
pixel and geometry backward run, then one fused kernel applies the SH
adjoint straight to torch-fused Adam on the coefficients and adds the view
direction's adjoint to dL/dmeans. No SH gradient tensor exists; the groups'
`.grad` stays None, so the trainer's `optimizer.step()` skips them, and the
counters and autograd versions advance once. Any other step renders through
the native rasterizer and records why in `last_reason`. A claim is checked
again right before the kernel: any change of ownership raises before a write.
Nothing is cached across steps, so checkpoint restore, densification and
pruning need no hook.

`consume_position=True` (an addition; the reference leaves xyz to torch's
Adam) also claims the "xyz" group: once the direction adjoint is added,
dL/dmeans is complete, so the same kernel applies the positions' Adam and the
backward returns no position gradient. An xyz group that cannot be claimed
leaves the positions to the optimizer (`position_reason` says why) without
affecting the SH groups.
"""

from __future__ import annotations

from dataclasses import dataclass, fields
from types import SimpleNamespace

import torch

from optimizer_claims import (ADAM_OPTIONS, STATE_KEYS, Claim, bias_corrections,
                              dense_fp32_cuda, finite_rate, last_failure, overlapping,
                              owns_only, read_counters, reference_betas,
                              settle, sole_group, state_or_fresh, state_problem, valid_counter)

SH_OPTIONS = ADAM_OPTIONS

# Positional layouts of the renderer extension's calls (the reference's
# adapter.py:21-47, 67-92): names of the values in call order. In the direct
# variants the packed "sh" slot is replaced by the two tensors dc, rest.
FORWARD_ARGS = ("bg", "means", "colors", "opacity", "scales", "rotations", "scale_modifier",
                "cov3d", "viewmatrix", "projmatrix", "tanfovx", "tanfovy", "image_height",
                "image_width", "sh", "sh_degree", "campos", "prefiltered", "antialiasing",
                "debug")
BACKWARD_ARGS = ("bg", "means", "radii", "colors", "opacity", "scales", "rotations",
                 "scale_modifier", "cov3d", "viewmatrix", "projmatrix", "tanfovx", "tanfovy",
                 "dout_color", "dout_invdepth", "sh", "sh_degree", "campos", "geom",
                 "num_rendered", "binning", "image", "antialiasing", "debug")
_SETTINGS = ("bg", "scale_modifier", "viewmatrix", "projmatrix", "tanfovx", "tanfovy",
             "image_height", "image_width", "sh_degree", "campos", "prefiltered",
             "antialiasing", "debug")


def _call_args(layout, values, split_sh):
    """Values in the extension's positional order; `split_sh` puts (dc, rest)
    where the packed coefficients would go."""
    out = []
    for name in layout:
        if name == "sh" and split_sh:
            out += [values["dc"], values["rest"]]
        else:
            out.append(values[name])
    return tuple(out)


def _settings_values(settings):
    return {name: getattr(settings, name) for name in _SETTINGS}


class ConsumerRender(torch.autograd.Function):
    """Renderer call whose backward hands the SH adjoint to the fused Adam
    kernel instead of returning it (the reference's adapter.py:13-119)."""

    @staticmethod
    def forward(ctx, means, screen, dc, rest, opacity, scale, rotation, settings, owner):
        empty = torch.empty(0, device=means.device)
        split = bool(getattr(owner, "direct_inputs", False))
        packed = empty if split else torch.cat((dc, rest), 1)
        values = dict(_settings_values(settings), means=means, colors=empty, opacity=opacity,
                      scales=scale, rotations=rotation, cov3d=empty, sh=packed, dc=dc,
                      rest=rest)
        render = (owner.extension.rasterize_gaussians_direct if split
                  else owner.extension.rasterize_gaussians)
        count, color, radii, geom, binning, image, depth = render(
            *_call_args(FORWARD_ARGS, values, split))
        ctx.settings, ctx.owner, ctx.count = settings, owner, count
        ctx.save_for_backward(means, opacity, scale, rotation, radii, packed, geom, binning,
                              image, dc, rest)
        return color, radii, depth

    @staticmethod
    def backward(ctx, seed, _radii_seed, depth_seed):
        owner = ctx.owner
        unconsumed = bool(getattr(owner, "native_only", False))
        if unconsumed and torch.is_grad_enabled():
            raise RuntimeError("Direct SH inputs support first-order backward only")
        (means, opacity, scale, rotation, radii, packed, geom, binning, image, dc,
         rest) = ctx.saved_tensors
        empty = torch.empty(0, device=means.device)
        values = dict(_settings_values(ctx.settings), means=means, radii=radii, colors=empty,
                      opacity=opacity, scales=scale, rotations=rotation, cov3d=empty,
                      dout_color=seed.contiguous(), dout_invdepth=depth_seed.contiguous(),
                      sh=packed, dc=dc, rest=rest, geom=geom, num_rendered=ctx.count,
                      binning=binning, image=image)
        if unconsumed:
            out = owner.extension.rasterize_gaussians_backward_direct(
                *_call_args(BACKWARD_ARGS, values, True))
            d_screen, _, d_opacity, d_means, _, d_sh, d_scale, d_rot = out
            return (d_means, d_screen, d_sh[:, :1], d_sh[:, 1:], d_opacity, d_scale, d_rot,
                    None, None)
        split = bool(getattr(owner, "direct_inputs", False))
        consume = (owner.extension.rasterize_gaussians_backward_consume_direct if split
                   else owner.extension.rasterize_gaussians_backward_consume)
        bias1, bias2 = bias_corrections(owner.iteration)
        (m_dc, v_dc), (m_rest, v_rest) = owner.moments["dc"], owner.moments["rest"]
        position = {}
        if "xyz" in owner.params:
            m_xyz, v_xyz = owner.moments["xyz"]
            position["xyz"] = dict(first=m_xyz, second=v_xyz, rate=owner.position_rate,
                                   bias1=bias1, bias2_sqrt=bias2)
        out = consume(*_call_args(BACKWARD_ARGS, values, split), owner.params["dc"],
                      owner.params["rest"], m_dc, v_dc, m_rest, v_rest, bias1, bias2,
                      **position)
        d_screen, _, d_opacity, d_means, _, _, d_scale, d_rot = out
        if position:
            d_means = None  # the kernel already applied the positions' Adam
        return d_means, d_screen, None, None, d_opacity, d_scale, d_rot, None, None


def render_direct_native(extension, means, screen, dc, rest, opacity, scale, rotation,
                         settings):
    """Render from dc/rest directly and return ordinary SH gradients for the
    trainer's own optimizer."""
    owner = SimpleNamespace(extension=extension, direct_inputs=True, native_only=True)
    return ConsumerRender.apply(means, screen, dc, rest, opacity, scale, rotation, settings,
                                owner)


@dataclass(frozen=True)
class StepPolicy:
    """What the trainer does between this step's backward and its Adam step.
    Any field away from its default makes the step ineligible."""

    optimizer_step: bool = True
    topology_change: bool = False
    observation_before_step: bool = False
    single_backward: bool = True
    unscaled_gradients: bool = True
    exclusive_sh_use: bool = True

    _REASONS = {
        "optimizer_step": "optimizer step skipped",
        "topology_change": "topology changes before optimizer step",
        "observation_before_step": "parameters observed before optimizer step",
        "single_backward": "gradient accumulation or multiple backward calls",
        "unscaled_gradients": "scaled gradients require native optimizer processing",
        "exclusive_sh_use": "SH parameters used by another loss or consumer",
    }

    def reason(self):
        for f in fields(self):
            if bool(getattr(self, f.name)) != f.default:
                return self._REASONS[f.name]
        return None


class BoundStep:
    """The claims of one consumed step; `validate` right before the kernel,
    `finish` after it."""

    def __init__(self, optimizer, claims, extension, iteration):
        self.optimizer = optimizer
        self.claims = dict(claims)          # "dc", "rest"[, "xyz"] -> Claim
        self.extension = extension
        self.iteration = iteration
        self.consumed = False
        self.direct_inputs = False
        xyz = self.claims.get("xyz")
        self.position_rate = float(xyz.group["lr"]) if xyz is not None else None

    @property
    def groups(self):
        return [c.group for c in self.claims.values()]

    @property
    def states(self):
        return [c.state for c in self.claims.values()]

    @property
    def params(self):
        return {k: c.param for k, c in self.claims.items()}

    @property
    def moments(self):
        return {k: c.moments for k, c in self.claims.items()}

    def validate(self):
        if self.consumed:
            raise RuntimeError("SH consumption permits one backward per optimizer step")
        if not all(c.intact(self.optimizer) for c in self.claims.values()):
            raise RuntimeError("SH ownership changed between forward and backward")

    def finish(self):
        settle(self.claims.values())
        self.consumed = True


class LifecycleRender(ConsumerRender):
    """ConsumerRender whose backward re-checks the claims before the kernel
    and settles them after it."""

    @staticmethod
    def backward(ctx, seed, radii_seed, depth_seed):
        if torch.is_grad_enabled():
            raise RuntimeError("SH consumption supports first-order backward only")
        ctx.owner.validate()
        grads = ConsumerRender.backward(ctx, seed, radii_seed, depth_seed)
        ctx.owner.finish()
        return grads


# Per-group screening of an SH or position group: (reason, predicate(group,
# param, shape, what)), general to specific; the last failing row names the
# fallback, which is how the reference's sequence of checks reports.
def _group_rules(what, rate_ok):
    return (
        (f"{what} parameter ownership mismatch", lambda g, p, s: not owns_only(g, p)),
        (f"unsupported {what} tensor layout", lambda g, p, s: not dense_fp32_cuda(p, s)),
        (f"frozen or accumulated {what} gradients",
         lambda g, p, s: not p.requires_grad or p.grad is not None),
        (f"unsupported {what} Adam hyperparameters",
         lambda g, p, s: not (rate_ok(g["lr"]) and reference_betas(g))),
        (f"{what} consumption requires fused Adam without foreach",
         lambda g, p, s: g.get("fused") is not True or bool(g.get("foreach"))),
        ("unsupported Adam option",
         lambda g, p, s: g.get("weight_decay", 0) != 0
         or any(g.get(k, False) for k in ("amsgrad", "maximize", "differentiable",
                                           "capturable"))),
    )


def _rate_is(value):
    return lambda lr: isinstance(lr, (float, int)) and lr == value


# (optimizer group name, claim key, coefficient rows, learning rate the
# kernel's arithmetic is checked against)
_SH_GROUPS = (("f_dc", "dc", 1, 0.0025), ("f_rest", "rest", 15, 0.000125))
_SH_RULES = {key: _group_rules("SH", _rate_is(rate)) for _, key, _, rate in _SH_GROUPS}
_POSITION_RULES = _group_rules("position", lambda lr: True)


class DenseSHConsumer:
    def __init__(self, optimizer, *, native, extension, direct_inputs=False,
                 consume_position=False):
        needed = ("rasterize_gaussians_direct", "rasterize_gaussians_backward_consume_direct")
        if direct_inputs and not all(hasattr(extension, n) for n in needed):
            raise ValueError("Build the extension with direct-input support first")
        self.native = native
        self.extension = extension
        self.direct_inputs = direct_inputs
        self.optimizer = optimizer
        self.consume_position = consume_position
        self.active = None
        self.last_reason = None
        self.position_reason = None

    # -- screening -------------------------------------------------------

    def _step_reason(self, policy):
        if torch.cuda.current_stream() != torch.cuda.default_stream():
            raise RuntimeError("the pinned rasterizer requires the default CUDA stream")
        if type(self.optimizer) is not torch.optim.Adam:
            return "unsupported optimizer"
        if not torch.is_grad_enabled():
            return "evaluation without gradients"
        return policy.reason()

    def _screen_sh(self, dc, rest):
        """(groups by claim key, reason)."""
        if dc.ndim != 3 or rest.ndim != 3:
            return None, "unsupported SH tensor layout"
        found, reason, tensors = {}, None, {"dc": dc, "rest": rest}
        for name, key, rows, _ in _SH_GROUPS:
            group = sole_group(self.optimizer, name)
            if group is None:
                reason = "missing or duplicate SH optimizer group"
                break
            found[key] = group
            reason = last_failure(_SH_RULES[key], group, tensors[key],
                                  (dc.shape[0], rows, 3)) or reason
        if dc.device != rest.device:
            reason = "SH device mismatch"
        return found, reason

    def _screen_position(self, means, count, device, sh_claims, sh_counter):
        """(group, state) of a claimable xyz group, or (None, None, reason)."""
        if means is None:
            return None, None, "positions not given"
        group = sole_group(self.optimizer, "xyz")
        if group is None:
            return None, None, "missing or duplicate xyz optimizer group"
        reason = last_failure(_POSITION_RULES, group, means, (count, 3))
        if reason is None and not finite_rate(group.get("lr")):
            reason = "unsupported position learning rate"
        if reason is None and means.device != device:
            reason = "position device mismatch"
        if reason is not None:
            return None, None, reason
        state = state_or_fresh(self.optimizer, means, means.device if group.get("fused")
                               else "cpu")
        problem = state_problem(state, means)
        if problem is not None:
            return None, None, ("unsupported position moment layout" if problem == "moments"
                                else "unsupported position step counter")
        if read_counters([state])[0] != sh_counter:
            return None, None, "position and SH Adam step counters differ"
        owned = [t for c in sh_claims for t in (c.param, *c.entries.values())]
        if overlapping(owned + [means] + [state[k] for k in STATE_KEYS]):
            return None, None, "positions overlap the SH parameters or moments"
        return group, state, None

    def _decline(self, reason):
        self.last_reason = reason
        return None

    # -- binding ---------------------------------------------------------

    def bind(self, dc, rest, policy, means=None):
        if self.active is not None:
            raise RuntimeError("finish the previous optimizer step first")
        reason = self._step_reason(policy)
        if reason is not None:
            return self._decline(reason)
        groups, reason = self._screen_sh(dc, rest)
        if reason is not None:
            return self._decline(reason)
        states = {}
        for key, group in groups.items():
            param = group["params"][0]
            state = state_or_fresh(self.optimizer, param,
                                   param.device if group.get("fused") else "cpu")
            problem = state_problem(state, param)
            if problem is not None:
                return self._decline("unsupported SH moment layout" if problem == "moments"
                                     else "unsupported SH step counter")
            states[key] = state
        written = [dc, rest] + [s[k] for s in states.values() for k in STATE_KEYS]
        if overlapping(written):
            return self._decline("overlapping SH parameters, moments or counters")
        counters = read_counters(list(states.values()))
        if not all(valid_counter(c) for c in counters):
            return self._decline("invalid SH step counter")
        if len(set(counters)) != 1:
            return self._decline("different SH Adam step counters")
        claims = {k: Claim.take(groups[k], states[k]) for k in groups}
        self.position_reason = None
        if self.consume_position:
            group, state, why = self._screen_position(means, dc.shape[0], dc.device,
                                                      claims.values(), counters[0])
            self.position_reason = why
            if why is None:
                claims["xyz"] = Claim.take(group, state)
        for claim in claims.values():
            self.optimizer.state[claim.param] = claim.state
        self.active = BoundStep(self.optimizer, claims, self.extension, int(counters[0]) + 1)
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
    """The policy of the stock trainer's loop at `iteration`: densification,
    opacity reset (and the white-background reset at densify_from_iter) change
    the Gaussian set before Adam; test and save iterations read parameters
    before it; the last iteration runs no Adam step."""
    in_window = iteration < options.densify_until_iter
    densify = iteration > options.densify_from_iter and \
        iteration % options.densification_interval == 0
    reset = iteration % options.opacity_reset_interval == 0 or \
        (white_background and iteration == options.densify_from_iter)
    observed = iteration in testing_iterations or iteration in saving_iterations
    return StepPolicy(optimizer_step=iteration < options.iterations,
                      topology_change=in_window and (densify or reset),
                      observation_before_step=observed)
