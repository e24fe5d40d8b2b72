"""Rotation, scaling and opacity updated inside their activation backward (the
trainer-facing `activation` module; same public names, arguments and reason
strings as the reference's activation.py:1-249).

`DenseActivationConsumer.bind(model, policy, exclusive_use=True)` returns the
activated (normalised rotation, exp scaling, sigmoid opacity) for the
renderer, or None when the step keeps torch's path (`last_reason` says why).
The three output adjoints of that call go to the fused CUDA kernel
(clad_quaternion.consume_activations), which applies the normalise / exp /
sigmoid VJPs and torch-fused Adam to the raw parameters and their moments in
place. The step then settles the claims: counters +1, autograd versions
bumped once, `.grad` left None so `optimizer.step()` skips the three groups.
"""

from __future__ import annotations

import torch

from optimizer_claims import (ADAM_OPTIONS, STATE_KEYS, Claim, bias_corrections,
                              dense_fp32_cuda, finite_rate, first_failure, overlapping,
                              owns_only, plain_fused_adam, read_counters, reference_betas,
                              settle, sole_group, state_or_fresh, state_problem, valid_counter)

NAMES = ("rotation", "scaling", "opacity")
ATTRS = ("_rotation", "_scaling", "_opacity")
OPTIONS = ADAM_OPTIONS
WIDTHS = (4, 3, 1)


class _ConsumeActivations(torch.autograd.Function):
    """Forward: the three activations, with what their VJPs need saved.
    Backward: the fused VJP + Adam launch; returns no gradients."""

    @staticmethod
    def forward(ctx, rotation, scaling, opacity, frame):
        norm = rotation.norm(2, dim=1, keepdim=True)
        exp_scale = scaling.exp()
        sig_opacity = opacity.sigmoid()
        ctx.save_for_backward(rotation, scaling, opacity, norm, exp_scale, sig_opacity)
        ctx.frame = frame
        ctx.set_materialize_grads(False)
        unit = rotation / norm.clamp_min(1e-12).expand_as(rotation)
        return unit, exp_scale, sig_opacity

    @staticmethod
    def backward(ctx, *seeds):
        frame = ctx.frame
        if frame.consumed or torch.is_grad_enabled():
            raise RuntimeError("Activation consumption requires one first-order backward")
        if any(s is None for s in seeds):
            raise RuntimeError("Activation consumption requires all three output adjoints")
        rotation, scaling, opacity, norm, exp_scale, sig_opacity = ctx.saved_tensors
        frame.validate_live()
        claims = frame.claims
        frame.extension.consume_activations(
            [rotation, scaling, opacity], list(seeds), [norm, exp_scale, sig_opacity],
            [c.moments[0] for c in claims], [c.moments[1] for c in claims],
            frame.rates, frame.bias1, frame.bias2)
        settle(claims)
        frame.consumed = True
        return None, None, None, None


def _unusable(group, raw, rows, width, device):
    return not (owns_only(group, raw) and raw.grad is None and raw.requires_grad
                and raw.ndim == 2 and dense_fp32_cuda(raw, (rows, width))
                and raw.device == device)


# Per-group screening, first failure raises (rows of (message, predicate)).
_GROUP_RULES = (
    ("Unsupported activation ownership or layout", _unusable),
    ("Unsupported activation optimizer options",
     lambda g, raw, rows, width, device: not (reference_betas(g) and plain_fused_adam(g))),
    ("unsupported activation learning rate",
     lambda g, raw, rows, width, device: not finite_rate(g["lr"]) or g["lr"] < 0),
)


class _ActivationStep:
    """The claims of one consumed activation step (raises ValueError, with the
    fallback reason as its message, when the model cannot be consumed)."""

    def __init__(self, model, extension):
        self.model, self.optimizer, self.extension = model, model.optimizer, extension
        if type(self.optimizer) is not torch.optim.Adam:
            raise ValueError("unsupported optimizer")
        self.parameters = [getattr(model, attr) for attr in ATTRS]
        rows, device = self.parameters[0].shape[0], self.parameters[0].device
        self.claims = []
        for name, raw, width in zip(NAMES, self.parameters, WIDTHS):
            group = sole_group(self.optimizer, name)
            if group is None:
                raise ValueError("Expected one optimizer group for " + name)
            failure = first_failure(_GROUP_RULES, group, raw, rows, width, device)
            if failure is not None:
                raise ValueError(failure)
            state = state_or_fresh(self.optimizer, raw, raw.device)
            problem = state_problem(state, raw)
            if problem is not None:
                raise ValueError("Unsupported activation moment layout" if problem == "moments"
                                 else "Unsupported activation counter")
            self.claims.append(Claim.take(group, state))
        if overlapping(self.parameters + [c.state[k] for c in self.claims for k in STATE_KEYS]):
            raise ValueError("overlapping activation parameters or moments")
        counters = read_counters([c.state for c in self.claims])
        if not all(valid_counter(c) for c in counters):
            raise ValueError("Invalid activation counters")
        for claim in self.claims:
            self.optimizer.state[claim.param] = claim.state
        self.rates = [c.group["lr"] for c in self.claims]
        corrections = [bias_corrections(int(c) + 1) for c in counters]
        self.bias1 = [b1 for b1, _ in corrections]
        self.bias2 = [b2 for _, b2 in corrections]
        self.consumed = False

    @property
    def groups(self):
        return [c.group for c in self.claims]

    @property
    def states(self):
        return [c.state for c in self.claims]

    def validate_live(self):
        if self.model.optimizer is not self.optimizer:
            raise RuntimeError("Activation optimizer was replaced")
        same_tensors = all(getattr(self.model, a) is p for a, p in zip(ATTRS, self.parameters))
        if not (same_tensors and all(c.intact(self.optimizer) for c in self.claims)):
            raise RuntimeError("Activation ownership changed after forward")


class DenseActivationConsumer:
    # Caller-declared conditions that keep torch's path, checked in order once
    # gradients are enabled.
    _DECLARED = (
        ("activation parameters have other consumers", lambda ex, gp, ho: not ex),
        ("activation gradients require native processing", lambda ex, gp, ho: gp),
        ("higher-order derivatives require native backward", lambda ex, gp, ho: ho),
    )

    def __init__(self, extension):
        if not hasattr(extension, "consume_activations"):
            raise ValueError("Build the combined activation consumer first")
        self.extension = extension
        self.active = None
        self.last_reason = None

    def bind(self, model, policy, *, exclusive_use=False, gradient_processing=False,
             higher_order=False):
        if not torch.is_grad_enabled():
            reason = "evaluation without gradients"
        else:
            reason = first_failure(self._DECLARED, exclusive_use, gradient_processing,
                                   higher_order)
        if reason is None:
            reason = "consumption disabled" if policy is None else policy.reason()
        if reason is not None:
            self.last_reason = reason
            return None
        if self.active is not None:
            raise RuntimeError("finish the previous activation step first")
        try:
            frame = _ActivationStep(model, self.extension)
        except (ValueError, KeyError, TypeError, AttributeError) as error:
            self.last_reason = str(error)
            return None
        self.active, self.last_reason = frame, None
        return _ConsumeActivations.apply(*frame.parameters, frame)

    def end_step(self):
        if self.active is not None and not self.active.consumed:
            raise RuntimeError("activation frame has no completed backward")
        self.active = None
