"""Trainer hooks (the trainer-facing `integration` module; same functions,
module globals and trace/summary JSON keys as the reference's
integration.py:1-219, which the patched trainer imports as clad_training and
calls from train.py and render(), trainer.patch:1-47).

Per training step:

* `begin_step` derives the step policy (`official_step_policy`) and opens the
  step's routing context and, in trace mode, its trace record;
* `activate_consumer` returns the activated (rotation, scaling, opacity) from
  the activation consumer, or None for torch's path;
* `render_consumer` renders through the SH consumer (which falls back to the
  plain rasterizer by itself);
* `after_backward` fixes the routing decision and, in trace mode, checks the
  once-only update rules after backward;
* `after_step` checks them again after the optimizer step, writes the trace
  row and closes both consumers' frames.

Globals set by the launcher: SUMMARY (a routing.RoutingSummary or None),
TRACE (path of a JSON trace; trace mode synchronises and copies parameters,
so it is for small functional runs only), DIRECT_INPUTS (render from dc/rest
without packing), ACTIVATION_EXTENSION (the clad_quaternion surface, or None
to leave activations to torch), POSITION (also consume the xyz group; an
addition of this package).
"""

from __future__ import annotations

import json
from pathlib import Path

import torch

import rasterizer as native
from activation import ATTRS, DenseActivationConsumer
from adapter import DenseSHConsumer, official_step_policy

extension = native  # the renderer-extension surface (rasterize_gaussians*, ...)

SUMMARY = None
TRACE = None
DIRECT_INPUTS = False
ACTIVATION_EXTENSION = None
POSITION = False

SKIPPED = "optimizer step skipped"


def counters(model, parameters=None):
    """Adam step counters of `parameters` (the two SH groups by default); 0 for
    a parameter without state."""
    if parameters is None:
        parameters = _sh_tensors(model)
    steps = (model.optimizer.state.get(p, {}).get("step") for p in parameters)
    return [0 if s is None else int(s.item()) for s in steps]


def _sh_tensors(model):
    return [model._features_dc, model._features_rest]


def _activation_tensors(model):
    return [getattr(model, a) for a in ATTRS]


def _trace_fail(what):
    raise AssertionError(f"trace: {what}")


class _Watch:
    """Counters and copies of one family of parameters at the stages of a step."""

    def __init__(self, model, tensors):
        self.model, self.tensors = model, tensors
        self.copies, self.counts = {}, {}

    def snap(self, stage, copy=True):
        tensors = self.tensors(self.model)
        self.counts[stage] = counters(self.model, tensors)
        if copy:
            self.copies[stage] = [t.detach().clone() for t in tensors]
        return self.counts[stage]

    def same_as(self, stage):
        return all(torch.equal(t, c) for t, c in zip(self.tensors(self.model),
                                                     self.copies[stage]))

    def moment_shapes(self):
        state = self.model.optimizer.state
        return [list(state[p]["exp_avg"].shape) if p in state else None
                for p in self.tensors(self.model)]

    def after_backward(self, consumed, label):
        """Consumed: counters advanced by one, no gradient left for the
        optimizer. Otherwise: nothing written."""
        now = self.counts["backward"]
        if consumed:
            if now != [c + 1 for c in self.counts["before"]]:
                _trace_fail(f"{label} counters did not advance once")
            if any(t.grad is not None for t in self.tensors(self.model)):
                _trace_fail(f"{label} gradients left for the optimizer")
        elif now != self.counts["before"] or not self.same_as("before"):
            _trace_fail(f"{label} changed without consumption")

    def after_step(self, consumed, skipped, label):
        """Consumed: the optimizer step left the group alone. Skipped step:
        nothing changed since the step began."""
        now = self.counts["step"]
        if consumed and (now != self.counts["backward"] or not self.same_as("backward")):
            _trace_fail(f"{label} updated twice")
        if skipped and (now != self.counts["before"] or not self.same_as("before")):
            _trace_fail(f"{label} changed on a skipped step")


class _TraceRecord:
    """The trace row of one step and the snapshots behind its checks."""

    def __init__(self, model, iteration, enabled, policy_reason, with_activations):
        self.sh = _Watch(model, _sh_tensors)
        self.act = _Watch(model, _activation_tensors) if with_activations else None
        self.row = {"iteration": iteration, "enabled": enabled,
                    "policy_reason": policy_reason, "count_before": len(model.get_xyz),
                    "degree": model.active_sh_degree,
                    "counters_before": self.sh.snap("before")}
        if self.act is not None:
            self.row["activation"] = {"counters_before": self.act.snap("before")}

    def after_backward(self, model, loss):
        consumer = getattr(model, "_clad_consumer", None)
        consumed = bool(consumer is not None and consumer.active is not None
                        and consumer.active.consumed)
        self.row["consumed"] = consumed
        self.row["loss"] = float(loss.detach())
        if not torch.isfinite(loss):
            _trace_fail("non-finite loss")
        self.row["counters_after_backward"] = self.sh.snap("backward")
        self.sh.after_backward(consumed, "SH")
        if self.act is not None:
            owner = getattr(model, "_clad_activations", None)
            frame = owner.active if owner is not None else None
            detail = self.row["activation"]
            detail["consumed"] = bool(frame is not None and frame.consumed)
            detail["reason"] = owner.last_reason if owner is not None else "disabled"
            detail["counters_after_backward"] = self.act.snap("backward")
            self.act.after_backward(detail["consumed"], "activation")

    def after_step(self, model):
        skipped = self.row["policy_reason"] == SKIPPED
        self.row["count_after"] = len(model.get_xyz)
        self.row["counters_after_step"] = self.sh.snap("step", copy=False)
        self.sh.after_step(self.row["consumed"], skipped, "SH")
        self.row["moment_shapes"] = self.sh.moment_shapes()
        if self.act is not None:
            detail = self.row["activation"]
            detail["counters_after_step"] = self.act.snap("step", copy=False)
            self.act.after_step(detail["consumed"], skipped, "activation")
            detail["moment_shapes"] = self.act.moment_shapes()
        return self.row


def _append_trace(row):
    path = Path(TRACE)
    rows = json.loads(path.read_text()) if path.exists() else []
    rows.append(row)
    path.write_text(json.dumps(rows, indent=2))


def _mark_called(model, key):
    if SUMMARY is not None and hasattr(model, "_clad_routing"):
        model._clad_routing[key] = True


def begin_step(model, iteration, options, dataset, testing, saving, enabled):
    policy = official_step_policy(iteration, options,
                                  white_background=dataset.white_background,
                                  testing_iterations=testing, saving_iterations=saving)
    owner = getattr(model, "_clad_activations", None)
    if owner is not None and owner.active is not None:
        raise RuntimeError("finish the previous activation step first")
    reason = policy.reason()
    if SUMMARY is not None:
        model._clad_routing = {"iteration": iteration, "enabled": enabled,
                               "policy_reason": reason,
                               "activation_enabled": ACTIVATION_EXTENSION is not None,
                               "sh_called": False, "activations_called": False}
    if TRACE is not None:
        model._clad_trace = _TraceRecord(model, iteration, enabled, reason,
                                         ACTIVATION_EXTENSION is not None)
    return policy if enabled else None


def activate_consumer(model, policy, *, eligible):
    _mark_called(model, "activations_called")
    if ACTIVATION_EXTENSION is None:
        return None
    consumer = getattr(model, "_clad_activations", None)
    if consumer is None:
        consumer = model._clad_activations = DenseActivationConsumer(ACTIVATION_EXTENSION)
    if not eligible:
        consumer.last_reason = "unsupported activation renderer path"
        return None
    return consumer.bind(model, policy, exclusive_use=True)


def _sh_consumer(model):
    """The model's SH consumer, rebuilt when the optimizer or the
    configuration it was made for changed (e.g. after a checkpoint restore)."""
    consumer = getattr(model, "_clad_consumer", None)
    if (consumer is None or consumer.optimizer is not model.optimizer
            or consumer.consume_position != POSITION
            or consumer.direct_inputs != DIRECT_INPUTS):
        consumer = model._clad_consumer = DenseSHConsumer(
            model.optimizer, native=native, extension=extension,
            direct_inputs=DIRECT_INPUTS, consume_position=POSITION)
    return consumer


def render_consumer(model, means, screen, opacity, scale, rotation, settings, policy):
    _mark_called(model, "sh_called")
    return _sh_consumer(model).render(means, screen, model._features_dc,
                                      model._features_rest, opacity, scale, rotation,
                                      settings, policy)


def after_backward(model, iteration, loss):
    if SUMMARY is not None:
        SUMMARY.capture(model._clad_routing, getattr(model, "_clad_consumer", None),
                        getattr(model, "_clad_activations", None))
    if TRACE is not None:
        model._clad_trace.after_backward(model, loss)


def after_step(model, iteration):
    if TRACE is not None:
        _append_trace(model._clad_trace.after_step(model))
        del model._clad_trace
    for name in ("_clad_consumer", "_clad_activations"):
        consumer = getattr(model, name, None)
        if consumer is not None:
            consumer.end_step()
    if SUMMARY is not None:
        SUMMARY.record(model._clad_routing)
        del model._clad_routing
