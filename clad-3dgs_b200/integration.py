"""Trainer hooks for SH and activation consumption (drop-in for the
reference's integration.py:1-219, which the reference copies into the patched
trainer as clad_training.py and calls from train.py and render(),
trainer.patch:1-47).

Per step: `begin_step` decides the step policy (official_step_policy) and, with
a summary or trace enabled, snapshots routing / state; `activate_consumer`
binds the activation consumer and returns the activated (rotation, scaling,
opacity) for the renderer, or None; `render_consumer` renders through the
dense SH consumer (falling back to the plain rasterizer); `after_backward`
records the routing decision and, in trace mode, checks the once-only update
rules; `after_step` releases the frames and writes the trace row.

Module globals, set by the launcher: SUMMARY (a routing.RoutingSummary),
TRACE (a JSON path; trace mode synchronises and snapshots parameters, for
small functional fixtures only), DIRECT_INPUTS (render from dc/rest directly),
ACTIVATION_EXTENSION (the clad_quaternion surface, or None to disable
activation consumption), POSITION (also consume the xyz group; not in the
reference).
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
POSITION = False  # also consume the xyz group (see adapter.DenseSHConsumer)


def counters(model, parameters=None):
    """Adam step counters of the given parameters (SH groups by default)."""
    values = []
    for p in ([model._features_dc, model._features_rest] if parameters is None else parameters):
        state = model.optimizer.state.get(p, {})
        values.append(int(state["step"].item()) if "step" in state else 0)
    return values


def begin_step(model, iteration, options, dataset, testing, saving, enabled):
    policy = official_step_policy(iteration, options,
                                  white_background=dataset.white_background,
                                  testing_iterations=testing, saving_iterations=saving)
    activation = getattr(model, "_clad_activations", None)
    if activation is not None and activation.active is not None:
        raise RuntimeError("finish the previous activation step first")
    if SUMMARY is not None:
        model._clad_routing = dict(iteration=iteration, enabled=enabled,
                                   policy_reason=policy.reason(),
                                   activation_enabled=ACTIVATION_EXTENSION is not None,
                                   sh_called=False, activations_called=False)
    if TRACE is not None:
        model._clad_trace = dict(iteration=iteration, enabled=enabled,
                                 policy_reason=policy.reason(), count_before=len(model.get_xyz),
                                 degree=model.active_sh_degree, counters_before=counters(model),
                                 dc=model._features_dc.detach().clone(),
                                 rest=model._features_rest.detach().clone())
        if ACTIVATION_EXTENSION is not None:
            raw = [getattr(model, name) for name in ATTRS]
            model._clad_trace["activation"] = dict(counters_before=counters(model, raw),
                                                   before=[p.detach().clone() for p in raw])
    return policy if enabled else None


def activate_consumer(model, policy, *, eligible):
    if SUMMARY is not None and hasattr(model, "_clad_routing"):
        model._clad_routing["activations_called"] = True
    if ACTIVATION_EXTENSION is None:
        return None
    consumer = getattr(model, "_clad_activations", None)
    if consumer is None:
        consumer = DenseActivationConsumer(ACTIVATION_EXTENSION)
        model._clad_activations = consumer
    if not eligible:
        consumer.last_reason = "unsupported activation renderer path"
        return None
    return consumer.bind(model, policy, exclusive_use=True)


def render_consumer(model, means, screen, opacity, scale, rotation, settings, policy):
    if SUMMARY is not None and hasattr(model, "_clad_routing"):
        model._clad_routing["sh_called"] = True
    consumer = getattr(model, "_clad_consumer", None)
    if (consumer is None or consumer.optimizer is not model.optimizer
            or consumer.consume_position != POSITION):
        consumer = DenseSHConsumer(model.optimizer, native=native, extension=extension,
                                   direct_inputs=DIRECT_INPUTS, consume_position=POSITION)
        model._clad_consumer = consumer
    return consumer.render(means, screen, model._features_dc, model._features_rest, opacity,
                           scale, rotation, settings, policy)


def _equal_all(tensors, saved):
    return all(torch.equal(t, s) for t, s in zip(tensors, saved))


def after_backward(model, iteration, loss):
    if SUMMARY is not None:
        SUMMARY.capture(model._clad_routing, getattr(model, "_clad_consumer", None),
                        getattr(model, "_clad_activations", None))
    if TRACE is None:
        return
    row = model._clad_trace
    consumer = getattr(model, "_clad_consumer", None)
    consumed = bool(consumer is not None and consumer.active is not None
                    and consumer.active.consumed)
    row["consumed"] = consumed
    row["loss"] = float(loss.detach())
    assert torch.isfinite(loss)
    row["counters_after_backward"] = counters(model)
    if consumed:
        assert row["counters_after_backward"] == [c + 1 for c in row["counters_before"]]
        assert model._features_dc.grad is None and model._features_rest.grad is None
    else:
        assert row["counters_after_backward"] == row["counters_before"]
        assert _equal_all([model._features_dc, model._features_rest], [row["dc"], row["rest"]])
    row["dc_after_backward"] = model._features_dc.detach().clone()
    row["rest_after_backward"] = model._features_rest.detach().clone()
    if "activation" in row:
        activation = getattr(model, "_clad_activations", None)
        frame = activation.active if activation is not None else None
        detail = row["activation"]
        detail["consumed"] = bool(frame is not None and frame.consumed)
        detail["reason"] = activation.last_reason if activation is not None else "disabled"
        raw = [getattr(model, name) for name in ATTRS]
        detail["counters_after_backward"] = counters(model, raw)
        if detail["consumed"]:
            assert detail["counters_after_backward"] == [c + 1 for c in detail["counters_before"]]
            assert all(p.grad is None for p in raw)
        else:
            assert detail["counters_after_backward"] == detail["counters_before"]
            assert _equal_all(raw, detail["before"])
        detail["after_backward"] = [p.detach().clone() for p in raw]


def _moment_shapes(model, params):
    return [list(model.optimizer.state[p]["exp_avg"].shape) if p in model.optimizer.state
            else None for p in params]


def after_step(model, iteration):
    consumer = getattr(model, "_clad_consumer", None)
    if TRACE is not None:
        row = model._clad_trace
        row["count_after"] = len(model.get_xyz)
        row["counters_after_step"] = counters(model)
        sh = [model._features_dc, model._features_rest]
        if row["consumed"]:
            # The following optimizer step must have skipped the consumed groups.
            assert row["counters_after_step"] == row["counters_after_backward"]
            assert _equal_all(sh, [row["dc_after_backward"], row["rest_after_backward"]])
        if row["policy_reason"] == "optimizer step skipped":
            assert row["counters_after_step"] == row["counters_before"]
            assert _equal_all(sh, [row["dc"], row["rest"]])
        row["moment_shapes"] = _moment_shapes(model, sh)
        if "activation" in row:
            detail = row["activation"]
            raw = [getattr(model, name) for name in ATTRS]
            detail["counters_after_step"] = counters(model, raw)
            if detail["consumed"]:
                assert detail["counters_after_step"] == detail["counters_after_backward"]
                assert _equal_all(raw, detail["after_backward"])
            if row["policy_reason"] == "optimizer step skipped":
                assert detail["counters_after_step"] == detail["counters_before"]
                assert _equal_all(raw, detail["before"])
            detail["moment_shapes"] = _moment_shapes(model, raw)
            del detail["before"], detail["after_backward"]
        for key in ("dc", "rest", "dc_after_backward", "rest_after_backward"):
            del row[key]
        path = Path(TRACE)
        rows = json.loads(path.read_text()) if path.exists() else []
        rows.append(row)
        path.write_text(json.dumps(rows, indent=2))
        del model._clad_trace
    if consumer is not None:
        consumer.end_step()
    activation = getattr(model, "_clad_activations", None)
    if activation is not None:
        activation.end_step()
    if SUMMARY is not None:
        SUMMARY.record(model._clad_routing)
        del model._clad_routing
