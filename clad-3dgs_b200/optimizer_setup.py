"""torch's fused dense Adam for the trainer's Gaussian optimizer (the
trainer-facing `optimizer_setup` module; same names and errors as the
reference's optimizer_setup.py:1-40).

The consumed SH and activation updates reproduce the arithmetic of
`torch.optim.Adam(fused=True, foreach=False)`, so the groups that stay with
the optimizer must use that implementation too for a consumed step and a
native one to agree. `fused_adam` builds that optimizer over the same
parameter groups and moves the existing per-parameter state across as it is:
moment tensors are handed over (not copied), and step counters, which fused
Adam keeps on the parameter's device, are moved there.
"""

from __future__ import annotations

import torch


def _unfusable(optimizer):
    """The error message when `optimizer` cannot become fused Adam, else None."""
    if type(optimizer) is not torch.optim.Adam:
        return "--fused-adam requires the default dense Adam optimizer"
    for group in optimizer.param_groups:
        for param in group["params"]:
            if not (param.is_cuda and param.dtype == torch.float32):
                return "--fused-adam requires CUDA float32 Gaussian parameters"
            step = optimizer.state.get(param, {}).get("step")
            if step is not None and not (torch.is_tensor(step) and step.dtype == torch.float32):
                return "--fused-adam requires native float32 Adam step counters"
    return None


def _moved_state(state, param):
    moved = dict(state)
    if "step" in moved:
        moved["step"] = moved["step"].to(device=param.device, dtype=torch.float32)
    return moved


def fused_adam(optimizer):
    problem = _unfusable(optimizer)
    if problem is not None:
        raise ValueError(problem)
    fused = {"fused": True, "foreach": False}
    replacement = torch.optim.Adam([{**g, **fused} for g in optimizer.param_groups],
                                   **{**optimizer.defaults, **fused})
    for param, state in optimizer.state.items():
        if state:
            replacement.state[param] = _moved_state(state, param)
    return replacement


def enable_fused_adam(model_type):
    """Swaps the model's optimizer for fused Adam after `training_setup` and
    after `restore` (a checkpoint restore rebuilds the optimizer)."""

    def after(method):
        def wrapped(model, *args, **kwargs):
            method(model, *args, **kwargs)
            model.optimizer = fused_adam(model.optimizer)
        return wrapped

    model_type.training_setup = after(model_type.training_setup)
    model_type.restore = after(model_type.restore)
