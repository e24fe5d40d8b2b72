"""Dense fused Adam for the trainer's Gaussian optimizer (drop-in for the
reference's optimizer_setup.py:1-40).

The consumed SH and activation updates reproduce torch's fused Adam
arithmetic, so the trainer's optimizer must be `torch.optim.Adam(fused=True,
foreach=False)` for the groups that fall back to it to match. `fused_adam`
rebuilds an existing Adam with those options and carries parameters,
moments and step counters over unchanged (step tensors move to the parameter
device, which fused Adam requires).
"""

from __future__ import annotations

import torch


def fused_adam(optimizer):
    if type(optimizer) is not torch.optim.Adam:
        raise ValueError("--fused-adam requires the default dense Adam optimizer")
    for group in optimizer.param_groups:
        for parameter in group["params"]:
            if not parameter.is_cuda or parameter.dtype != torch.float32:
                raise ValueError("--fused-adam requires CUDA float32 Gaussian parameters")
            step = optimizer.state.get(parameter, {}).get("step")
            if step is not None and (not torch.is_tensor(step) or step.dtype != torch.float32):
                raise ValueError("--fused-adam requires native float32 Adam step counters")
    defaults = dict(optimizer.defaults, fused=True, foreach=False)
    groups = [dict(group, fused=True, foreach=False) for group in optimizer.param_groups]
    replacement = torch.optim.Adam(groups, **defaults)
    saved = optimizer.state_dict()
    for group in saved["param_groups"]:
        group.update(fused=True, foreach=False)
    replacement.load_state_dict(saved)
    return replacement


def enable_fused_adam(model_type):
    """Re-wraps GaussianModel.training_setup and .restore so the optimizer is
    fused Adam after setup and after a checkpoint restore."""
    setup, restore = model_type.training_setup, model_type.restore

    def training_setup(model, *args, **kwargs):
        setup(model, *args, **kwargs)
        model.optimizer = fused_adam(model.optimizer)

    def restore_checkpoint(model, *args, **kwargs):
        restore(model, *args, **kwargs)
        model.optimizer = fused_adam(model.optimizer)

    model_type.training_setup = training_setup
    model_type.restore = restore_checkpoint
