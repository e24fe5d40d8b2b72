"""Claims on torch.optim.Adam groups for steps whose update runs inside a
CUDA backward instead of `optimizer.step()`.

A consumed step writes a parameter, its two Adam moments and (from Python) its
step counter without the optimizer seeing a gradient. That is only sound while
the optimizer still owns exactly those objects, so every consumer works in
three phases built from this module:

1. *screen*: rule tables decide, before anything is written, whether a group
   can be consumed at all (`first_failure` / `last_failure` evaluate a table
   of ``(reason, predicate)`` rows);
2. *claim*: `Claim.take` records the identity and version counter of every
   object the kernel will touch (group dict, parameter, state dict, moments,
   counter, hyperparameters);
3. *verify / settle*: `Claim.intact` re-checks all of it right before the
   kernel launch, and `settle` advances the counters and autograd versions
   once the kernel has run.

The SH consumer (adapter.py), the activation consumer (activation.py) and the
position group share these pieces; their reason strings are those of the
reference's adapter.py / activation.py so routing summaries read the same.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

# Adam hyperparameters whose values fix the update arithmetic; a claim keeps
# them and any change between bind and backward voids the claim.
ADAM_OPTIONS = ("lr", "betas", "eps", "fused", "foreach", "weight_decay", "amsgrad",
                "maximize", "capturable", "differentiable")
MOMENT_KEYS = ("exp_avg", "exp_avg_sq")
STATE_KEYS = MOMENT_KEYS + ("step",)
# Options that select a different Adam variant (all must be falsy).
VARIANT_FLAGS = ("amsgrad", "maximize", "differentiable", "capturable")
# Largest step counter whose successor is still exact in float32.
COUNTER_LIMIT = 2 ** 24


def first_failure(rules, *args):
    """Reason of the first row whose predicate holds, or None."""
    for reason, broken in rules:
        if broken(*args):
            return reason
    return None


def last_failure(rules, *args):
    """Reason of the last row whose predicate holds, or None (tables written
    from general to specific: the most specific finding names the fallback)."""
    found = None
    for reason, broken in rules:
        if broken(*args):
            found = reason
    return found


def byte_extent(tensor):
    start = tensor.data_ptr()
    return start, start + tensor.numel() * tensor.element_size()


def overlapping(tensors) -> bool:
    """True when two non-empty tensors share a byte of storage."""
    extents = sorted(byte_extent(t) for t in tensors if t.numel())
    return any(prev_end > start for (_, prev_end), (start, _) in zip(extents, extents[1:]))


def sole_group(optimizer, name):
    """The one param group called `name`, or None when there are none or several."""
    found = [g for g in optimizer.param_groups if g.get("name") == name]
    return found[0] if len(found) == 1 else None


def owns_only(group, param) -> bool:
    return len(group["params"]) == 1 and group["params"][0] is param


def dense_fp32_cuda(tensor, shape=None) -> bool:
    return (tensor.is_cuda and tensor.dtype == torch.float32 and tensor.is_contiguous()
            and (shape is None or tuple(tensor.shape) == tuple(shape)))


def plain_fused_adam(group) -> bool:
    """torch's fused dense Adam without decay or any variant flag: the update
    the CUDA kernels reproduce."""
    return (group.get("fused") is True and not group.get("foreach")
            and group.get("weight_decay", 0) == 0
            and not any(group.get(k, False) for k in VARIANT_FLAGS))


def reference_betas(group) -> bool:
    return group["betas"] == (0.9, 0.999) and group["eps"] == 1e-15


def finite_rate(rate) -> bool:
    return isinstance(rate, (float, int)) and math.isfinite(rate)


def state_or_fresh(optimizer, param, counter_device):
    """The optimizer's state for `param`, or a new zero state (not installed
    until the claim is taken) with its counter on `counter_device`."""
    state = optimizer.state.get(param)
    if state:
        return state
    return {"step": torch.zeros((), device=counter_device),
            "exp_avg": torch.zeros_like(param),
            "exp_avg_sq": torch.zeros_like(param)}


def state_problem(state, param):
    """'moments' or 'counter' when the state cannot be written by the kernel
    (moments not dense like the parameter; counter not one float32 on the
    parameter's device), else None."""
    for key in MOMENT_KEYS:
        value = state.get(key)
        if not (torch.is_tensor(value) and value.shape == param.shape
                and value.dtype == param.dtype and value.device == param.device
                and value.is_contiguous()):
            return "moments"
    step = state.get("step")
    if not (torch.is_tensor(step) and step.device == param.device
            and step.dtype == torch.float32 and step.numel() == 1):
        return "counter"
    return None


def read_counters(states):
    """All step counters with one device-to-host read."""
    return torch.stack([s["step"].reshape(()) for s in states]).cpu().tolist()


def valid_counter(value) -> bool:
    return (math.isfinite(value) and value >= 0 and value == int(value)
            and value < COUNTER_LIMIT)


def bias_corrections(step):
    """(1 - 0.9^t, sqrt(1 - 0.999^t)) in Python double, as torch's Adam forms them."""
    return 1 - 0.9 ** step, math.sqrt(1 - 0.999 ** step)


@dataclass
class Claim:
    """What one consumed group may write, as it was when the step was bound."""

    group: dict
    param: torch.Tensor
    state: dict
    entries: dict = field(default_factory=dict)   # key -> tensor at bind time
    versions: tuple = ()                          # param, then entries, versions
    options: tuple = ()

    @classmethod
    def take(cls, group, state):
        param = group["params"][0]
        entries = {k: state[k] for k in STATE_KEYS}
        return cls(group=group, param=param, state=state, entries=entries,
                   versions=cls._versions(param, entries),
                   options=tuple(group.get(k) for k in ADAM_OPTIONS))

    @staticmethod
    def _versions(param, entries):
        return (param._version,) + tuple(v._version for v in entries.values())

    @property
    def moments(self):
        return self.entries["exp_avg"], self.entries["exp_avg_sq"]

    def intact(self, optimizer) -> bool:
        """True when the optimizer still owns exactly what was claimed and
        nothing was written or re-bound since."""
        p = self.param
        if not (owns_only(self.group, p) and any(g is self.group for g in optimizer.param_groups)
                and optimizer.state.get(p) is self.state):
            return False
        if any(self.state.get(k) is not v for k, v in self.entries.items()):
            return False
        if p.grad is not None or not p.requires_grad:
            return False
        return (self._versions(p, self.entries) == self.versions
                and tuple(self.group.get(k) for k in ADAM_OPTIONS) == self.options)


@torch.no_grad()
def settle(claims):
    """After the kernel ran: one optimizer step on every counter, one version
    bump on every written tensor (so autograd sees the in-place update)."""
    for claim in claims:
        claim.state["step"].add_(1)
    torch.autograd.graph.increment_version(
        [t for c in claims for t in (c.param, *c.moments)])
