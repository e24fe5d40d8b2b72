"""Routing summary: how many training steps consumed their SH and activation
gradients and why the others fell back (the trainer-facing `routing`
module; same class, JSON keys and reason strings as the reference's
routing.py:1-68).

Everything is counted in Python from the consumers' own flags: no tensor is
read and nothing synchronises. The report file is created exclusively (an
existing report is never overwritten), reads "running" while training and
"completed" or "failed" (with the error) when the `with` block exits.
"""

from __future__ import annotations

import json
from collections import Counter
from enum import Enum

FAMILIES = ("sh", "activations")


class Fallback(str, Enum):
    """Reasons the summary itself assigns; the policy's and the consumers' own
    reasons are passed through as given."""

    DISABLED = "consumption disabled"
    ACTIVATIONS_DISABLED = "activation consumption disabled"
    NOT_CALLED = "unsupported renderer path"
    NOT_CONSUMED = "backward did not consume"


def route(context, family, owner):
    """(consumed, reason) of one family for the step described by `context`
    (iteration, enabled, activation_enabled, policy_reason, sh_called,
    activations_called). The first matching row decides."""
    frame = getattr(owner, "active", None) if owner is not None else None
    if frame is not None and frame.consumed:
        return True, None
    rows = (
        (not context["enabled"], Fallback.DISABLED.value),
        (family == "activations" and not context["activation_enabled"],
         Fallback.ACTIVATIONS_DISABLED.value),
        (bool(context["policy_reason"]), context["policy_reason"]),
        (not context[family + "_called"], Fallback.NOT_CALLED.value),
    )
    for applies, reason in rows:
        if applies:
            return False, reason
    return False, (getattr(owner, "last_reason", None) or Fallback.NOT_CONSUMED.value)


class _Tally:
    def __init__(self):
        self.consumed = 0
        self.reasons = Counter()

    def add(self, consumed, reason):
        if consumed:
            self.consumed += 1
        else:
            self.reasons[reason] += 1

    def as_json(self):
        return {"consumed_steps": self.consumed,
                "fallback_steps": sum(self.reasons.values()),
                "fallback_reasons": dict(self.reasons)}


class RoutingSummary:
    def __init__(self, path, configuration):
        self.path = path
        self.configuration = configuration
        self.status = "running"
        self.error = None
        self.steps = 0
        self.first = self.last = None
        self.tallies = {f: _Tally() for f in FAMILIES}
        with path.open("x") as stream:  # refuse to replace an earlier report
            stream.write(self._text())

    @property
    def result(self):
        doc = {"status": self.status, "configuration": self.configuration,
               "completed_training_steps": self.steps, "first_iteration": self.first,
               "last_iteration": self.last}
        doc.update({f: self.tallies[f].as_json() for f in FAMILIES})
        if self.error is not None:
            doc["error"] = self.error
        return doc

    def _text(self):
        return json.dumps(self.result, indent=2) + "\n"

    def __enter__(self):
        return self

    def __exit__(self, kind, error, traceback):
        clean = kind is None or (isinstance(error, SystemExit) and error.code in (None, 0))
        self.status = "completed" if clean else "failed"
        if not clean:
            self.error = f"{kind.__name__}: {error}"
        self.path.write_text(self._text())
        print(f"Routing summary: {self.path} ({self.status}, {self.steps} completed steps)")
        return False

    def capture(self, context, sh, activations):
        """Fixes this step's route right after backward, before evaluation
        code can overwrite a consumer's last_reason."""
        for family, owner in zip(FAMILIES, (sh, activations)):
            consumed, reason = route(context, family, owner)
            context[family] = {"consumed": consumed, "reason": reason}

    def record(self, context):
        """Counts a step whose lifecycle hooks have all run."""
        for family in FAMILIES:
            self.tallies[family].add(context[family]["consumed"], context[family]["reason"])
        self.steps += 1
        if self.first is None:
            self.first = context["iteration"]
        self.last = context["iteration"]
