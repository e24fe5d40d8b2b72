"""Routing summary: which training steps consumed SH / activation gradients and
why the others fell back (drop-in for the reference's routing.py:1-68).

Counts are kept in Python; nothing here reads a tensor or synchronises. The
report is created with exclusive-create so an existing file is never
overwritten, says "running" while training, and "completed" or "failed" (with
the error) at exit.
"""

from __future__ import annotations

import json


class RoutingSummary:
    def __init__(self, path, configuration):
        self.path = path
        self.result = {
            "status": "running",
            "configuration": configuration,
            "completed_training_steps": 0,
            "first_iteration": None,
            "last_iteration": None,
            "sh": {"consumed_steps": 0, "fallback_steps": 0, "fallback_reasons": {}},
            "activations": {"consumed_steps": 0, "fallback_steps": 0, "fallback_reasons": {}},
        }
        with path.open("x") as stream:
            stream.write(json.dumps(self.result, indent=2) + "\n")

    def __enter__(self):
        return self

    def __exit__(self, kind, error, traceback):
        ok = kind is None or (isinstance(error, SystemExit) and error.code in (None, 0))
        self.result["status"] = "completed" if ok else "failed"
        if not ok:
            self.result["error"] = f"{kind.__name__}: {error}"
        self.path.write_text(json.dumps(self.result, indent=2) + "\n")
        print(f"Routing summary: {self.path} ({self.result['status']}, "
              f"{self.result['completed_training_steps']} completed steps)")
        return False

    def capture(self, context, sh, activations):
        """Records this step's route before evaluation code can overwrite the
        consumers' last_reason."""
        for name, owner in (("sh", sh), ("activations", activations)):
            frame = None if owner is None else owner.active
            consumed = bool(frame is not None and frame.consumed)
            if consumed:
                reason = None
            elif not context["enabled"]:
                reason = "consumption disabled"
            elif name == "activations" and not context["activation_enabled"]:
                reason = "activation consumption disabled"
            elif context["policy_reason"]:
                reason = context["policy_reason"]
            elif not context[name + "_called"]:
                reason = "unsupported renderer path"
            else:
                reason = (owner.last_reason if owner is not None else None) or \
                    "backward did not consume"
            context[name] = {"consumed": consumed, "reason": reason}

    def record(self, context):
        """Counts a completed step (after its lifecycle hooks ran)."""
        for name in ("sh", "activations"):
            route, counts = context[name], self.result[name]
            if route["consumed"]:
                counts["consumed_steps"] += 1
            else:
                counts["fallback_steps"] += 1
                reasons = counts["fallback_reasons"]
                reasons[route["reason"]] = reasons.get(route["reason"], 0) + 1
        self.result["completed_training_steps"] += 1
        if self.result["first_iteration"] is None:
            self.result["first_iteration"] = context["iteration"]
        self.result["last_iteration"] = context["iteration"]
