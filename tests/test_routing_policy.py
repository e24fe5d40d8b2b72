"""Routing summary and step policy (host logic, CPU).

Cases follow the reference's check.py:675-740 (routing) and the trainer
policy of adapter.py:365-389.
"""

import json
from types import SimpleNamespace

import pytest

from adapter import StepPolicy, official_step_policy
from routing import RoutingSummary


def _context(iteration):
    return dict(iteration=iteration, enabled=True, activation_enabled=True,
                policy_reason=None, sh_called=True, activations_called=True)


def test_routing_summary_counts_and_reasons(tmp_path):
    path = tmp_path / "routing.json"
    sh = SimpleNamespace(active=SimpleNamespace(consumed=True), last_reason=None)
    activation = SimpleNamespace(active=None, last_reason="unsupported optimizer")
    with RoutingSummary(path, dict(fused_adam=True)) as summary:
        row = _context(7)
        summary.capture(row, sh, activation)
        activation.last_reason = "evaluation without gradients"  # captured before this
        summary.record(row)
        skipped = _context(8)
        skipped["policy_reason"] = "topology changes before optimizer step"
        sh.active = None
        summary.capture(skipped, sh, activation)
        summary.record(skipped)
        uncompleted = _context(9)
        summary.capture(uncompleted, sh, activation)
        assert json.loads(path.read_text())["completed_training_steps"] == 0
    result = json.loads(path.read_text())
    assert result["status"] == "completed"
    assert result["completed_training_steps"] == 2
    assert (result["first_iteration"], result["last_iteration"]) == (7, 8)
    assert result["sh"]["consumed_steps"] == 1
    assert result["activations"]["fallback_reasons"] == {
        "unsupported optimizer": 1, "topology changes before optimizer step": 1}
    saved = path.read_bytes()
    with pytest.raises(FileExistsError):
        RoutingSummary(path, {})
    assert path.read_bytes() == saved


def test_routing_summary_failure_and_reasons(tmp_path):
    failed = tmp_path / "failed.json"
    with pytest.raises(RuntimeError, match="fixture failure"):
        with RoutingSummary(failed, {}) as summary:
            row = _context(10)
            row["enabled"] = False
            summary.capture(row, None, None)
            summary.record(row)
            raise RuntimeError("fixture failure")
    result = json.loads(failed.read_text())
    assert result["status"] == "failed" and result["completed_training_steps"] == 1
    assert result["sh"]["fallback_reasons"] == {"consumption disabled": 1}
    assert "fixture failure" in result["error"]
    for enabled, called, reason in ((False, False, "activation consumption disabled"),
                                    (True, False, "unsupported renderer path"),
                                    (True, True, "backward did not consume")):
        row = _context(11)
        row.update(activation_enabled=enabled, activations_called=called)
        summary.capture(row, None, None)
        assert row["activations"]["reason"] == reason


def test_step_policy_reasons():
    assert StepPolicy().reason() is None
    cases = {
        StepPolicy(optimizer_step=False): "optimizer step skipped",
        StepPolicy(topology_change=True): "topology changes before optimizer step",
        StepPolicy(observation_before_step=True): "parameters observed before optimizer step",
        StepPolicy(single_backward=False): "gradient accumulation or multiple backward calls",
        StepPolicy(unscaled_gradients=False): "scaled gradients require native optimizer processing",
        StepPolicy(exclusive_sh_use=False): "SH parameters used by another loss or consumer",
    }
    for policy, reason in cases.items():
        assert policy.reason() == reason


def test_official_step_policy_marks_trainer_mutations():
    options = SimpleNamespace(densify_until_iter=15000, densify_from_iter=500,
                              densification_interval=100, opacity_reset_interval=3000,
                              iterations=30000)
    assert official_step_policy(7, options).reason() is None
    assert official_step_policy(600, options).topology_change          # densify
    assert not official_step_policy(500, options).topology_change      # from_iter excluded
    assert official_step_policy(500, options, white_background=True).topology_change
    assert official_step_policy(3000, options).topology_change         # opacity reset
    assert not official_step_policy(16000, options).topology_change    # after densify window
    assert official_step_policy(7000, options, testing_iterations=(7000,)).observation_before_step
    assert official_step_policy(30000, options, saving_iterations=(30000,)).reason()
    assert not official_step_policy(30000, options).optimizer_step     # final iteration
