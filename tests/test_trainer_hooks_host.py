"""Host logic of the trainer hooks on CPU tensors: the claim layer shared by
the SH and activation consumers, fused-Adam setup errors, the activation
consumer's declared-condition precedence, and the trace invariants of the
integration hooks driven by stand-in consumers.

The GPU side of the same lifecycle (binding real CUDA groups, the kernels'
updates) is in test_gpu_binding.py and test_gpu_training_step.py; the cases
follow the reference's check.py:304-497 (binding), 501-622 (SH binding) and
625-672 (optimizer setup).
"""

import json
from types import SimpleNamespace

import pytest
import torch

import optimizer_claims as oc


def _adam_group(n=4, name="probe"):
    p = torch.nn.Parameter(torch.zeros(n, 3))
    opt = torch.optim.Adam([dict(params=[p], name=name, lr=0.001)], eps=1e-15)
    opt.state[p] = dict(step=torch.zeros(()), exp_avg=torch.zeros_like(p),
                        exp_avg_sq=torch.zeros_like(p))
    return p, opt


def test_rule_tables_pick_first_and_last_failure():
    rules = (("a", lambda x: x > 0), ("b", lambda x: x > 1), ("c", lambda x: x > 5))
    assert oc.first_failure(rules, 0) is None and oc.last_failure(rules, 0) is None
    assert oc.first_failure(rules, 3) == "a"
    assert oc.last_failure(rules, 3) == "b"
    assert oc.last_failure(rules, 9) == "c"


def test_overlap_detection_by_byte_extent():
    base = torch.zeros(16)
    assert not oc.overlapping([base[:8], base[8:]])
    assert oc.overlapping([base[:9], base[8:]])
    assert not oc.overlapping([base[:0], base])          # empty tensors own nothing
    assert oc.overlapping([base, torch.zeros(2), base[3:4]])


def test_counter_validity():
    for good in (0.0, 1.0, 2.0 ** 24 - 1):
        assert oc.valid_counter(good)
    for bad in (float("nan"), float("inf"), -1.0, 0.5, 2.0 ** 24):
        assert not oc.valid_counter(bad)
    b1, b2 = oc.bias_corrections(1)
    assert b1 == 1 - 0.9 and b2 == (1 - 0.999) ** 0.5


@pytest.mark.parametrize("case", ["none", "parameter", "state", "moment", "moment-write",
                                  "counter", "options", "group", "gradient", "frozen",
                                  "second-param"])
def test_claim_detects_every_change(case):
    p, opt = _adam_group()
    claim = oc.Claim.take(opt.param_groups[0], opt.state[p])
    if case == "parameter":
        with torch.no_grad():
            p.add_(1)
    elif case == "state":
        opt.state[p] = dict(opt.state[p])
    elif case == "moment":
        opt.state[p]["exp_avg"] = opt.state[p]["exp_avg"].clone()
    elif case == "moment-write":
        opt.state[p]["exp_avg_sq"].add_(1)
    elif case == "counter":
        opt.state[p]["step"].add_(1)
    elif case == "options":
        opt.param_groups[0]["betas"] = (0.8, 0.999)
    elif case == "group":
        opt.param_groups[0] = dict(opt.param_groups[0])
    elif case == "gradient":
        p.grad = torch.ones_like(p)
    elif case == "frozen":
        p.requires_grad_(False)
    elif case == "second-param":
        opt.param_groups[0]["params"].append(torch.nn.Parameter(torch.zeros(1)))
    assert claim.intact(opt) == (case == "none")


def test_settle_advances_counters_and_versions_once():
    p, opt = _adam_group()
    claim = oc.Claim.take(opt.param_groups[0], opt.state[p])
    tensors = [p, *claim.moments]
    versions = [t._version for t in tensors]
    oc.settle([claim])
    assert float(opt.state[p]["step"]) == 1.0
    assert [t._version for t in tensors] == [v + 1 for v in versions]


def test_fresh_state_and_state_problems():
    p, opt = _adam_group()
    fresh = oc.state_or_fresh(opt, torch.nn.Parameter(torch.zeros(2)), "cpu")
    assert float(fresh["step"]) == 0 and fresh["exp_avg"].shape == (2,)
    state = opt.state[p]
    assert oc.state_problem(state, p) is None
    assert oc.state_problem(dict(state, exp_avg=state["exp_avg"].t()), p) == "moments"
    assert oc.state_problem(dict(state, exp_avg_sq=None), p) == "moments"
    assert oc.state_problem(dict(state, step=torch.zeros(2)), p) == "counter"
    assert oc.state_problem(dict(state, step=torch.zeros((), dtype=torch.float64)), p) == \
        "counter"
    assert oc.state_problem({k: v for k, v in state.items() if k != "step"}, p) == "counter"


def test_fused_adam_rejects_what_it_cannot_fuse():
    from optimizer_setup import fused_adam

    p = torch.nn.Parameter(torch.zeros(2))
    with pytest.raises(ValueError, match="default dense Adam"):
        fused_adam(torch.optim.SGD([p], lr=0.1))
    with pytest.raises(ValueError, match="CUDA float32"):
        fused_adam(torch.optim.Adam([p]))


def test_enable_fused_adam_wraps_setup_and_restore(monkeypatch):
    import optimizer_setup

    calls = []

    class Model:
        def training_setup(self, *args):
            calls.append(("setup", args))
            self.optimizer = "plain"

        def restore(self, *args):
            calls.append(("restore", args))
            self.optimizer = "restored"

    monkeypatch.setattr(optimizer_setup, "fused_adam", lambda opt: ("fused", opt))
    optimizer_setup.enable_fused_adam(Model)
    model = Model()
    model.training_setup(1)
    assert model.optimizer == ("fused", "plain")
    model.restore(2, 3)
    assert model.optimizer == ("fused", "restored")
    assert calls == [("setup", (1,)), ("restore", (2, 3))]


def test_activation_declared_conditions_and_policy_precedence():
    from activation import DenseActivationConsumer
    from adapter import StepPolicy

    consumer = DenseActivationConsumer(SimpleNamespace(consume_activations=None))
    model = SimpleNamespace()
    cases = [
        (dict(policy=None, exclusive_use=True), "consumption disabled"),
        (dict(policy=StepPolicy(topology_change=True), exclusive_use=True),
         "topology changes before optimizer step"),
        (dict(policy=StepPolicy(topology_change=True)),
         "activation parameters have other consumers"),
        (dict(policy=StepPolicy(), exclusive_use=True, gradient_processing=True),
         "activation gradients require native processing"),
        (dict(policy=None, exclusive_use=True, higher_order=True),
         "higher-order derivatives require native backward"),
    ]
    for kwargs, reason in cases:
        policy = kwargs.pop("policy")
        assert consumer.bind(model, policy, **kwargs) is None
        assert consumer.last_reason == reason and consumer.active is None
    with torch.no_grad():
        assert consumer.bind(model, StepPolicy(), exclusive_use=True) is None
    assert consumer.last_reason == "evaluation without gradients"
    with pytest.raises(ValueError):
        DenseActivationConsumer(SimpleNamespace())


def test_activation_binding_declines_host_tensors():
    """A model whose parameters are not on a CUDA device keeps torch's path
    with the layout reason and an untouched optimizer."""
    from activation import DenseActivationConsumer
    from adapter import StepPolicy

    model = SimpleNamespace()
    groups = []
    for name, width in (("rotation", 4), ("scaling", 3), ("opacity", 1)):
        raw = torch.nn.Parameter(torch.randn(5, width))
        setattr(model, "_" + name, raw)
        groups.append(dict(params=[raw], name=name, lr=0.01))
    model.optimizer = torch.optim.Adam(groups, eps=1e-15)
    consumer = DenseActivationConsumer(SimpleNamespace(consume_activations=None))
    assert consumer.bind(model, StepPolicy(), exclusive_use=True) is None
    assert consumer.last_reason == "Unsupported activation ownership or layout"
    assert not model.optimizer.state
    model.optimizer = torch.optim.SGD(groups, lr=0.1)
    assert consumer.bind(model, StepPolicy(), exclusive_use=True) is None
    assert consumer.last_reason == "unsupported optimizer"


# ------------------------------------------------------------- trace hooks

class _Model(SimpleNamespace):
    @property
    def get_xyz(self):
        return self._xyz


def _trace_model():
    tensors = dict(_xyz=torch.zeros(3, 3), _features_dc=torch.zeros(3, 1, 3),
                   _features_rest=torch.zeros(3, 15, 3))
    model = _Model(active_sh_degree=3, **{k: torch.nn.Parameter(v) for k, v in tensors.items()})
    params = [model._xyz, model._features_dc, model._features_rest]
    model.optimizer = torch.optim.Adam([dict(params=[p]) for p in params])
    for p in params:
        model.optimizer.state[p] = dict(step=torch.tensor(4.0), exp_avg=torch.zeros_like(p),
                                        exp_avg_sq=torch.zeros_like(p))
    return model


class _FakeSH:
    """Stands in for DenseSHConsumer after the render call."""

    def __init__(self, consumed):
        self.active = SimpleNamespace(consumed=consumed)
        self.last_reason = None if consumed else "unsupported optimizer"
        self.ended = False

    def end_step(self):
        self.ended = True


def _consume(model):
    """What the consumed backward does to the SH groups."""
    with torch.no_grad():
        for p in (model._features_dc, model._features_rest):
            p.add_(0.5)
            model.optimizer.state[p]["step"].add_(1)


@pytest.mark.parametrize("scenario", ["consumed", "native", "double-update", "silent-write",
                                      "skipped"])
def test_trace_checks_once_only_updates(tmp_path, scenario):
    import integration
    from routing import RoutingSummary

    options = SimpleNamespace(densify_until_iter=0, densify_from_iter=0,
                              densification_interval=100, opacity_reset_interval=3000,
                              iterations=30000 if scenario != "skipped" else 5)
    model = _trace_model()
    trace = tmp_path / "trace.json"
    integration.TRACE = str(trace)
    try:
        with RoutingSummary(tmp_path / "routing.json", {}) as summary:
            integration.SUMMARY = summary
            policy = integration.begin_step(model, 7, options,
                                            SimpleNamespace(white_background=False), (), (),
                                            True)
            assert policy.reason() == (None if scenario != "skipped"
                                       else "optimizer step skipped")
            model._clad_consumer = _FakeSH(scenario in ("consumed", "double-update"))
            model._clad_routing["sh_called"] = True
            if scenario in ("consumed", "double-update", "silent-write"):
                _consume(model)
            loss = torch.tensor(1.25)
            if scenario == "silent-write":
                with pytest.raises(AssertionError, match="changed without consumption"):
                    integration.after_backward(model, 7, loss)
                return
            integration.after_backward(model, 7, loss)
            if scenario == "double-update":
                with torch.no_grad():
                    model._features_rest.add_(1)
                with pytest.raises(AssertionError, match="updated twice"):
                    integration.after_step(model, 7)
                return
            integration.after_step(model, 7)
    finally:
        integration.TRACE = integration.SUMMARY = None
    assert model._clad_consumer is not None
    row = json.loads(trace.read_text())[0]
    assert row["iteration"] == 7 and row["loss"] == 1.25 and row["degree"] == 3
    assert row["counters_before"] == [4, 4]
    consumed = scenario == "consumed"
    assert row["consumed"] is consumed
    assert row["counters_after_backward"] == ([5, 5] if consumed else [4, 4])
    assert row["counters_after_step"] == row["counters_after_backward"]
    assert row["moment_shapes"] == [[3, 1, 3], [3, 15, 3]]
    assert set(row) == {"iteration", "enabled", "policy_reason", "count_before", "degree",
                        "counters_before", "consumed", "loss", "counters_after_backward",
                        "count_after", "counters_after_step", "moment_shapes"}
    routing = json.loads((tmp_path / "routing.json").read_text())
    assert routing["sh"]["consumed_steps"] == int(consumed)
    if not consumed:
        expected = ("optimizer step skipped" if scenario == "skipped"
                    else "unsupported optimizer")
        assert routing["sh"]["fallback_reasons"] == {expected: 1}
    assert routing["activations"]["fallback_reasons"] == {"activation consumption disabled": 1}
