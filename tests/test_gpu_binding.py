"""Trainer-facing lifecycle on CUDA tensors: SH binding, activation binding and
fused-Adam setup. Cases follow the reference's check.py:304-497 (activation
binding), 501-622 (SH binding) and 625-672 (optimizer setup).
"""

import copy
import math
from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu


# ---------------------------------------------------------------- SH binding

def _sh_setup(device):
    from adapter import DenseSHConsumer

    dc = torch.nn.Parameter(torch.zeros((2, 1, 3), device=device))
    rest = torch.nn.Parameter(torch.zeros((2, 15, 3), device=device))
    optimizer = torch.optim.Adam([dict(params=[dc], name="f_dc", lr=0.0025),
                                  dict(params=[rest], name="f_rest", lr=0.000125)],
                                 eps=1e-15, fused=True, foreach=False)
    for parameter in (dc, rest):
        optimizer.state[parameter] = dict(step=torch.zeros((), device=device),
                                          exp_avg=torch.zeros_like(parameter),
                                          exp_avg_sq=torch.zeros_like(parameter))
    return dc, rest, optimizer, DenseSHConsumer(optimizer, native=None, extension=None)


def _sh_capture(dc, rest, optimizer):
    return [v for p in (dc, rest)
            for v in (p, *[x for x in optimizer.state[p].values() if torch.is_tensor(x)])]


@pytest.mark.parametrize("case", ["parameter", "state", "moment", "moment-write", "counter",
                                  "options", "group", "gradient", "frozen"])
def test_sh_ownership_change_rejected_before_write(cuda, case):
    from adapter import StepPolicy

    dc, rest, optimizer, consumer = _sh_setup(cuda)
    frame = consumer.bind(dc, rest, StepPolicy())
    if case == "parameter":
        with torch.no_grad():
            dc.add_(1)
    elif case == "state":
        optimizer.state[dc] = dict(optimizer.state[dc])
    elif case == "moment":
        optimizer.state[dc]["exp_avg"] = optimizer.state[dc]["exp_avg"].clone()
    elif case == "moment-write":
        optimizer.state[dc]["exp_avg"].add_(1)
    elif case == "counter":
        optimizer.state[dc]["step"].add_(1)
    elif case == "options":
        optimizer.param_groups[0]["lr"] = 0.1
    elif case == "group":
        optimizer.param_groups[0] = dict(optimizer.param_groups[0])
    elif case == "gradient":
        dc.grad = torch.ones_like(dc)
    elif case == "frozen":
        dc.requires_grad_(False)
    values = _sh_capture(dc, rest, optimizer)
    before = [v.detach().clone() for v in values]
    versions = [v._version for v in values]
    with pytest.raises(RuntimeError):
        frame.validate()
    for value, previous, version in zip(values, before, versions):
        assert torch.equal(value, previous) and value._version == version


@pytest.mark.parametrize("case", ["moment-alias", "cross-group", "counter-alias",
                                  "shared-counter", "counter-device", "counter-dtype",
                                  "counter-shape", "counter-missing", "counter-nan",
                                  "counter-negative", "counter-fraction", "counter-overflow",
                                  "tensor-rate"])
def test_sh_invalid_state_falls_back_untouched(cuda, case):
    from adapter import StepPolicy

    dc, rest, optimizer, consumer = _sh_setup(cuda)
    state = optimizer.state[dc]
    if case == "moment-alias":
        state["exp_avg"] = state["exp_avg_sq"]
    elif case == "cross-group":
        state["exp_avg"] = rest.detach().reshape(-1)[:dc.numel()].view_as(dc)
    elif case == "counter-alias":
        state["step"] = dc.detach().reshape(-1)[0]
    elif case == "shared-counter":
        optimizer.state[rest]["step"] = state["step"]
    elif case == "counter-device":
        state["step"] = torch.zeros(())
    elif case == "counter-dtype":
        state["step"] = state["step"].double()
    elif case == "counter-shape":
        state["step"] = torch.zeros(2, device=cuda)
    elif case == "counter-missing":
        del state["step"]
    elif case.startswith("counter-"):
        state["step"].fill_({"counter-nan": math.nan, "counter-negative": -1,
                             "counter-fraction": 0.5, "counter-overflow": 2**24}[case])
    else:
        optimizer.param_groups[0]["lr"] = torch.tensor(0.0025, device=cuda)
    values = _sh_capture(dc, rest, optimizer)
    before = [v.detach().clone() for v in values]
    versions = [v._version for v in values]
    assert consumer.bind(dc, rest, StepPolicy()) is None
    assert consumer.active is None and consumer.last_reason
    for value, previous, version in zip(values, before, versions):
        torch.testing.assert_close(value, previous, rtol=0, atol=0, equal_nan=True)
        assert value._version == version


def test_sh_counter_and_version_advance(cuda):
    from adapter import StepPolicy

    dc, rest, optimizer, consumer = _sh_setup(cuda)
    for state in optimizer.state.values():
        state["step"].fill_(99)
    frame = consumer.bind(dc, rest, StepPolicy())
    frame.validate()
    writable = [dc, rest, *[v for pair in frame.moments.values() for v in pair]]
    versions = [v._version for v in writable]
    assert frame.iteration == 100
    frame.finish()
    assert all(v._version == version + 1 for v, version in zip(writable, versions))
    assert all(int(state["step"]) == 100 for state in optimizer.state.values())
    before = [v.detach().clone() for v in _sh_capture(dc, rest, optimizer)]
    optimizer.step()  # consumed groups have no .grad: native Adam skips them
    for value, previous in zip(_sh_capture(dc, rest, optimizer), before):
        assert torch.equal(value, previous)
    with pytest.raises(RuntimeError):
        frame.validate()
    consumer.end_step()
    assert consumer.bind(dc, rest, StepPolicy()).iteration == 101
    for policy in (StepPolicy(topology_change=True), StepPolicy(optimizer_step=False)):
        dc, rest, optimizer, consumer = _sh_setup(cuda)
        optimizer.state.clear()
        assert consumer.bind(dc, rest, policy) is None and not optimizer.state


# -------------------------------------------------------- activation binding

def _activation_model(device):
    model = SimpleNamespace()
    groups = []
    for name, attr, width, rate in zip(("rotation", "scaling", "opacity"),
                                       ("_rotation", "_scaling", "_opacity"), (4, 3, 1),
                                       (0.001, 0.005, 0.025)):
        raw = torch.nn.Parameter(torch.randn((35, width), device=device))
        setattr(model, attr, raw)
        groups.append(dict(name=name, params=[raw], lr=rate))
    model.optimizer = torch.optim.Adam(groups, eps=1e-15, fused=True, foreach=False)
    for group, counter in zip(model.optimizer.param_groups, (99, 3, 29854)):
        raw = group["params"][0]
        model.optimizer.state[raw] = dict(step=torch.tensor(float(counter), device=device),
                                          exp_avg=torch.randn_like(raw) * 0.02,
                                          exp_avg_sq=torch.rand_like(raw) * 0.03)
    return model


def _activation_capture(model):
    values = []
    for group in model.optimizer.param_groups:
        raw = group["params"][0]
        state = model.optimizer.state[raw]
        values.extend([raw] + [state[k] for k in ("exp_avg", "exp_avg_sq", "step")])
    return [v.detach().clone() for v in values]


def _unchanged(model, before):
    for actual, expected in zip(_activation_capture(model), before):
        assert torch.equal(actual, expected)


def test_activation_binding_matches_torch_fused_adam(cuda):
    import clad_quaternion
    from activation import ATTRS, DenseActivationConsumer
    from adapter import StepPolicy
    from normalization import normalize_quaternion

    torch.manual_seed(42)
    model, reference = _activation_model(cuda), _activation_model(cuda)
    with torch.no_grad():
        for group, ref_group in zip(model.optimizer.param_groups,
                                    reference.optimizer.param_groups):
            raw, ref = group["params"][0], ref_group["params"][0]
            ref.copy_(raw)
            for key, val in model.optimizer.state[raw].items():
                reference.optimizer.state[ref][key].copy_(val)
    expected_outputs = (normalize_quaternion(reference._rotation, clad_quaternion),
                        reference._scaling.exp(), reference._opacity.sigmoid())
    consumer = DenseActivationConsumer(clad_quaternion)
    actual_outputs = consumer.bind(model, StepPolicy(), exclusive_use=True)
    for actual, expected in zip(actual_outputs, expected_outputs):
        assert torch.equal(actual, expected)
    seeds = [torch.randn_like(v) * 0.001 for v in actual_outputs]
    torch.autograd.backward(expected_outputs, seeds)
    reference.optimizer.step()
    torch.autograd.backward(actual_outputs, seeds, retain_graph=True)
    assert consumer.active.consumed
    for attr, counter in zip(ATTRS, (100, 4, 29855)):
        raw = getattr(model, attr)
        assert raw.grad is None
        assert int(model.optimizer.state[raw]["step"]) == counter
    for actual, expected in zip(_activation_capture(model), _activation_capture(reference)):
        torch.testing.assert_close(actual, expected, rtol=3e-6, atol=2e-7)
    before = _activation_capture(model)
    model.optimizer.step()
    _unchanged(model, before)
    with pytest.raises(RuntimeError):
        torch.autograd.backward(actual_outputs, seeds)
    _unchanged(model, before)


@pytest.mark.parametrize("invalid", ["higher-order", "missing-seed", "late-gradient",
                                     "late-freeze", "parameter", "state", "counter",
                                     "options", "group"])
def test_activation_unsafe_backward_rejected(cuda, invalid):
    import clad_quaternion
    from activation import DenseActivationConsumer
    from adapter import StepPolicy

    model = _activation_model(cuda)
    consumer = DenseActivationConsumer(clad_quaternion)
    outputs = consumer.bind(model, StepPolicy(), exclusive_use=True)
    if invalid == "late-gradient":
        model._opacity.grad = torch.ones_like(model._opacity)
    if invalid == "late-freeze":
        model._opacity.requires_grad_(False)
    if invalid == "parameter":
        model._scaling = torch.nn.Parameter(model._scaling.detach().clone())
    if invalid == "state":
        state = model.optimizer.state[model._opacity]
        state["exp_avg"] = state["exp_avg"].clone()
    if invalid == "counter":
        model.optimizer.state[model._scaling]["step"].add_(1)
    if invalid == "options":
        model.optimizer.param_groups[1]["eps"] = 1e-8
    if invalid == "group":
        model.optimizer.param_groups[1] = dict(model.optimizer.param_groups[1])
    before = _activation_capture(model)
    with pytest.raises(RuntimeError):
        if invalid == "higher-order":
            torch.autograd.grad(sum(v.sum() for v in outputs), model._rotation,
                                create_graph=True)
        elif invalid == "missing-seed":
            outputs[0].sum().backward()
        else:
            torch.autograd.backward(outputs, [torch.ones_like(v) for v in outputs])
    _unchanged(model, before)


FALLBACKS = ("disabled", "skipped", "topology", "observation", "accumulation", "scaled",
             "exclusive", "processing", "declared-higher", "optimizer", "foreach", "frozen",
             "accumulated", "learning-rate", "moment-alias", "counter-alias", "shared-counter")


@pytest.mark.parametrize("case", FALLBACKS)
def test_activation_fallback_leaves_state_alone(cuda, case):
    import clad_quaternion
    from activation import DenseActivationConsumer
    from adapter import StepPolicy

    model = _activation_model(cuda)
    policy, flags = StepPolicy(), dict(exclusive_use=True)
    policy = {"disabled": None, "skipped": StepPolicy(optimizer_step=False),
              "topology": StepPolicy(topology_change=True),
              "observation": StepPolicy(observation_before_step=True),
              "accumulation": StepPolicy(single_backward=False),
              "scaled": StepPolicy(unscaled_gradients=False)}.get(case, policy)
    if case == "exclusive":
        flags["exclusive_use"] = False
    if case == "processing":
        flags["gradient_processing"] = True
    if case == "declared-higher":
        flags["higher_order"] = True
    if case == "optimizer":
        model.optimizer = torch.optim.SGD(model.optimizer.param_groups, lr=0.01)
    if case == "foreach":
        model.optimizer.param_groups[1]["foreach"] = True
    if case == "frozen":
        model._scaling.requires_grad_(False)
    if case == "accumulated":
        model._opacity.grad = torch.ones_like(model._opacity)
    if case == "learning-rate":
        model.optimizer.param_groups[1]["lr"] = torch.tensor(0.005, device=cuda)
    if case == "moment-alias":
        model.optimizer.state[model._scaling]["exp_avg"] = \
            model._rotation.view(-1)[:105].view(35, 3)
    if case == "counter-alias":
        with torch.no_grad():
            model._opacity[0].zero_()
        model.optimizer.state[model._opacity]["step"] = model._opacity.view(-1)[:1]
    if case == "shared-counter":
        step = torch.zeros((), device=cuda)
        for state in model.optimizer.state.values():
            state["step"] = step
    if case not in ("moment-alias", "counter-alias", "shared-counter"):
        model.optimizer.state.clear()
    before = [p.detach().clone() for p in (model._rotation, model._scaling, model._opacity)]
    keys = list(model.optimizer.state)
    old_state = _activation_capture(model) if keys else None
    consumer = DenseActivationConsumer(clad_quaternion)
    assert consumer.bind(model, policy, **flags) is None
    assert consumer.last_reason and consumer.active is None
    assert list(model.optimizer.state) == keys
    if old_state is not None:
        _unchanged(model, old_state)
    for raw, previous in zip((model._rotation, model._scaling, model._opacity), before):
        assert torch.equal(raw, previous)


def test_activation_fresh_state_counts_from_zero(cuda):
    import clad_quaternion
    from activation import ATTRS, DenseActivationConsumer
    from adapter import StepPolicy

    model = _activation_model(cuda)
    model.optimizer.state.clear()
    consumer = DenseActivationConsumer(clad_quaternion)
    for expected in (1, 2):
        outputs = consumer.bind(model, StepPolicy(), exclusive_use=True)
        torch.autograd.backward(outputs, [torch.ones_like(v) for v in outputs])
        assert [int(model.optimizer.state[getattr(model, a)]["step"]) for a in ATTRS] == \
            [expected] * 3
        consumer.end_step()
        assert consumer.active is None
        model.optimizer.zero_grad(set_to_none=True)


# ------------------------------------------------------------ optimizer setup

def test_fused_adam_preserves_state_and_matches_native(cuda):
    from optimizer_setup import fused_adam

    parameter = torch.nn.Parameter(torch.tensor([1., -2.], device=cuda))
    original = torch.optim.Adam([dict(params=[parameter], name="probe")], lr=.003,
                                eps=1e-15, foreach=False, fused=False)
    parameter.grad = torch.tensor([.2, -.4], device=cuda)
    original.step()
    saved = copy.deepcopy(original.state_dict())
    before = parameter.detach().clone()
    selected = fused_adam(original)
    group = selected.param_groups[0]
    assert group["params"][0] is parameter and group["lr"] == .003
    assert group["fused"] is True and group["foreach"] is False
    state, prior = selected.state[parameter], saved["state"][0]
    assert state["step"].device == parameter.device
    assert torch.equal(state["step"].cpu(), prior["step"].cpu())
    assert torch.equal(state["exp_avg"], prior["exp_avg"])
    assert torch.equal(state["exp_avg_sq"], prior["exp_avg_sq"])
    assert torch.equal(parameter, before)
    assert original.param_groups[0]["fused"] is False
    other = torch.nn.Parameter(before.clone())
    reference = torch.optim.Adam([dict(params=[other], name="probe")], lr=.003, eps=1e-15,
                                 fused=True, foreach=False)
    for g in saved["param_groups"]:
        g.update(fused=True, foreach=False)
    reference.load_state_dict(saved)
    parameter.grad = torch.tensor([-.3, .1], device=cuda)
    other.grad = parameter.grad.clone()
    selected.step()
    reference.step()
    assert torch.equal(parameter, other)
    for key in ("step", "exp_avg", "exp_avg_sq"):
        assert torch.equal(selected.state[parameter][key], reference.state[other][key])
    for unsupported in (torch.optim.SGD([parameter], lr=.1),
                        torch.optim.Adam([torch.nn.Parameter(torch.ones(2))])):
        with pytest.raises(ValueError):
            fused_adam(unsupported)
