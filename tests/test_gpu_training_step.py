"""A full training step through the trainer hooks (integration.py), consumed vs
native.

The model is a stand-in for the trainer's GaussianModel (the same attribute
names and optimizer groups); `render` follows the patched trainer's render()
(trainer.patch:22-47). One step through the consumed path (activation consumer
+ SH consumer inside the rasterizer backward + the optimizer's own step for the
remaining groups) must leave the same parameters and Adam state as the native
path (rasterizer backward + torch fused Adam on every group), within the
reference's consume-vs-native tolerance (check.py:1011: rtol 3e-5, atol 2e-7);
SH elements whose gradient is zero up to rounding may flip the sign of their
first Adam update.
"""

import json
from types import SimpleNamespace

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

OPTIONS = SimpleNamespace(densify_until_iter=15000, densify_from_iter=500,
                          densification_interval=100, opacity_reset_interval=3000,
                          iterations=30000)
DATASET = SimpleNamespace(white_background=False)
RATES = dict(xyz=0.00016, f_dc=0.0025, f_rest=0.000125, opacity=0.025, scaling=0.005,
             rotation=0.001)


class Model(SimpleNamespace):
    @property
    def get_xyz(self):
        return self._xyz


def make_model(scene, device):
    from optimizer_setup import fused_adam

    P = scene["P"]
    t = lambda a: torch.as_tensor(np.ascontiguousarray(a), dtype=torch.float32, device=device)
    sh = t(scene["sh"]).reshape(P, 16, 3)
    m = Model(
        _xyz=torch.nn.Parameter(t(scene["means"])),
        _features_dc=torch.nn.Parameter(sh[:, :1].contiguous().clone()),
        _features_rest=torch.nn.Parameter(sh[:, 1:].contiguous().clone()),
        _scaling=torch.nn.Parameter(torch.log(t(scene["scales"]))),
        _rotation=torch.nn.Parameter(t(scene["rotations"]) * 1.7),
        _opacity=torch.nn.Parameter(torch.logit(t(scene["opacities"]).reshape(P, 1))),
        active_sh_degree=3)
    groups = [dict(params=[m._xyz], lr=RATES["xyz"], name="xyz"),
              dict(params=[m._features_dc], lr=RATES["f_dc"], name="f_dc"),
              dict(params=[m._features_rest], lr=RATES["f_rest"], name="f_rest"),
              dict(params=[m._opacity], lr=RATES["opacity"], name="opacity"),
              dict(params=[m._scaling], lr=RATES["scaling"], name="scaling"),
              dict(params=[m._rotation], lr=RATES["rotation"], name="rotation")]
    m.optimizer = fused_adam(torch.optim.Adam(groups, lr=0.0, eps=1e-15))
    return m


def render(model, settings, policy):
    import integration
    import rasterizer

    means2d = torch.zeros_like(model._xyz, requires_grad=True)
    activated = integration.activate_consumer(model, policy, eligible=True)
    if activated is not None:
        rotation, scale, opacity = activated
    else:
        opacity = torch.sigmoid(model._opacity)
        scale = torch.exp(model._scaling)
        rotation = torch.nn.functional.normalize(model._rotation)
    if policy is not None:
        return integration.render_consumer(model, model._xyz, means2d, opacity, scale, rotation,
                                           settings, policy)
    return rasterizer.GaussianRasterizer(settings)(
        means3D=model._xyz, means2D=means2d, opacities=opacity,
        shs=torch.cat((model._features_dc, model._features_rest), 1), scales=scale,
        rotations=rotation)


def train_step(model, settings, target, iteration, enabled):
    import integration

    policy = integration.begin_step(model, iteration, OPTIONS, DATASET, (), (), enabled)
    image, radii, depth = render(model, settings, policy)
    loss = ((image - target) ** 2).sum()
    loss.backward()
    integration.after_backward(model, iteration, loss)
    model.optimizer.step()
    model.optimizer.zero_grad(set_to_none=True)
    integration.after_step(model, iteration)


def _state(model):
    out = {}
    for name in ("_xyz", "_features_dc", "_features_rest", "_opacity", "_scaling", "_rotation"):
        p = getattr(model, name)
        st = model.optimizer.state[p]
        out[name] = (p.detach().clone(), st["exp_avg"].clone(), st["exp_avg_sq"].clone(),
                     int(st["step"].item()))
    return out


@pytest.mark.parametrize("position", [False, True])
def test_consumed_training_step_matches_native(cuda, tmp_path, position):
    """With `position` the xyz group is consumed too (integration.POSITION)."""
    import clad_quaternion
    import integration
    import rasterizer
    from routing import RoutingSummary

    scene = oracle.raster_scene(512, 64, 96, seed=21)
    settings = rasterizer.GaussianRasterizationSettings(
        image_height=64, image_width=96, tanfovx=scene["tanx"], tanfovy=scene["tany"],
        bg=torch.tensor(scene["bg"], dtype=torch.float32, device=cuda), scale_modifier=1.0,
        viewmatrix=torch.tensor(scene["view"], dtype=torch.float32, device=cuda),
        projmatrix=torch.tensor(scene["proj"], dtype=torch.float32, device=cuda), sh_degree=3,
        campos=torch.tensor(scene["campos"], dtype=torch.float32, device=cuda),
        prefiltered=False, debug=False)
    torch.manual_seed(0)
    target = torch.rand(3, 64, 96, device=cuda)
    consumed, native = make_model(scene, cuda), make_model(scene, cuda)
    integration.ACTIVATION_EXTENSION = clad_quaternion
    integration.TRACE = str(tmp_path / "trace.json")
    integration.POSITION = position
    try:
        with RoutingSummary(tmp_path / "routing.json", dict(test=True)) as summary:
            integration.SUMMARY = summary
            train_step(consumed, settings, target, 7, enabled=True)
        integration.SUMMARY = None
        integration.TRACE = None
        train_step(native, settings, target, 7, enabled=False)
        consumer = consumed._clad_consumer
        assert consumer.position_reason is None or not position, consumer.position_reason
    finally:
        integration.SUMMARY = integration.TRACE = None
        integration.ACTIVATION_EXTENSION = None
        integration.POSITION = False
    torch.cuda.synchronize()
    if position:
        # The kernel updated xyz, so the optimizer never saw a position gradient.
        assert consumed._xyz.grad is None
    routing = json.loads((tmp_path / "routing.json").read_text())
    assert routing["status"] == "completed"
    assert routing["sh"]["consumed_steps"] == 1 and routing["activations"]["consumed_steps"] == 1
    trace = json.loads((tmp_path / "trace.json").read_text())
    assert trace[0]["consumed"] and trace[0]["activation"]["consumed"]
    a, b = _state(consumed), _state(native)
    for name in a:
        pa, ma, va, sa = a[name]
        pb, mb, vb, sb = b[name]
        assert sa == sb == 1, name
        torch.testing.assert_close(ma, mb, rtol=3e-5, atol=2e-7, msg=name + " exp_avg")
        torch.testing.assert_close(va, vb, rtol=3e-5, atol=2e-7, msg=name + " exp_avg_sq")
        close = (pa - pb).abs() <= 2e-7 + 3e-5 * pb.abs()
        # Step 1 updates are lr * sign(g): a rounding-level gradient may flip.
        tiny = mb.abs() <= 1e-5 * mb.abs().max()
        lr = RATES[{"_xyz": "xyz", "_features_dc": "f_dc", "_features_rest": "f_rest",
                    "_opacity": "opacity", "_scaling": "scaling", "_rotation": "rotation"}[name]]
        close |= tiny & ((pa - pb).abs() <= 2.0001 * lr)
        assert close.all(), (name, int((~close).sum()))
