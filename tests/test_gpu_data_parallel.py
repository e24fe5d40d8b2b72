"""The data-parallel step on the GPU.

* `clad3dgs_shard_update` bit for bit against the oracle, for 1, 2, 3 and 8
  ranks emulated on one GPU (separate gradient arrays and parameter replicas
  per rank, every share updated in turn), over consecutive steps, and with a
  share-sized gradient buffer (the collective path's form);
* the activation and L1-loss kernels against torch;
* one trainer step on one GPU against the same step through the autograd
  rasterizer front end, torch activations and torch fused Adam (the path's
  tolerances: rtol 3e-5 / atol 2e-7, Adam step-1 sign flips of rounding-level
  gradients allowed);
* the seed form of the exchange (colour seeds per view, the SH backward
  inside the update) bit-identical to the gradient form for 2, 3, 4 and 8
  ranks' views emulated on one GPU (the gradients formed from the same seeds by the
  rasterizer's SH backward: two backward passes differ in the order of their
  float atomics, so only shared inputs compare bit for bit); the trainer step
  in both forms against the autograd path;
* on two GPUs (skipped with fewer): both exchanges (peer memory, in seed and
  gradient form, and NCCL collectives), each rank's replica and moments
  bit-identical to the emulation of the same inputs.
"""

import os
import socket

import pytest
import torch

from dp_helpers import GROUP_NAMES, RATES, initial_values, oracle_update, saved_from

pytestmark = pytest.mark.gpu
RATE_TUPLE = tuple(RATES[r] for r in ("xyz", "f_dc", "f_rest", "scaling", "rotation",
                                      "opacity"))
WIDTHS = (3, 48, 3, 4, 1)


def _bias(t):
    return 1 - 0.9 ** t, (1 - 0.999 ** t) ** 0.5


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shard_update_matches_oracle(cuda, world):
    from data_parallel import ShardStep, native_update, plan

    n = 203
    padded, share = plan(n, world)
    values = initial_values(n)
    dev = lambda a: torch.as_tensor(a).to(cuda).contiguous()
    # Host copies (oracle) and device copies (kernel) of every replica.
    host_params = {k: torch.zeros(padded, w) for k, w in zip(GROUP_NAMES, WIDTHS)}
    for k in GROUP_NAMES:
        host_params[k][:n] = values[k].reshape(n, -1)
    replicas = [{k: dev(host_params[k]) for k in GROUP_NAMES} for _ in range(world)]
    zeros = lambda: {k: torch.zeros(share, w) for k, w in zip(GROUP_NAMES, WIDTHS)}
    host_m = [zeros() for _ in range(world)]
    host_v = [zeros() for _ in range(world)]
    dev_m = [{k: dev(t) for k, t in m.items()} for m in host_m]
    dev_v = [{k: dev(t) for k, t in v.items()} for v in host_v]
    for step in range(3):
        g = torch.Generator().manual_seed(step)
        grads = [{k: torch.randn(padded, w, generator=g) * 1e-3 for k, w in
                  zip(GROUP_NAMES, WIDTHS)} for _ in range(world)]
        saved = saved_from(host_params)
        saved_t = dict(scaling=torch.from_numpy(saved["scaling"]),
                       opacity=torch.from_numpy(saved["opacity"]).view(-1, 1),
                       norm=torch.from_numpy(saved["norm"]))
        saved_d = {k: dev(v) for k, v in saved_t.items()}
        dev_grads = [{k: dev(v) for k, v in gr.items()} for gr in grads]
        b1, b2 = _bias(step + 1)
        for r in range(world):
            common = dict(begin=r * share, end=(r + 1) * share, grad_origin=0, local=r,
                          rates=RATE_TUPLE, bias1=b1, bias2_sqrt=b2)
            oracle_update(ShardStep(
                grads=[[grads[q][k] for k in GROUP_NAMES] for q in range(world)],
                params=[[host_params[k] for k in GROUP_NAMES] for _ in range(world)],
                first=[host_m[r][k] for k in GROUP_NAMES],
                second=[host_v[r][k] for k in GROUP_NAMES], saved_scaling=saved_t["scaling"],
                saved_opacity=saved_t["opacity"], saved_norm=saved_t["norm"], **common))
            native_update(ShardStep(
                grads=[[dev_grads[q][k] for k in GROUP_NAMES] for q in range(world)],
                params=[[replicas[q][k] for k in GROUP_NAMES] for q in range(world)],
                first=[dev_m[r][k] for k in GROUP_NAMES],
                second=[dev_v[r][k] for k in GROUP_NAMES], saved_scaling=saved_d["scaling"],
                saved_opacity=saved_d["opacity"], saved_norm=saved_d["norm"], **common))
        torch.cuda.synchronize()
        for q in range(world):
            for k in GROUP_NAMES:
                assert torch.equal(replicas[q][k].cpu(), host_params[k]), (step, q, k)
        for r in range(world):
            for k in GROUP_NAMES:
                assert torch.equal(dev_m[r][k].cpu(), host_m[r][k]), (step, r, k)
                assert torch.equal(dev_v[r][k].cpu(), host_v[r][k]), (step, r, k)


def test_shard_update_from_a_reduced_share(cuda):
    """grad_origin = begin: gradients of the share only (after reduce-scatter)."""
    from data_parallel import ShardStep, native_update

    n, begin, end = 64, 16, 48
    values = initial_values(n)
    host = {k: values[k].reshape(n, -1).clone() for k in GROUP_NAMES}
    params = {k: v.to(cuda) for k, v in host.items()}
    g = torch.Generator().manual_seed(9)
    share = {k: torch.randn(end - begin, w, generator=g) * 1e-3 for k, w in
             zip(GROUP_NAMES, WIDTHS)}
    full = {k: torch.zeros(n, w) for k, w in zip(GROUP_NAMES, WIDTHS)}
    for k in GROUP_NAMES:
        full[k][begin:end] = share[k]
    saved = saved_from(host)
    saved_t = dict(scaling=torch.from_numpy(saved["scaling"]),
                   opacity=torch.from_numpy(saved["opacity"]).view(-1, 1),
                   norm=torch.from_numpy(saved["norm"]))
    m = {k: torch.zeros(end - begin, w) for k, w in zip(GROUP_NAMES, WIDTHS)}
    v = {k: torch.zeros(end - begin, w) for k, w in zip(GROUP_NAMES, WIDTHS)}
    md = {k: t.to(cuda) for k, t in m.items()}
    vd = {k: t.to(cuda) for k, t in v.items()}
    b1, b2 = _bias(1)
    oracle_update(ShardStep(begin, end, 0, [[full[k] for k in GROUP_NAMES]],
                            [[host[k] for k in GROUP_NAMES]], 0, [m[k] for k in GROUP_NAMES],
                            [v[k] for k in GROUP_NAMES], saved_t["scaling"],
                            saved_t["opacity"], saved_t["norm"], RATE_TUPLE, b1, b2))
    native_update(ShardStep(begin, end, begin, [[share[k].to(cuda) for k in GROUP_NAMES]],
                            [[params[k] for k in GROUP_NAMES]], 0,
                            [md[k] for k in GROUP_NAMES], [vd[k] for k in GROUP_NAMES],
                            saved_t["scaling"].to(cuda), saved_t["opacity"].to(cuda),
                            saved_t["norm"].to(cuda), RATE_TUPLE, b1, b2))
    torch.cuda.synchronize()
    for k in GROUP_NAMES:
        assert torch.equal(params[k].cpu(), host[k]), k
        assert torch.equal(md[k].cpu(), m[k]) and torch.equal(vd[k].cpu(), v[k]), k
    assert torch.equal(params["xyz"][:begin].cpu(), values["xyz"][:begin])


def test_shard_update_rejects_bad_ranges(cuda):
    from data_parallel import ShardStep, native_update

    t = torch.zeros(64, 48, device=cuda)
    row = [t] * 5
    bad = ShardStep(2, 34, 0, [row], [row], 0, row, row, t, t, t, RATE_TUPLE, 0.1, 0.03)
    with pytest.raises(ValueError, match="multiples of 4"):
        native_update(bad)
    with pytest.raises(ValueError, match="local replica"):
        native_update(bad._replace(begin=0, end=32, local=1))


def test_activate_and_l1_loss_kernels(cuda):
    import _native as native

    n = 1001
    v = initial_values(n, device=cuda)
    out = dict(scaling=torch.empty(n, 3, device=cuda), rotation=torch.empty(n, 4, device=cuda),
               opacity=torch.empty(n, 1, device=cuda), norm=torch.empty(n, device=cuda))
    v["rotation"][5] = 0.0  # clamp branch
    native.check(native.library().clad3dgs_activate(
        n, v["scaling"].data_ptr(), v["rotation"].data_ptr(), v["opacity"].data_ptr(),
        out["scaling"].data_ptr(), out["rotation"].data_ptr(), out["opacity"].data_ptr(),
        out["norm"].data_ptr(), native.stream_handle()), "activate")
    torch.testing.assert_close(out["scaling"], torch.exp(v["scaling"]), rtol=2e-7, atol=0)
    torch.testing.assert_close(out["opacity"], torch.sigmoid(v["opacity"]), rtol=4e-7, atol=0)
    torch.testing.assert_close(out["rotation"], torch.nn.functional.normalize(v["rotation"]),
                               rtol=4e-7, atol=1e-30)
    torch.testing.assert_close(out["norm"], v["rotation"].norm(dim=1), rtol=4e-7, atol=0)
    img = torch.rand(3, 37, 53, device=cuda)
    tgt = torch.rand(3, 37, 53, device=cuda)
    tgt[0, 0, 0] = img[0, 0, 0]
    x = img.clone().requires_grad_()
    ref = (x - tgt).abs().mean()
    ref.backward()
    dimg = torch.empty_like(img)
    loss = torch.zeros(1, device=cuda)
    native.check(native.library().clad3dgs_l1_loss(img.numel(), img.data_ptr(), tgt.data_ptr(),
                                                   dimg.data_ptr(), loss.data_ptr(),
                                                   native.stream_handle()), "l1")
    assert torch.equal(dimg, x.grad)
    torch.testing.assert_close(loss[0], ref.detach(), rtol=1e-5, atol=0)


def _small_scene(n, cuda):
    v = initial_values(n, seed=5)
    v["xyz"] = v["xyz"] * 0.6
    v["scaling"] = torch.rand(n, 3, generator=torch.Generator().manual_seed(6)) * 2 - 5
    return {k: t.to(cuda) for k, t in v.items()}


@pytest.mark.parametrize("sh_exchange", ["seeds", "grads"])
def test_trainer_step_on_one_gpu_matches_autograd_path(cuda, sh_exchange):
    import rasterizer
    from data_parallel import DataParallelTrainer, orbit_camera

    n, W, H = 3000, 96, 64
    values = _small_scene(n, cuda)
    cam = orbit_camera(1, 8, width=W, height=H, device=cuda)
    torch.manual_seed(1)
    target = torch.rand(3, H, W, device=cuda)
    trainer = DataParallelTrainer(values, RATES, device=cuda, sh_exchange=sh_exchange)
    assert trainer.adam.sh_exchange == sh_exchange
    loss, rendered = trainer.step(cam, target)
    assert rendered > 0
    if sh_exchange == "seeds":
        # Drawn Gaussians carry flag 1; padding Gaussians have no seed.
        flags = trainer.adam.seeds[:, 3]
        assert ((flags == 0) | (flags == 1)).all() and (flags[:n] == 1).any()
        assert (trainer.adam.seeds[n:] == 0).all()
    # The same step through the autograd front end and torch fused Adam.
    P = {k: torch.nn.Parameter(values[k].clone()) for k in ("xyz", "scaling", "rotation",
                                                             "opacity")}
    dc = torch.nn.Parameter(values["sh"].view(n, 16, 3)[:, :1].clone())
    rest = torch.nn.Parameter(values["sh"].view(n, 16, 3)[:, 1:].clone())
    opt = torch.optim.Adam([dict(params=[P["xyz"]], lr=RATES["xyz"]),
                            dict(params=[dc], lr=RATES["f_dc"]),
                            dict(params=[rest], lr=RATES["f_rest"]),
                            dict(params=[P["scaling"]], lr=RATES["scaling"]),
                            dict(params=[P["rotation"]], lr=RATES["rotation"]),
                            dict(params=[P["opacity"]], lr=RATES["opacity"])],
                           eps=1e-15, fused=True)
    settings = rasterizer.GaussianRasterizationSettings(
        image_height=H, image_width=W, tanfovx=cam.tan_x, tanfovy=cam.tan_y,
        bg=torch.zeros(3, device=cuda), scale_modifier=1.0, viewmatrix=cam.view,
        projmatrix=cam.proj, sh_degree=3, campos=cam.campos, prefiltered=False, debug=False)
    image, _radii, _depth = rasterizer.GaussianRasterizer(settings)(
        means3D=P["xyz"], means2D=torch.zeros_like(P["xyz"], requires_grad=True),
        opacities=torch.sigmoid(P["opacity"]), shs=torch.cat((dc, rest), 1),
        scales=torch.exp(P["scaling"]), rotations=torch.nn.functional.normalize(P["rotation"]))
    ref_loss = (image - target).abs().mean()
    ref_loss.backward()
    grads = {"xyz": P["xyz"].grad, "sh": torch.cat((dc.grad, rest.grad), 1).reshape(n, 48),
             "scaling": P["scaling"].grad, "rotation": P["rotation"].grad,
             "opacity": P["opacity"].grad}
    opt.step()
    torch.cuda.synchronize()
    torch.testing.assert_close(loss[0], ref_loss.detach(), rtol=1e-5, atol=0)
    got = trainer.adam.params
    expect = {"xyz": P["xyz"], "sh": torch.cat((dc, rest), 1).reshape(n, 48),
              "scaling": P["scaling"], "rotation": P["rotation"], "opacity": P["opacity"]}
    lr = {"xyz": RATES["xyz"], "sh": RATES["f_dc"], "scaling": RATES["scaling"],
          "rotation": RATES["rotation"], "opacity": RATES["opacity"]}
    for k in GROUP_NAMES:
        a, b = got[k][:n], expect[k].detach()
        close = (a - b).abs() <= 2e-7 + 3e-5 * b.abs()
        g = grads[k]
        tiny = g.abs() <= 1e-4 * g.abs().max()
        close |= tiny & ((a - b).abs() <= 2.0001 * lr[k])
        assert close.all(), (k, int((~close).sum()))
    moved = (got["xyz"][:n] != values["xyz"]).any(dim=1)
    assert moved.sum() > n // 4
    trainer.close()


@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_seed_form_matches_gradient_form_for_emulated_ranks(cuda, world):
    """`world` views rendered on one GPU stand for the ranks. From each view's
    seeds and geometry gradients, the rasterizer's own SH backward
    (`clad3dgs_raster_sh_backward`, at the current parameters) forms the full
    gradients; the seed-form update of every share then equals the
    gradient-form update, bit for bit, over consecutive steps."""
    import _native as native
    from data_parallel import (DataParallelTrainer, ShardStep, carve, native_update,
                               orbit_camera, plan)

    n, W, H = 2400, 96, 64  # padded alike for 1, 2, 3, 4 and 8 ranks
    padded, share = plan(n, world)
    assert padded == plan(n, 1)[0]
    values = _small_scene(n, cuda)
    trainer = DataParallelTrainer(values, RATES, device=cuda, sh_exchange="seeds")
    a = trainer.adam
    grads_s, seeds, cams = [], [], []
    for q in range(world):
        cam = orbit_camera((2 * q + 1) % 8, 8, width=W, height=H, device=cuda)
        target = torch.rand(3, H, W, device=cuda,
                            generator=torch.Generator(device=cuda).manual_seed(10 + q))
        trainer.backward(cam, target)
        grads_s.append(carve(a.grad_slab.clone(), padded))
        seeds.append(a.seeds.clone())
        cams.append(a.camera.clone())
    names = GROUP_NAMES
    replica_f = carve(a.param_slab.clone(), padded)
    replica_s = carve(a.param_slab.clone(), padded)
    saved = a.saved
    zeros = lambda: {k: torch.zeros(share, w, device=cuda) for k, w in zip(names, WIDTHS)}
    moments = [(zeros(), zeros(), zeros(), zeros()) for _ in range(world)]
    clamped = torch.zeros(n, 3, dtype=torch.bool, device=cuda)

    def gradient_form(q):
        """View q's full gradients at the current parameters: SH gradients
        and the direction adjoint from its seeds (drawn flag as radius,
        nothing clamped) added to its geometry gradients."""
        g_f = {k: v.clone() for k, v in grads_s[q].items()}
        radii = (seeds[q][:n, 3] != 0).to(torch.int32)
        dcolor = seeds[q][:n, :3].contiguous()
        native.check(native.library().clad3dgs_raster_sh_backward(
            n, 3, replica_f["xyz"].data_ptr(), radii.data_ptr(), replica_f["sh"].data_ptr(),
            None, None, cams[q].data_ptr(), clamped.data_ptr(), dcolor.data_ptr(),
            g_f["sh"].data_ptr(), g_f["xyz"].data_ptr(), native.stream_handle()),
            "SH backward")
        return g_f

    for step in range(2):
        b1, b2 = _bias(step + 1)
        grads_f = [gradient_form(q) for q in range(world)]
        for r in range(world):
            m_f, v_f, m_s, v_s = moments[r]
            common = dict(begin=r * share, end=(r + 1) * share, grad_origin=0, local=0,
                          saved_scaling=saved["scaling"], saved_opacity=saved["opacity"],
                          saved_norm=saved["norm"], rates=RATE_TUPLE, bias1=b1, bias2_sqrt=b2)
            native_update(ShardStep(
                grads=[[grads_f[q][k] for k in names] for q in range(world)],
                params=[[replica_f[k] for k in names]] * world,
                first=[m_f[k] for k in names], second=[v_f[k] for k in names], **common))
            native_update(ShardStep(
                grads=[[grads_s[q][k] for k in names] for q in range(world)],
                params=[[replica_s[k] for k in names]] * world,
                first=[m_s[k] for k in names], second=[v_s[k] for k in names],
                seeds=seeds, cameras=cams, degree=3, **common))
        torch.cuda.synchronize()
        for r in range(world):
            m_f, v_f, m_s, v_s = moments[r]
            for k in names:
                assert torch.equal(m_f[k], m_s[k]), (step, r, k)
                assert torch.equal(v_f[k], v_s[k]), (step, r, k)
        for k in names:
            assert torch.equal(replica_f[k], replica_s[k]), (step, k)
    # The updates moved the parameters, and SH gradients were not all zero.
    assert not torch.equal(replica_s["sh"], a.params["sh"])
    assert not torch.equal(replica_s["xyz"], a.params["xyz"])
    assert sum(int((g["sh"] != 0).sum()) for g in grads_f) > 0
    trainer.close()


def _clamping_scene(n, cuda):
    """The small scene with every fifth Gaussian's base colour pushed below
    zero in one channel (so the colour clamp cuts channels in every view)."""
    v = _small_scene(n, cuda)
    sh = v["sh"].view(n, 16, 3)
    idx = torch.arange(0, n, 5, device=cuda)
    sh[idx, 0, (idx // 5) % 3] = -2.5
    return v


def _unmasked_seeds(trainer, n):
    """This view's dL/dcolour with the drawn flag, no channel masked: what a
    rank renders from the owners' colours publishes."""
    a = trainer.adam
    u = torch.zeros_like(a.seeds)
    u[:n, :3] = trainer.scratch_grads["colors"]
    u[:n, 3] = (trainer.radii > 0).float()
    return u


@pytest.mark.parametrize("world,degree", [(1, 3), (2, 3), (4, 3), (8, 3), (2, 0), (4, 1),
                                          (3, 2)])
def test_colour_form_matches_seed_form_for_emulated_ranks(cuda, world, degree):
    """`world` views on one GPU stand for the ranks. The owners' first colours
    (`clad3dgs_shard_colours`) render each view exactly as the SH do; their
    clamp bits mask the unmasked seeds as each rank's clamp flags masked its
    seeds, so the colour-form update of every share equals the seed-form
    update bit for bit, over consecutive steps; the colours each update writes
    equal the colours made afresh from the updated parameters."""
    from data_parallel import DataParallelTrainer, ShardStep, carve, native_colours, native_update
    from data_parallel import orbit_camera, plan

    n, W, H = 2400, 96, 64
    padded, share = plan(n, world)
    values = _clamping_scene(n, cuda)
    seeded = DataParallelTrainer(values, RATES, device=cuda, sh_exchange="seeds",
                                 degree=degree)
    coloured = DataParallelTrainer(values, RATES, device=cuda, sh_exchange="colours",
                                   degree=degree)
    a = seeded.adam
    grads, masked, unmasked, cams, images = [], [], [], [], []
    for q in range(world):
        cam = orbit_camera((2 * q + 1) % 8, 8, width=W, height=H, device=cuda)
        target = torch.rand(3, H, W, device=cuda,
                            generator=torch.Generator(device=cuda).manual_seed(10 + q))
        seeded.backward(cam, target)
        grads.append(carve(a.grad_slab.clone(), padded))
        masked.append(a.seeds.clone())
        unmasked.append(_unmasked_seeds(seeded, n))
        cams.append(a.camera.clone())
        images.append((cam, target, seeded.image.clone()))
    names = GROUP_NAMES
    replica_s = carve(a.param_slab.clone(), padded)
    replica_c = carve(a.param_slab.clone(), padded)
    saved = a.saved
    colours = [torch.zeros(padded, 3, device=cuda) for _ in range(world)]
    bits = torch.zeros(padded, dtype=torch.int32, device=cuda)

    def shares(replica, **extra):
        for r in range(world):
            yield ShardStep(begin=r * share, end=(r + 1) * share, grad_origin=0,
                            grads=[[grads[q][k] for k in names] for q in range(world)],
                            params=[[replica[k] for k in names]] * world, local=0,
                            first=[None] * 5, second=[None] * 5,
                            saved_scaling=saved["scaling"],
                            saved_opacity=saved["opacity"], saved_norm=saved["norm"],
                            rates=RATE_TUPLE, bias1=1.0, bias2_sqrt=1.0, degree=degree,
                            **extra), r

    def prime(replica, out, out_bits):
        for step, r in shares(replica, colours=out, next_cameras=cams):
            native_colours(step._replace(clamp_bits=out_bits[r * share:(r + 1) * share]))

    prime(replica_c, colours, bits)
    torch.cuda.synchronize()
    # The colours render every view as its SH do (the rasterizer's own pass).
    for q, (cam, target, image) in enumerate(images):
        coloured.adam.colours.copy_(colours[q])
        coloured.backward(cam, target)
        assert torch.equal(coloured.image, image), q
    assert int((bits != 0).sum()) > n // 20
    zeros = lambda: {k: torch.zeros(share, w, device=cuda) for k, w in zip(names, WIDTHS)}
    moments = [(zeros(), zeros(), zeros(), zeros()) for _ in range(world)]
    for step in range(2):
        b1, b2 = _bias(step + 1)
        if step:
            # Seed form: each view's seeds masked by its clamp flags at the
            # current parameters (the bits the colour form keeps).
            masked = [u.clone() for u in unmasked]
            for q in range(world):
                for k in range(3):
                    cut = (bits >> (3 * q + k)) & 1 == 1
                    masked[q][:, k] = torch.where(cut, 0.0, masked[q][:, k])
        for (s_step, r), (c_step, _) in zip(shares(replica_s), shares(replica_c)):
            m_s, v_s, m_c, v_c = moments[r]
            native_update(s_step._replace(first=[m_s[k] for k in names],
                                          second=[v_s[k] for k in names],
                                          bias1=b1, bias2_sqrt=b2, seeds=masked,
                                          cameras=cams))
            native_update(c_step._replace(first=[m_c[k] for k in names],
                                          second=[v_c[k] for k in names],
                                          bias1=b1, bias2_sqrt=b2, seeds=unmasked,
                                          cameras=cams, colours=colours, next_cameras=cams,
                                          clamp_bits=bits[r * share:(r + 1) * share]))
        torch.cuda.synchronize()
        for r in range(world):
            m_s, v_s, m_c, v_c = moments[r]
            for k in names:
                assert torch.equal(m_s[k], m_c[k]), (step, r, k)
                assert torch.equal(v_s[k], v_c[k]), (step, r, k)
        for k in names:
            assert torch.equal(replica_s[k], replica_c[k]), (step, k)
        fresh = [torch.zeros(padded, 3, device=cuda) for _ in range(world)]
        fresh_bits = torch.zeros_like(bits)
        prime(replica_c, fresh, fresh_bits)
        torch.cuda.synchronize()
        for q in range(world):
            assert torch.equal(colours[q][:n], fresh[q][:n]), (step, q)
        assert torch.equal(bits, fresh_bits), step
    assert not torch.equal(replica_c["sh"], a.params["sh"])
    seeded.close()
    coloured.close()


def test_colour_form_trainer_renders_the_updated_parameters(cuda):
    """The colour-form trainer on one GPU: each step renders, from the
    colours the previous update made for the declared camera, the image the
    autograd front end renders from the current SH coefficients; a step whose
    camera is not the declared one, or without a next camera, is refused."""
    import rasterizer
    from data_parallel import DataParallelTrainer, orbit_camera

    n, W, H = 3000, 96, 64
    values = _clamping_scene(n, cuda)
    trainer = DataParallelTrainer(values, RATES, device=cuda, sh_exchange="colours")
    a = trainer.adam
    views = [orbit_camera(v, 8, width=W, height=H, device=cuda) for v in (1, 4, 6, 3)]
    torch.manual_seed(2)
    targets = [torch.rand(3, H, W, device=cuda) for _ in views]
    with pytest.raises(ValueError):
        trainer.step(views[0], targets[0])
    trainer.step(views[0], targets[0], next_camera=views[1])
    with pytest.raises(ValueError):
        trainer.step(views[2], targets[2], next_camera=views[3])
    for t in (1, 2):
        cam = views[t]
        trainer.backward(cam, targets[t])
        got = trainer.image.clone()
        p, act = a.params, a.saved
        settings = rasterizer.GaussianRasterizationSettings(
            image_height=H, image_width=W, tanfovx=cam.tan_x, tanfovy=cam.tan_y,
            bg=torch.zeros(3, device=cuda), scale_modifier=1.0, viewmatrix=cam.view,
            projmatrix=cam.proj, sh_degree=3, campos=cam.campos, prefiltered=False,
            debug=False)
        with torch.no_grad():
            image, _radii, _depth = rasterizer.GaussianRasterizer(settings)(
                means3D=p["xyz"][:n], means2D=torch.zeros(n, 3, device=cuda),
                opacities=act["opacity"][:n], shs=p["sh"][:n].view(n, 16, 3),
                scales=act["scaling"][:n], rotations=act["rotation"][:n])
        assert torch.equal(got, image), t
        # The rest of the step, with the next camera declared.
        a.next_camera.copy_(views[t + 1].campos)
        a.step()
        trainer._declared = views[t + 1]
    moved = (a.params["xyz"][:n] != values["xyz"]).any(dim=1)
    assert moved.sum() > n // 4
    # A checkpoint restores the step: a fresh trainer primes the declared
    # camera's colours from it and renders the same image.
    state = trainer.state_dict()
    assert state["t"] == a.t
    resumed = DataParallelTrainer(_clamping_scene(n, cuda), RATES, device=cuda,
                                  sh_exchange="colours")
    resumed.load_state_dict(state)
    resumed.prime(views[3])
    trainer.backward(views[3], targets[3])
    resumed.backward(views[3], targets[3])
    assert torch.equal(resumed.image, trainer.image)
    for k in GROUP_NAMES:
        assert torch.equal(resumed.adam.params[k][:n], a.params[k][:n]), k
    resumed.close()
    trainer.close()


def test_seed_form_rejects_bad_arguments(cuda):
    from data_parallel import DataParallelTrainer, ShardedAdam, native_update

    with pytest.raises(ValueError):
        ShardedAdam(64, RATES, device="cpu", sh_exchange="seeds")
    with pytest.raises(ValueError):
        ShardedAdam(64, RATES, device=cuda, sh_exchange="colors")
    with pytest.raises(ValueError):
        ShardedAdam(64, RATES, device="cpu", sh_exchange="colours")
    trainer = DataParallelTrainer(_small_scene(64, cuda), RATES, device=cuda)
    a = trainer.adam
    a.t = 1
    step = a._shard_step([[a.grads[k] for k in GROUP_NAMES]],
                         [[a.params[k] for k in GROUP_NAMES]], 0, 0, [a.seeds], [a.camera])
    with pytest.raises(ValueError):
        native_update(step._replace(degree=4))
    with pytest.raises(ValueError):
        native_update(step._replace(seeds=[a.seeds.view(-1)[1:]]))  # misaligned
    with pytest.raises(ValueError):
        native_update(step._replace(grad_origin=4, begin=4))
    trainer.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _dp_worker(rank, world, port, exchange, sh_exchange, out_dir, size="small"):
    from datetime import timedelta

    import torch.distributed as dist
    from data_parallel import DataParallelTrainer, ShardStep, carve, native_update, orbit_camera

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=timedelta(seconds=120), device_id=device)
    trainer = None
    try:
        if size == "small":
            n, W, H = 2003, 96, 64
            values = _small_scene(n, device)
        else:
            # The 8-view training configuration: 6,000,000 Gaussians, 1920x1080 views.
            from bench import train_values

            n, W, H = 6_000_000, 1920, 1080
            values = train_values(n, device, seed=3)
        trainer = DataParallelTrainer(values, RATES, exchange=exchange, device=device,
                                      sh_exchange=sh_exchange)
        a = trainer.adam
        assert a.world == world and a.exchange == exchange and a.sh_exchange == sh_exchange
        seeded = sh_exchange != "grads"
        coloured = sh_exchange == "colours"
        cam = orbit_camera(rank, 8, width=W, height=H, device=device)
        target = torch.rand(3, H, W, device=device,
                            generator=torch.Generator(device=device).manual_seed(rank))
        if coloured:
            trainer.prime(cam)
        for step in range(3):
            trainer.backward(cam, target)
            if coloured:
                a.next_camera.copy_(cam.campos)
            # Every rank's gradients, the replica and this share's moments before the exchange.
            mine = a.grad_slab.clone()
            every = torch.empty(world * mine.numel(), device=device)
            dist.all_gather_into_tensor(every, mine)
            every = every.view(world, -1)
            seeds = cameras = colours = next_cameras = bits = None
            if seeded:
                mine = a.seed_slab.clone()
                all_seeds = torch.empty(world * mine.numel(), device=device)
                dist.all_gather_into_tensor(all_seeds, mine)
                all_seeds = all_seeds.view(world, -1)
                seeds = [all_seeds[q, 8:8 + 4 * a.padded].view(-1, 4) for q in range(world)]
                cameras = [all_seeds[q, :3] for q in range(world)]
            if coloured:
                next_cameras = [all_seeds[q, 4:7] for q in range(world)]
                colours = [torch.zeros(a.padded, 3, device=device) for _ in range(world)]
                bits = a.clamp_bits.clone()
            params = a.param_slab.clone()
            first = {k: v.clone() for k, v in a.first.items()}
            second = {k: v.clone() for k, v in a.second.items()}
            a.step()
            torch.cuda.synchronize()
            # Emulation: the same kernel over local copies of all ranks' data.

            grads = [carve(every[q], a.padded) for q in range(world)]
            replica = carve(params, a.padded)
            names = GROUP_NAMES
            b1, b2 = _bias(step + 1)
            native_update(ShardStep(a.begin, a.end, 0,
                                    [[grads[q][k] for k in names] for q in range(world)],
                                    [[replica[k] for k in names]] * world, 0,
                                    [first[k] for k in names],
                                    [second[k] for k in names], a.saved["scaling"],
                                    a.saved["opacity"], a.saved["norm"], RATE_TUPLE, b1, b2,
                                    seeds, cameras, 3, colours, next_cameras, bits))
            lo, hi = a.begin, a.end
            torch.cuda.synchronize()
            for k in names:
                assert torch.equal(a.params[k][lo:hi], replica[k][lo:hi]), (rank, step, k)
                assert torch.equal(a.first[k], first[k]), (rank, step, k)
                assert torch.equal(a.second[k], second[k]), (rank, step, k)
            # Replicas agree across ranks (colour form: all but the SH, which
            # only their owner keeps; the colours it made for every rank).
            ref = a.param_slab.clone()
            dist.broadcast(ref, 0)
            ref = carve(ref, a.padded)
            for k in names:
                if not (coloured and k == "sh"):
                    assert torch.equal(ref[k], a.params[k]), (rank, step, k)
            if coloured:
                assert torch.equal(a.clamp_bits, bits), (rank, step)
                mine = a.colours.clone()
                made = torch.empty(world * mine.numel(), device=device)
                dist.all_gather_into_tensor(made, mine)
                made = made.view(world, a.padded, 3)
                for q in range(world):
                    assert torch.equal(made[q, lo:hi], colours[q][lo:hi]), (rank, step, q)
        if coloured:
            # After gather_sh every replica holds every share's coefficients.
            a.gather_sh()
            ref = a.params["sh"].clone()
            dist.broadcast(ref, 0)
            assert torch.equal(ref, a.params["sh"]), rank
        with open(os.path.join(out_dir, f"ok{rank}"), "w") as f:
            f.write("ok")
    finally:
        torch.cuda.synchronize()
        if trainer is not None:
            trainer.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange,sh_exchange",
                         [("peer", "seeds"), ("peer", "colours"), ("peer", "grads"),
                          ("collective", "grads")])
def test_two_gpu_exchange_matches_emulation(cuda, exchange, sh_exchange, tmp_path):
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.spawn(_dp_worker, args=(2, _free_port(), exchange, sh_exchange, str(tmp_path)),
             nprocs=2)
    assert (tmp_path / "ok0").exists() and (tmp_path / "ok1").exists()


@pytest.mark.parametrize("exchange,sh_exchange",
                         [("peer", "seeds"), ("peer", "colours"), ("collective", "grads")])
def test_two_gpu_exchange_matches_emulation_at_full_size(cuda, exchange, sh_exchange,
                                                         tmp_path):
    """The 8-view data-parallel configuration on two GPUs: 6,000,000 Gaussians,
    one 1920x1080 orbit view per GPU, three steps; after each exchange every
    rank's share, moments and replica are bit-identical to the same update
    kernel run over local copies of both ranks' gradients (or seeds)."""
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.spawn(_dp_worker, args=(2, _free_port(), exchange, sh_exchange, str(tmp_path), "full"),
             nprocs=2)
    assert (tmp_path / "ok0").exists() and (tmp_path / "ok1").exists()
