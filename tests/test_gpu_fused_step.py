"""The fused per-Gaussian pass (SH consume + activation consume in one kernel)
and its host-buffer pipeline vs the oracle: both must equal the two separate
reference computations bit for bit."""

import numpy as np
import pytest
import torch

import cases
import oracle

pytestmark = pytest.mark.gpu


def _bits_equal(a, b):
    return ((a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))).all()


def _problem(n, seed):
    sh = cases.sh_problem(n, seed=seed, moments=True)
    act = cases.activation_problem(n, seed=seed + 1, moments=True)
    return sh, act


def _oracle(sh, act, degree, step, act_bias1, act_bias2):
    out = {k: sh[k].copy() for k in cases.SH_KEYS}
    b1, b2 = cases.bias(step)
    oracle.sh_consume("split_torch_adam", degree, sh["means"], sh["radii"], sh["clamped"],
                      sh["camera"], sh["seed"], out["dm"], dc=out["dc"], rest=out["rest"],
                      dc_first=out["dc_first"], dc_second=out["dc_second"],
                      rest_first=out["rest_first"], rest_second=out["rest_second"],
                      bias1=b1, bias2_sqrt=b2)
    a = {k: [x.copy() for x in act[k]] for k in ("params", "first", "second")}
    oracle.activation_consume(a["params"], act["seeds"],
                              [act["saved"][0].reshape(-1).copy(), act["saved"][1],
                               act["saved"][2].reshape(-1).copy()], a["first"],
                              a["second"], act["rates"], act_bias1, act_bias2)
    return out, a


@pytest.mark.parametrize("n", [1, 64, 1000, 64 * 200 + 5, 1_100_000])
def test_fused_step_bit_exact(cuda, n):
    import consume

    sh, act = _problem(n, seed=n % 1000)
    step = 5
    b1, b2 = cases.bias(step)
    ab1, ab2 = [0.41, 0.41, 0.41], [0.0707, 0.0707, 0.0707]
    d = {k: torch.from_numpy(np.ascontiguousarray(v)).to(cuda) for k, v in sh.items()}
    da = {k: [torch.from_numpy(x).to(cuda) for x in act[k]] for k in
          ("params", "seeds", "saved", "first", "second")}
    consume.gaussian_step(d["means"], d["radii"], d["clamped"], d["camera"], d["seed"],
                          d["dm"], d["dc"], d["rest"], d["dc_first"], d["dc_second"],
                          d["rest_first"], d["rest_second"], bias1=b1, bias2_sqrt=b2,
                          degree=3, act_parameters=da["params"], act_seeds=da["seeds"],
                          act_saved=da["saved"], act_first=da["first"],
                          act_second=da["second"], act_rates=act["rates"],
                          act_bias1=ab1, act_bias2=ab2)
    torch.cuda.synchronize()
    want_sh, want_act = _oracle(sh, act, 3, step, ab1, ab2)
    for k in cases.SH_KEYS:
        assert _bits_equal(d[k].cpu().numpy(), want_sh[k]), k
    for k in ("params", "first", "second"):
        for j in range(3):
            assert _bits_equal(da[k][j].cpu().numpy(), want_act[k][j]), (k, j)


@pytest.mark.parametrize("memory", ["pinned", "pageable", "mixed"])
@pytest.mark.parametrize("n,chunk", [(1, 64), (1000, 256), (100_000, 8192)])
def test_host_buffer_pipeline_bit_exact(cuda, n, chunk, memory):
    """The staged copy pipeline with pinned, pageable or mixed host buffers
    (pageable copies are synchronous on the host side): bit-exact."""
    import consume

    sh, act = _problem(n, seed=3)
    step = 2
    b1, b2 = cases.bias(step)
    ab1, ab2 = [0.19, 0.19, 0.19], [0.0447, 0.0447, 0.0447]

    def host(v, pageable):
        t = torch.from_numpy(np.array(v, copy=True))  # the oracle keeps the inputs
        return t if pageable else t.pin_memory()

    h = {k: host(v, memory == "pageable" or (memory == "mixed" and k == "rest"))
         for k, v in sh.items()}
    ha = {k: [host(x, memory == "pageable") for x in act[k]]
          for k in ("params", "seeds", "saved", "first", "second")}
    ws = torch.empty(consume.host_step_workspace(chunk), dtype=torch.uint8, device=cuda)
    consume.gaussian_step_host(h["means"], h["radii"], h["clamped"], h["camera"], h["seed"],
                               h["dm"], h["dc"], h["rest"], h["dc_first"], h["dc_second"],
                               h["rest_first"], h["rest_second"], bias1=b1, bias2_sqrt=b2,
                               degree=3, act_parameters=ha["params"], act_seeds=ha["seeds"],
                               act_saved=ha["saved"], act_first=ha["first"],
                               act_second=ha["second"], act_rates=act["rates"],
                               act_bias1=ab1, act_bias2=ab2, workspace=ws, chunk=chunk)
    want_sh, want_act = _oracle(sh, act, 3, step, ab1, ab2)
    for k in cases.SH_KEYS:
        assert _bits_equal(h[k].numpy(), want_sh[k]), k
    for k in ("params", "first", "second"):
        for j in range(3):
            assert _bits_equal(ha[k][j].numpy(), want_act[k][j]), (k, j)


def _saved_of(params):
    """Saved activations of the current raw parameters (|q|, exp(scale),
    sigmoid(opacity)), as the activation forward produces them."""
    rot, scl, opa = params
    norm = np.sqrt((rot.astype(np.float64) ** 2).sum(1, keepdims=True)).astype(np.float32)
    sig = (1 / (1 + np.exp(-opa.astype(np.float64)))).astype(np.float32)
    return [norm, np.exp(scl).astype(np.float32), sig]


def test_thirty_consecutive_steps_at_full_size(cuda):
    """The fused-step configuration: 1,100,000 Gaussians, SH degree 3 +
    activations, 30 consecutive steps from a fresh Adam state (bias
    corrections of steps 1..30, moments carried over), new upstream adjoints
    each step and the saved activations of the current parameters. After every
    step every parameter, moment and dm must equal the oracle's bit for bit."""
    import consume

    n, steps = 1_100_000, 30
    sh = cases.sh_problem(n, seed=42, moments=False)
    act = cases.activation_problem(n, seed=43, moments=False)
    d = {k: torch.from_numpy(np.ascontiguousarray(v)).to(cuda) for k, v in sh.items()}
    da = {k: [torch.from_numpy(np.ascontiguousarray(x)).to(cuda) for x in act[k]]
          for k in ("params", "seeds", "saved", "first", "second")}
    ref = {k: sh[k].copy() for k in cases.SH_KEYS}
    ref_act = {k: [x.copy() for x in act[k]] for k in ("params", "first", "second")}
    rng = np.random.default_rng(44)
    for t in range(1, steps + 1):
        seed = (rng.standard_normal((n, 3)) * 1e-3).astype(np.float32)
        dm = (rng.standard_normal((n, 3)) * 1e-4).astype(np.float32)
        act_seeds = [(rng.standard_normal(p.shape) * 1e-4).astype(np.float32)
                     for p in ref_act["params"]]
        saved = _saved_of(ref_act["params"])
        d["seed"].copy_(torch.from_numpy(seed))
        d["dm"].copy_(torch.from_numpy(dm))
        for j in range(3):
            da["seeds"][j].copy_(torch.from_numpy(act_seeds[j]))
            da["saved"][j].copy_(torch.from_numpy(saved[j]))
        b1, b2 = cases.bias(t)
        consume.gaussian_step(d["means"], d["radii"], d["clamped"], d["camera"], d["seed"],
                              d["dm"], d["dc"], d["rest"], d["dc_first"], d["dc_second"],
                              d["rest_first"], d["rest_second"], bias1=b1, bias2_sqrt=b2,
                              degree=3, act_parameters=da["params"], act_seeds=da["seeds"],
                              act_saved=da["saved"], act_first=da["first"],
                              act_second=da["second"], act_rates=act["rates"],
                              act_bias1=[b1] * 3, act_bias2=[b2] * 3)
        ref["dm"] = dm.copy()
        oracle.sh_consume("split_torch_adam", 3, sh["means"], sh["radii"], sh["clamped"],
                          sh["camera"], seed, ref["dm"], dc=ref["dc"], rest=ref["rest"],
                          dc_first=ref["dc_first"], dc_second=ref["dc_second"],
                          rest_first=ref["rest_first"], rest_second=ref["rest_second"],
                          bias1=b1, bias2_sqrt=b2)
        oracle.activation_consume(ref_act["params"], act_seeds,
                                  [saved[0].reshape(-1).copy(), saved[1],
                                   saved[2].reshape(-1).copy()],
                                  ref_act["first"], ref_act["second"], act["rates"],
                                  [b1] * 3, [b2] * 3)
        torch.cuda.synchronize()
        for k in cases.SH_KEYS:
            assert _bits_equal(d[k].cpu().numpy(), ref[k]), (t, k)
        for k in ("params", "first", "second"):
            for j in range(3):
                assert _bits_equal(da[k][j].cpu().numpy(), ref_act[k][j]), (t, k, j)
