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


@pytest.mark.parametrize("n,chunk", [(1, 64), (1000, 256), (100_000, 8192)])
def test_host_buffer_pipeline_bit_exact(cuda, n, chunk):
    import consume

    sh, act = _problem(n, seed=3)
    step = 2
    b1, b2 = cases.bias(step)
    ab1, ab2 = [0.19, 0.19, 0.19], [0.0447, 0.0447, 0.0447]
    h = {k: torch.from_numpy(np.ascontiguousarray(v)).pin_memory() for k, v in sh.items()}
    ha = {k: [torch.from_numpy(np.ascontiguousarray(x)).pin_memory() for x in act[k]]
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
