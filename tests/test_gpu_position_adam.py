"""Positions' Adam inside the per-Gaussian kernels (clad3dgs_sh_consume_xyz,
clad3dgs_gaussian_step_xyz) vs the oracle, bit for bit: the SH consume (or the
fused SH + activation pass) followed by torch-fused Adam on means with the
final dm as the gradient, for every Gaussian (invisible ones included), over
consecutive steps, with and without the coefficient snapshot, at tail sizes and
with misaligned buffers (the one-tile kernel)."""

import numpy as np
import pytest
import torch

import cases
import oracle

pytestmark = pytest.mark.gpu
RATE = 0.00016 * 3.7  # a position rate from the schedule, not a round number


def _bits_equal(a, b):
    return ((a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))).all()


def _xyz_state(n, seed):
    rng = np.random.default_rng(seed)
    return dict(first=(rng.standard_normal((n, 3)) * 1e-4).astype(np.float32),
                second=(rng.random((n, 3)) * 1e-8).astype(np.float32))


def _oracle_step(sh, xyz, step, snapshot):
    b1, b2 = cases.bias(step)
    coefficient = (np.concatenate([sh["dc"], sh["rest"]], 1).copy() if snapshot else None)
    oracle.sh_consume("split_torch_adam", 3, sh["means"], sh["radii"], sh["clamped"],
                      sh["camera"], sh["seed"], sh["dm"], coefficient=coefficient,
                      dc=sh["dc"], rest=sh["rest"], dc_first=sh["dc_first"],
                      dc_second=sh["dc_second"], rest_first=sh["rest_first"],
                      rest_second=sh["rest_second"], bias1=b1, bias2_sqrt=b2)
    oracle.xyz_adam(sh["means"], sh["dm"], xyz["first"], xyz["second"], RATE, b1, b2)


def _to(cuda, arrays, offset=0):
    """Device copies; offset > 0 places each array 4 bytes into its buffer, so
    no array is 16-byte aligned (the one-tile kernel's path)."""
    out = {}
    for k, v in arrays.items():
        v = np.ascontiguousarray(v)
        flat = torch.from_numpy(v).reshape(-1)
        if offset:
            buf = torch.empty(flat.numel() + offset, dtype=flat.dtype, device=cuda)
            buf[offset:] = flat.to(cuda)
            out[k] = buf[offset:].view(v.shape)
        else:
            out[k] = flat.to(cuda).view(v.shape)
    return out


@pytest.mark.parametrize("n", [1, 31, 32, 1000, 70_001])
@pytest.mark.parametrize("snapshot", [False, True])
@pytest.mark.parametrize("misaligned", [False, True])
def test_sh_consume_with_positions_bit_exact(cuda, n, snapshot, misaligned):
    import consume

    sh = cases.sh_problem(n, seed=n % 997, moments=True)
    xyz = _xyz_state(n, n + 1)
    d = _to(cuda, sh, 1 if misaligned else 0)
    dx = _to(cuda, xyz, 1 if misaligned else 0)
    for step in (1, 2, 3):
        b1, b2 = cases.bias(step)
        coefficient = (torch.cat([d["dc"], d["rest"]], 1).contiguous() if snapshot else None)
        consume.sh_consume_split_torch_adam(
            d["means"], d["radii"], d["clamped"], d["camera"], d["seed"], d["dm"], d["dc"],
            d["rest"], d["dc_first"], d["dc_second"], d["rest_first"], d["rest_second"],
            bias1=b1, bias2_sqrt=b2, degree=3, coefficient=coefficient,
            xyz=dict(first=dx["first"], second=dx["second"], rate=RATE, bias1=b1,
                     bias2_sqrt=b2))
        _oracle_step(sh, xyz, step, snapshot)
        torch.cuda.synchronize()
        for k in ("means",) + cases.SH_KEYS:
            assert _bits_equal(d[k].cpu().numpy(), sh[k]), (step, k)
        for k in ("first", "second"):
            assert _bits_equal(dx[k].cpu().numpy(), xyz[k]), (step, k)


@pytest.mark.parametrize("n", [5, 1000, 64 * 200 + 5])
def test_fused_step_with_positions_bit_exact(cuda, n):
    """All 59 parameters of a Gaussian in one pass."""
    import consume

    sh = cases.sh_problem(n, seed=11, moments=True)
    act = cases.activation_problem(n, seed=12, moments=True)
    xyz = _xyz_state(n, 13)
    d = _to(cuda, sh)
    dx = _to(cuda, xyz)
    da = {k: [torch.from_numpy(x).to(cuda) for x in act[k]] for k in
          ("params", "seeds", "saved", "first", "second")}
    ab1, ab2 = [0.271, 0.271, 0.271], [0.0548, 0.0548, 0.0548]
    step = 3
    b1, b2 = cases.bias(step)
    consume.gaussian_step(d["means"], d["radii"], d["clamped"], d["camera"], d["seed"],
                          d["dm"], d["dc"], d["rest"], d["dc_first"], d["dc_second"],
                          d["rest_first"], d["rest_second"], bias1=b1, bias2_sqrt=b2,
                          degree=3, act_parameters=da["params"], act_seeds=da["seeds"],
                          act_saved=da["saved"], act_first=da["first"],
                          act_second=da["second"], act_rates=act["rates"], act_bias1=ab1,
                          act_bias2=ab2, xyz=dict(first=dx["first"], second=dx["second"],
                                                  rate=RATE, bias1=b1, bias2_sqrt=b2))
    torch.cuda.synchronize()
    _oracle_step(sh, xyz, step, False)
    a = {k: [x.copy() for x in act[k]] for k in ("params", "first", "second")}
    oracle.activation_consume(a["params"], act["seeds"],
                              [act["saved"][0].reshape(-1).copy(), act["saved"][1],
                               act["saved"][2].reshape(-1).copy()], a["first"], a["second"],
                              act["rates"], ab1, ab2)
    for k in ("means",) + cases.SH_KEYS:
        assert _bits_equal(d[k].cpu().numpy(), sh[k]), k
    for k in ("first", "second"):
        assert _bits_equal(dx[k].cpu().numpy(), xyz[k]), k
    for k in ("params", "first", "second"):
        for j in range(3):
            assert _bits_equal(da[k][j].cpu().numpy(), a[k][j]), (k, j)


def test_position_adam_matches_torch_fused_adam(cuda):
    """The oracle's position update is torch's fused Adam (tolerance of the
    float-rounded bias corrections the C boundary carries)."""
    n = 4096
    sh = cases.sh_problem(n, seed=5, moments=False)
    xyz = {"first": np.zeros((n, 3), np.float32), "second": np.zeros((n, 3), np.float32)}
    means0 = sh["means"].copy()
    _oracle_step(sh, xyz, 1, False)
    p = torch.nn.Parameter(torch.from_numpy(means0).to(cuda))
    opt = torch.optim.Adam([p], lr=RATE, eps=1e-15, fused=True)
    p.grad = torch.from_numpy(sh["dm"]).to(cuda)  # the final dm is the gradient
    opt.step()
    torch.testing.assert_close(p.detach().cpu(), torch.from_numpy(sh["means"]), rtol=1e-6,
                               atol=1e-9)
    torch.testing.assert_close(opt.state[p]["exp_avg"].cpu(), torch.from_numpy(xyz["first"]),
                               rtol=1e-6, atol=0)
