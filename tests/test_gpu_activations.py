"""Activation consumer and quaternion backward vs the oracle and vs torch.

Bit-exact against the oracle (same evaluation order, no contraction). Against
torch autograd + torch's fused Adam the reference's own tolerances apply
(check.py:23-118 and 121-230): quaternion VJP within a conditioning-scaled
bound, consumed parameters and moments within rtol 3e-6, atol 2e-7. Invalid
inputs are rejected before any write (check.py:231-260).
"""

import math

import numpy as np
import pytest
import torch

import cases
import oracle

pytestmark = pytest.mark.gpu


def _dev(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def _bits_equal(a, b):
    a, b = np.asarray(a), np.asarray(b)
    return ((a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))).all()


def _strided(t):
    storage = torch.full((*t.shape, 4), -17.0, device=t.device, dtype=t.dtype)
    storage[..., 0] = t
    out = storage[..., 0]
    assert not out.is_contiguous()
    return out


@pytest.mark.parametrize("n", [0, 1, 35, 257, 4097, 65537])
@pytest.mark.parametrize("scale", [0.0, 1e-14, 1e-12, 1.0, 1e4])
@pytest.mark.parametrize("counter", [0, 99, 29854])
def test_activation_consume_bit_exact(cuda, n, scale, counter):
    import clad_quaternion

    p = cases.activation_problem(n, seed=n + counter, scale=scale, moments=counter > 0)
    counters = [counter, counter + 3, counter + 7]
    bias1 = [1 - 0.9 ** (c + 1) for c in counters]
    bias2 = [math.sqrt(1 - 0.999 ** (c + 1)) for c in counters]
    dev = {k: [_dev(a, cuda) for a in p[k]] for k in ("params", "seeds", "saved", "first", "second")}
    seeds = [_strided(s) for s in dev["seeds"]] if n == 35 else dev["seeds"]
    saved = [_strided(s) for s in dev["saved"]] if n == 35 else dev["saved"]
    clad_quaternion.consume_activations(dev["params"], seeds, saved, dev["first"],
                                        dev["second"], p["rates"], bias1, bias2)
    ref = {k: [a.copy() for a in p[k]] for k in ("params", "first", "second")}
    oracle.activation_consume(ref["params"], p["seeds"],
                              [p["saved"][0].reshape(-1).copy(), p["saved"][1],
                               p["saved"][2].reshape(-1).copy()],
                              ref["first"], ref["second"], p["rates"],
                              [float(np.float32(b)) for b in bias1],
                              [float(np.float32(b)) for b in bias2])
    torch.cuda.synchronize()
    for key in ("params", "first", "second"):
        for j in range(3):
            assert _bits_equal(dev[key][j].cpu().numpy(), ref[key][j]), (key, j)


@pytest.mark.parametrize("n", [1, 35, 257])
@pytest.mark.parametrize("counter", [0, 99, 29854])
def test_activation_consume_matches_torch_fused_adam(cuda, n, counter):
    """check.py:121-230: consumed update vs autograd grads + torch fused Adam."""
    import clad_quaternion

    torch.manual_seed(42 + n + counter)
    rates = [0.001, 0.005, 0.025]
    q = torch.randn((n, 4), device=cuda)
    raw_scale = torch.rand((n, 3), device=cuda) * 20 - 15
    extremes = torch.tensor([-120.0, -100.0, -90.0, -40.0, -20.0, -10.0, 0.0, 10.0, 16.0,
                             20.0, 40.0, 100.0, 120.0], device=cuda)
    opacity = extremes.repeat((n + 12) // 13)[:n, None].contiguous()
    raw = [q, raw_scale, opacity]
    seeds = [torch.randn_like(v) * 0.001 for v in raw]
    saved = [q.norm(2, dim=1, keepdim=True), raw_scale.exp(), opacity.sigmoid()]
    reference = [torch.nn.Parameter(v.clone()) for v in raw]
    optimizer = torch.optim.Adam([dict(params=[v], lr=r) for v, r in zip(reference, rates)],
                                 eps=1e-15, fused=True, foreach=False)
    counters = [counter, counter + 3, counter + 7]
    first, second = [], []
    for value, step in zip(reference, counters):
        m = torch.randn_like(value) * 0.02 if counter else torch.zeros_like(value)
        v = torch.rand_like(value) * 0.03 if counter else torch.zeros_like(value)
        optimizer.state[value] = dict(step=torch.tensor(float(step), device=cuda),
                                      exp_avg=m.clone(), exp_avg_sq=v.clone())
        first.append(m)
        second.append(v)
    outputs = [torch.nn.functional.normalize(reference[0], dim=1, eps=1e-12),
               reference[1].exp(), reference[2].sigmoid()]
    grads = list(torch.autograd.grad(outputs, reference, seeds))
    generated_q = clad_quaternion.backward(reference[0].detach(), seeds[0], saved[0])
    bound = 2e-6 * seeds[0].double().norm(dim=1, keepdim=True) / q.double().norm(
        dim=1, keepdim=True).clamp_min(1e-12)
    assert ((generated_q.double() - grads[0].double()).abs() <= bound + 1e-7).all()
    grads[0] = generated_q
    for value, grad in zip(reference, grads):
        value.grad = grad
    optimizer.step()
    clad_quaternion.consume_activations(raw, seeds, saved, first, second, rates,
                                        [1 - 0.9 ** (s + 1) for s in counters],
                                        [math.sqrt(1 - 0.999 ** (s + 1)) for s in counters])
    for value, m, v, expected in zip(raw, first, second, reference):
        for actual, wanted in ((value, expected), (m, optimizer.state[expected]["exp_avg"]),
                               (v, optimizer.state[expected]["exp_avg_sq"])):
            assert torch.isfinite(actual).all()
            torch.testing.assert_close(actual, wanted.detach(), rtol=3e-6, atol=2e-7)


@pytest.mark.parametrize("invalid", ["cross-group", "moments", "seed", "saved", "bias", "rate"])
def test_invalid_activation_inputs_rejected_before_write(cuda, invalid):
    import clad_quaternion

    raw = [torch.randn((35, w), device=cuda) for w in (4, 3, 1)]
    seeds = [torch.randn_like(v) for v in raw]
    saved = [raw[0].norm(2, dim=1, keepdim=True), raw[1].exp(), raw[2].sigmoid()]
    first = [torch.zeros_like(v) for v in raw]
    second = [torch.ones_like(v) for v in raw]
    if invalid == "cross-group":
        first[1] = raw[0].view(-1)[:105].view(35, 3)
    elif invalid == "moments":
        second[2] = first[2]
    elif invalid == "seed":
        seeds[0] = raw[0]
    elif invalid == "saved":
        saved[1] = raw[1]
    bias, rate = [0.1] * 3, [0.001, 0.005, 0.025]
    if invalid == "bias":
        bias[1] = 0
    if invalid == "rate":
        rate[2] = float("nan")
    before = [v.clone() for v in raw + first + second]
    with pytest.raises(RuntimeError):
        clad_quaternion.consume_activations(raw, seeds, saved, first, second, rate, bias,
                                            [math.sqrt(0.001)] * 3)
    torch.cuda.synchronize()
    for value, previous in zip(raw + first + second, before):
        assert torch.equal(value, previous)


@pytest.mark.parametrize("n", [0, 1, 35, 4097])
@pytest.mark.parametrize("scale", [0.0, 1e-14, 1e-12, 1.0, 1e4])
@pytest.mark.parametrize("packed", [True, False])
def test_quaternion_backward(cuda, n, scale, packed):
    """check.py:23-52: vs F.normalize autograd (relative L2 < 2e-6 and the
    conditioning bound) and bit-exact vs the oracle."""
    import clad_quaternion
    import normalization

    torch.manual_seed(42 + n)
    raw = torch.randn((n, 4), device=cuda) * scale
    seed = torch.randn_like(raw)
    if not packed and raw.numel():
        raw, seed = _strided(raw).detach(), _strided(seed)
    raw.requires_grad_(True)
    forward = torch.nn.functional.normalize(raw, dim=1, eps=1e-12)
    expected = torch.autograd.grad(forward, raw, seed)[0]
    actual_forward = normalization.normalize_quaternion(raw, clad_quaternion)
    actual = torch.autograd.grad(actual_forward, raw, seed)[0]
    assert torch.equal(actual_forward, forward)
    assert torch.isfinite(actual).all()
    diff = actual.double() - expected.double()
    assert diff.norm() / expected.double().norm().clamp_min(1e-30) < 2e-6
    bound = seed.double().norm(dim=1, keepdim=True) / raw.double().norm(
        dim=1, keepdim=True).clamp_min(1e-12)
    assert (diff.abs() <= 2e-6 * bound + 1e-7).all()
    q = raw.detach().contiguous().cpu().numpy()
    s = seed.contiguous().cpu().numpy()
    norms = raw.detach().norm(2, dim=1, keepdim=True).cpu().numpy()
    assert _bits_equal(actual.cpu().numpy(), oracle.quaternion_backward(q, s, norms))


def test_quaternion_clamp_boundary_and_streams(cuda):
    import clad_quaternion
    import normalization

    eps = torch.tensor(1e-12, device=cuda)
    raw = torch.zeros((4, 4), device=cuda)
    raw[:3, 0] = torch.stack((torch.nextafter(eps, torch.zeros_like(eps)), eps,
                              torch.nextafter(eps, torch.full_like(eps, float("inf")))))
    raw.requires_grad_(True)
    seed = torch.ones_like(raw)
    expected = torch.autograd.grad(torch.nn.functional.normalize(raw, dim=1), raw, seed)[0]
    actual = clad_quaternion.backward(raw, seed, raw.norm(2, dim=1, keepdim=True))
    assert ((actual - expected).abs() <= 2e-6 * seed.norm(dim=1, keepdim=True) / eps).all()
    with pytest.raises(RuntimeError, match="first-order"):
        x = torch.randn((35, 4), device=cuda, requires_grad=True)
        torch.autograd.grad(normalization.normalize_quaternion(x, clad_quaternion).sum(),
                            x, create_graph=True)
    with torch.cuda.stream(torch.cuda.Stream()):
        x = torch.randn((35, 4), device=cuda, requires_grad=True)
        got = torch.autograd.grad(normalization.normalize_quaternion(x, clad_quaternion).sum(), x)[0]
        want = torch.autograd.grad(torch.nn.functional.normalize(x, dim=1).sum(), x)[0]
        torch.testing.assert_close(got, want, rtol=2e-5, atol=2e-6)
    torch.cuda.synchronize()


def test_activation_full_size_bit_exact(cuda):
    """1M Gaussians (the activation benchmark size) against the oracle."""
    import clad_quaternion

    n = 1_000_000
    p = cases.activation_problem(n, seed=7, moments=True)
    dev = {k: [_dev(a, cuda) for a in p[k]] for k in ("params", "seeds", "saved", "first", "second")}
    b1, b2 = [0.1, 0.19, 0.271], [0.0316, 0.0447, 0.0547]
    clad_quaternion.consume_activations(dev["params"], dev["seeds"], dev["saved"],
                                        dev["first"], dev["second"], p["rates"], b1, b2)
    ref = {k: [a.copy() for a in p[k]] for k in ("params", "first", "second")}
    oracle.activation_consume(ref["params"], p["seeds"],
                              [p["saved"][0].reshape(-1).copy(), p["saved"][1],
                               p["saved"][2].reshape(-1).copy()], ref["first"],
                              ref["second"], p["rates"], b1, b2)
    torch.cuda.synchronize()
    for key in ("params", "first", "second"):
        for j in range(3):
            assert _bits_equal(dev[key][j].cpu().numpy(), ref[key][j]), (key, j)
