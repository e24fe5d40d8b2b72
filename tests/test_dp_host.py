"""Host logic of the data-parallel step on CPU: share planning and the
collective exchange (reduce-scatter -> update -> all-gather) with two gloo
ranks, the oracle standing in for the update kernel. Every replica must end
bit-identical to a one-process emulation of the same ranks."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dp_helpers import RATES, GROUP_NAMES, initial_values, oracle_update, saved_from, view_gradients


def test_plan_pads_to_equal_shares_of_four():
    from data_parallel import plan

    for n in (0, 1, 5, 63, 64, 1000, 6_000_000):
        for world in (1, 2, 3, 8):
            padded, share = plan(n, world)
            assert padded >= n and padded - n < 4 * world
            assert share * world == padded and share % 4 == 0
    with pytest.raises(ValueError):
        plan(-1, 2)


def test_carve_lays_groups_end_to_end():
    from data_parallel import FLOATS_PER_GAUSSIAN, carve

    slab = torch.arange(FLOATS_PER_GAUSSIAN * 8, dtype=torch.float32)
    views = carve(slab, 8)
    assert [tuple(v.shape) for v in views.values()] == [(8, 3), (8, 48), (8, 3), (8, 4), (8, 1)]
    assert views["sh"][0, 0].item() == 24 and views["opacity"][7, 0].item() == 59 * 8 - 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _apply_saved(adam):
    saved = saved_from({k: adam.params[k] for k in ("scaling", "rotation", "opacity")})
    adam.saved["scaling"].copy_(torch.from_numpy(saved["scaling"]))
    adam.saved["opacity"].copy_(torch.from_numpy(saved["opacity"]).view(-1, 1))
    adam.saved["norm"].copy_(torch.from_numpy(saved["norm"]))


def _worker(rank, world, port, n, steps, out_dir):
    from datetime import timedelta

    from data_parallel import ShardedAdam

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        adam = ShardedAdam(n, RATES, device="cpu", update=oracle_update)
        assert adam.exchange == "collective"
        adam.load(initial_values(n))
        for step in range(steps):
            grads = view_gradients(rank, step, adam.padded, n)
            for name in GROUP_NAMES:
                adam.grads[name].copy_(grads[name])
            _apply_saved(adam)
            adam.step()
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"),
                 **{f"p_{k}": v.numpy() for k, v in adam.params.items()},
                 **{f"m_{k}": v.numpy() for k, v in adam.first.items()},
                 **{f"v_{k}": v.numpy() for k, v in adam.second.items()})
    finally:
        dist.destroy_process_group()


def _emulate(world, n, steps):
    """All ranks in one process: the oracle over every share, same order."""
    from data_parallel import ShardedAdam, ShardStep, plan

    padded, share = plan(n, world)
    adam = ShardedAdam(n, RATES, device="cpu", update=oracle_update)  # world 1 layout
    adam.load(initial_values(n))
    firsts = [{k: torch.zeros(share, w) for k, w in zip(GROUP_NAMES, (3, 48, 3, 4, 1))}
              for _ in range(world)]
    seconds = [{k: torch.zeros(share, w) for k, w in zip(GROUP_NAMES, (3, 48, 3, 4, 1))}
               for _ in range(world)]
    for step in range(steps):
        grads = [view_gradients(r, step, padded, n) for r in range(world)]
        _apply_saved(adam)
        t = step + 1
        for r in range(world):
            oracle_update(ShardStep(
                begin=r * share, end=(r + 1) * share, grad_origin=0,
                grads=[[grads[q][k] for k in GROUP_NAMES] for q in range(world)],
                params=[[adam.params[k] for k in GROUP_NAMES]], local=0,
                first=[firsts[r][k] for k in GROUP_NAMES],
                second=[seconds[r][k] for k in GROUP_NAMES],
                saved_scaling=adam.saved["scaling"], saved_opacity=adam.saved["opacity"],
                saved_norm=adam.saved["norm"],
                rates=tuple(RATES[x] for x in ("xyz", "f_dc", "f_rest", "scaling", "rotation",
                                               "opacity")),
                bias1=1 - 0.9 ** t, bias2_sqrt=(1 - 0.999 ** t) ** 0.5))
    return adam.params, firsts, seconds


def test_collective_exchange_on_two_gloo_ranks(tmp_path):
    world, n, steps = 2, 37, 3
    mp.spawn(_worker, args=(world, _free_port(), n, steps, str(tmp_path)), nprocs=world)
    params, firsts, seconds = _emulate(world, n, steps)
    for rank in range(world):
        got = np.load(tmp_path / f"rank{rank}.npz")
        for k in GROUP_NAMES:
            assert np.array_equal(got[f"p_{k}"], params[k].numpy()), (rank, k)
            assert np.array_equal(got[f"m_{k}"], firsts[rank][k].numpy()), (rank, k)
            assert np.array_equal(got[f"v_{k}"], seconds[rank][k].numpy()), (rank, k)
        # Parameters moved, padding rows did not.
        assert not np.array_equal(got["p_xyz"][:n], initial_values(n)["xyz"].numpy())
        assert (got["p_xyz"][n:] == 0).all()


def test_sh_exchange_form_choice_on_cpu():
    """The seed and colour forms need CUDA (their SH backward runs in the
    update kernel): on the CPU the gradient form is the default and both are
    refused; an unknown form is refused everywhere."""
    from data_parallel import ShardedAdam

    adam = ShardedAdam(37, RATES, device="cpu", update=oracle_update)
    assert adam.sh_exchange == "grads" and adam.seeds is None and adam.camera is None
    assert adam.colours is None and adam.clamp_bits is None
    for form in ("seeds", "colours", "colors"):
        with pytest.raises(ValueError):
            ShardedAdam(37, RATES, device="cpu", update=oracle_update, sh_exchange=form)


def _collective_seeds_worker(rank, world, port, out_dir):
    from datetime import timedelta

    from data_parallel import ShardedAdam

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        refused = False
        try:
            ShardedAdam(37, RATES, device="cpu", exchange="collective", sh_exchange="seeds")
        except ValueError:
            refused = True
        with open(os.path.join(out_dir, f"refused{rank}"), "w") as f:
            f.write(str(refused))
    finally:
        dist.destroy_process_group()


def test_collective_exchange_refuses_the_seed_form(tmp_path):
    """A collective reduce-scatter sums gradients, so with more than one rank
    the collective exchange cannot take colour seeds."""
    mp.spawn(_collective_seeds_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2)
    for rank in range(2):
        assert (tmp_path / f"refused{rank}").read_text() == "True"


def _resume_worker(rank, world, port, n, out_dir):
    from datetime import timedelta

    from data_parallel import ShardedAdam

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        def run(adam, steps):
            for step in steps:
                grads = view_gradients(rank, step, adam.padded, n)
                for name in GROUP_NAMES:
                    adam.grads[name].copy_(grads[name])
                _apply_saved(adam)
                adam.step()

        first = ShardedAdam(n, RATES, device="cpu", update=oracle_update)
        first.load(initial_values(n))
        run(first, range(2))
        state = first.state_dict()
        run(first, range(2, 4))
        resumed = ShardedAdam(n, RATES, device="cpu", update=oracle_update)
        resumed.load_state_dict(state)
        assert resumed.t == 2
        run(resumed, range(2, 4))
        for k in GROUP_NAMES:
            assert torch.equal(resumed.params[k], first.params[k]), (rank, k)
            assert torch.equal(resumed.first[k], first.first[k]), (rank, k)
            assert torch.equal(resumed.second[k], first.second[k]), (rank, k)
        other = dict(state, rank=1 - rank)
        try:
            resumed.load_state_dict(other)
            refused = False
        except ValueError:
            refused = True
        with open(os.path.join(out_dir, f"resumed{rank}"), "w") as f:
            f.write(str(refused))
    finally:
        dist.destroy_process_group()


def test_checkpoint_resume_on_two_gloo_ranks(tmp_path):
    """A rank's `state_dict` after two steps, loaded into a fresh optimizer,
    continues bit for bit like the uninterrupted run (parameters, sharded
    moments, step counter); another rank's checkpoint is refused."""
    mp.spawn(_resume_worker, args=(2, _free_port(), 37, str(tmp_path)), nprocs=2)
    for rank in range(2):
        assert (tmp_path / f"resumed{rank}").read_text() == "True"
