"""Failure detection of the data-parallel step on CPU gloo ranks (no GPU).

Each case runs three ranks of the collective exchange (the oracle standing in
for the update kernel) with a rank_health.StepGate of a short timeout, while
the process group's own timeout stays long (60 s). A rank that leaves between
steps, one that crashes without a word, and one that stalls past the gate's
timeout must each make the others raise RankFailure within a few seconds,
before any of them enters the step's collectives, naming the rank and the
reason. The failures are made on the host: a rank that returns, one that
exits the process, one that sleeps.
"""

import json
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dp_helpers import GROUP_NAMES, RATES, initial_values, oracle_update, view_gradients

WORLD, N, GATE_TIMEOUT = 3, 37, 1.5


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, port, scenario, out_dir):
    from datetime import timedelta

    from data_parallel import ShardedAdam
    from rank_health import RankFailure, default_gate

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD,
                            timeout=timedelta(seconds=60))
    record = {"rank": rank, "steps": 0}
    adam = ShardedAdam(N, RATES, device="cpu", update=oracle_update,
                       gate=default_gate(timeout=GATE_TIMEOUT))
    adam.load(initial_values(N))
    try:
        for step in range(6):
            if rank == 2 and step == 2:
                if scenario == "leave":
                    adam.leave()
                    record["left"] = True
                    break
                if scenario == "crash":
                    with open(os.path.join(out_dir, "rank2.json"), "w") as f:
                        json.dump({"rank": 2, "crashed": True}, f)
                    os._exit(3)  # a hard exit: no leave(), no teardown
                if scenario == "stall":
                    time.sleep(3 * GATE_TIMEOUT)
            grads = view_gradients(rank, step, adam.padded, N)
            for name in GROUP_NAMES:
                adam.grads[name].copy_(grads[name])
            started = time.monotonic()
            try:
                adam.step()
            except RankFailure as failure:
                record.update(failed_at=failure.step, ranks=list(failure.ranks),
                              reason=failure.reason,
                              seconds=time.monotonic() - started)
                break
            record["steps"] += 1
    finally:
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
            json.dump(record, f)
        adam.gate.depart(linger=4 * GATE_TIMEOUT)
        if scenario == "none":
            dist.destroy_process_group()
        # After a failure the group is not torn down collectively (a peer is
        # gone); each process exits, rank 0 (the store's host) last.


def _run(scenario, tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, port, scenario, str(tmp_path)))
             for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail(f"{scenario}: a rank did not finish")
    return {r: json.loads((tmp_path / f"rank{r}.json").read_text()) for r in range(WORLD)}


def test_healthy_ranks_pass_every_gate(tmp_path):
    out = _run("none", tmp_path)
    assert all(out[r]["steps"] == 6 and "reason" not in out[r] for r in range(WORLD))


def test_rank_that_leaves_between_steps_stops_the_others(tmp_path):
    out = _run("leave", tmp_path)
    assert out[2].get("left") and out[2]["steps"] == 2
    for r in (0, 1):
        assert out[r]["steps"] == 2 and out[r]["failed_at"] == 3
        assert out[r]["ranks"] == [2] and out[r]["reason"] == "left"
        assert out[r]["seconds"] < GATE_TIMEOUT  # told, not timed out


def test_rank_that_crashes_is_caught_by_the_gate_timeout(tmp_path):
    out = _run("crash", tmp_path)
    assert out[2].get("crashed")
    for r in (0, 1):
        assert out[r]["steps"] == 2 and out[r]["failed_at"] == 3
        # Either this rank timed out on rank 2, or the other survivor did first
        # and this one saw its "failed" mark; both well inside 60 s.
        if out[r]["reason"] == "timeout":
            assert 2 in out[r]["ranks"]
        else:
            assert out[r]["reason"] == "failed" and out[r]["ranks"] == [1 - r]
        assert out[r]["seconds"] < GATE_TIMEOUT + 5
    assert any(out[r]["reason"] == "timeout" for r in (0, 1))


def test_store_loss_is_a_rank_failure():
    """A gate whose store is gone (its host exited) raises RankFailure with
    reason "lost" instead of a network error."""
    from rank_health import RankFailure, StepGate

    class Gone:
        def set(self, *a):
            raise RuntimeError("Broken pipe")

        check = delete_key = set

    with pytest.raises(RankFailure) as info:
        StepGate(Gone(), 1, 2).arrive_and_wait(4)
    assert info.value.reason == "lost" and info.value.ranks == (0,)


def test_rank_stalled_past_the_timeout_fails_with_the_others(tmp_path):
    out = _run("stall", tmp_path)
    for r in (0, 1):
        assert out[r]["failed_at"] == 3 and out[r]["reason"] in ("timeout", "failed")
        assert out[r]["seconds"] < GATE_TIMEOUT + 5
    # The slow rank arrives after the others gave up and fails at the same gate
    # instead of entering the collectives alone.
    assert out[2]["steps"] == 2 and out[2]["failed_at"] == 3
    assert out[2]["reason"] == "failed" and set(out[2]["ranks"]) <= {0, 1}


def test_gate_unit_behaviour():
    from rank_health import RankFailure, StepGate

    store = dist.HashStore()
    a, b = StepGate(store, 0, 2, timeout=0.05), StepGate(store, 1, 2, timeout=0.05)
    b.store.set("clad3dgs/arrived/1/1", "1")
    a.arrive_and_wait(1)                    # b already arrived at step 1
    with pytest.raises(RankFailure) as info:
        a.arrive_and_wait(2)                # b never arrives at step 2
    assert info.value.reason == "timeout" and info.value.ranks == (1,)
    with pytest.raises(RankFailure) as info:
        b.arrive_and_wait(2)                # a gave up at step 2
    assert info.value.reason == "failed"
    solo = StepGate(dist.HashStore(), 0, 1)
    solo.arrive_and_wait(1)
    solo.leave()
    with pytest.raises(RuntimeError):
        solo.arrive_and_wait(2)
    with pytest.raises(ValueError):
        StepGate(store, 2, 2)
