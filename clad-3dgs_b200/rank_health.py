"""Host-side failure detection for the data-parallel step.

The exchange of a data-parallel step starts with collectives (a one-element
all-reduce ordering the GPUs, or NCCL reduce-scatters). A rank that died,
left or stalls between steps would leave the others blocked inside that
collective until the process group's timeout (minutes), with work in flight
on their GPUs. `StepGate` settles it on the host first, through the process
group's key-value store, before any rank enqueues the step's collectives:

* every rank posts "arrived at step t" and waits, polling the store, until all
  ranks have posted;
* a rank that leaves between steps (normal exit, or an exception it catches)
  posts "left"; a rank that gives up posts "failed"; the others see either
  at their next gate and raise `RankFailure` at once, naming the rank;
* a rank that neither arrives nor says anything within `timeout` seconds
  (crashed, hung, or merely slow) makes the waiting ranks raise `RankFailure`
  with reason "timeout"; each of them posts "failed", so the slow rank, if
  it does arrive later, fails at that gate instead of entering a collective
  the others have abandoned (or, when the store's host, rank 0, has exited
  meanwhile, raises with reason "lost").

So a step either starts on every rank or on none: no rank is ever left inside
a collective because of a peer that is gone, and the failure surfaces within
the gate's timeout rather than the group's.
"""

from __future__ import annotations

import time
from datetime import timedelta


class RankFailure(RuntimeError):
    """A peer left, failed or missed the gate. `ranks` are the peers
    concerned, `reason` is "left", "failed" or "timeout"."""

    def __init__(self, step, ranks, reason):
        self.step, self.ranks, self.reason = step, tuple(ranks), reason
        super().__init__(f"step {step}: rank(s) {list(self.ranks)} {reason}")


class StepGate:
    def __init__(self, store, rank, world, *, timeout=5.0, poll=0.002, prefix="clad3dgs"):
        if world < 1 or not 0 <= rank < world:
            raise ValueError("StepGate: need 0 <= rank < world")
        if timeout <= 0:
            raise ValueError("StepGate: timeout must be positive")
        self.store, self.rank, self.world = store, rank, world
        self.timeout, self.poll, self.prefix = float(timeout), float(poll), prefix
        self.closed = False

    def _key(self, kind, who, step=None):
        return f"{self.prefix}/{kind}/{who}" if step is None else \
            f"{self.prefix}/{kind}/{step}/{who}"

    def _peers(self):
        return [q for q in range(self.world) if q != self.rank]

    def _marked(self, kind):
        return [q for q in self._peers() if self.store.check([self._key(kind, q)])]

    def arrive_and_wait(self, step):
        """Returns once every rank has arrived at `step`; raises RankFailure
        (after posting "failed") when a peer left, failed or stays away past
        the timeout, or with reason "lost" when the store itself is gone (its
        host, rank 0 of the group, has exited)."""
        if self.closed:
            raise RuntimeError("StepGate used after leave()")
        try:
            self._gate(step)
        except RankFailure:
            raise
        except (RuntimeError, OSError) as error:  # DistNetworkError and kin
            raise RankFailure(step, [0], "lost") from error

    def _gate(self, step):
        self.store.set(self._key("arrived", self.rank, step), "1")
        if self.world == 1:
            return
        waiting = self._peers()
        deadline = time.monotonic() + self.timeout
        while True:
            for kind in ("left", "failed"):
                gone = self._marked(kind)
                if gone:
                    self._give_up(step)
                    raise RankFailure(step, gone, kind)
            waiting = [q for q in waiting
                       if not self.store.check([self._key("arrived", q, step)])]
            if not waiting:
                if step >= 2:  # every rank is past step - 1: drop this rank's old key
                    self.store.delete_key(self._key("arrived", self.rank, step - 2))
                return
            if time.monotonic() > deadline:
                self._give_up(step)
                raise RankFailure(step, waiting, "timeout")
            time.sleep(self.poll)

    def _give_up(self, step):
        self.store.set(self._key("failed", self.rank), str(step))

    def leave(self):
        """Tells the other ranks this one takes part in no further step (call
        between steps, with no collective of this rank in flight)."""
        if not self.closed:
            self.store.set(self._key("left", self.rank), "1")
            self.closed = True

    def depart(self, linger=5.0):
        """Call once before the process exits, after any failure was handled.
        Rank 0 hosts the store, so it waits (at most `linger` seconds) until
        every other rank has departed too, letting survivors finish reading
        the store instead of losing it mid-gate."""
        try:
            self.store.set(self._key("departed", self.rank), "1")
            if self.rank != 0:
                return
            deadline = time.monotonic() + linger
            while time.monotonic() < deadline:
                if all(self.store.check([self._key("departed", q)]) for q in self._peers()):
                    return
                time.sleep(self.poll)
        except (RuntimeError, OSError):
            pass  # the store is already gone: nothing left to wait for


def default_gate(timeout=5.0, group=None):
    """A gate over the default process group's store (rank and size of
    `group`, the whole world by default)."""
    import torch.distributed as dist

    store = dist.distributed_c10d._get_default_store()
    return StepGate(store, dist.get_rank(group), dist.get_world_size(group), timeout=timeout)


def group_timeout(seconds):
    """A process-group timeout for init_process_group(timeout=...): keep it
    well above the gate's, as the last bound."""
    return timedelta(seconds=float(seconds))
