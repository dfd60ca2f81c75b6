"""Host-side failure detection for the sharded step.

The reference trains in one process and has no failure handling beyond
``Result`` and panics (crates/mmn-optim/src/lib.rs:148,161). A sharded step
runs one process per GPU and every step ends in a collective (the exchange
fence), so one rank that dies or stalls would leave the others blocked in
that collective until the process group's timeout. ``RankMonitor`` turns both
cases into errors on every rank before the next collective is issued:

- a rank that raises inside ``monitor.step_guard()`` publishes its failure in
  the job's key-value store (the rendezvous ``TCPStore`` of torch.distributed);
- every rank publishes a heartbeat (its completed step) after each step and,
  before issuing the next step's collectives, waits for all peers to have
  completed the previous one, up to a deadline. A peer that published a
  failure raises ``RankFailure``; one that never arrives raises
  ``RankTimeout``;
- a step whose collective the process group's (short) timeout ends names its
  cause the same way, and marks this rank "lost" rather than "failed", so the
  root cause stays the one every rank reports.

The check runs between steps, on the host, with none of this rank's kernels
or collectives in flight, so detecting a failure never needs a GPU fault.
"""
from __future__ import annotations

import contextlib
import time


class RankFailure(RuntimeError):
    """A peer rank reported that it failed."""

    def __init__(self, rank: int, reason: str):
        super().__init__(f"rank {rank} failed: {reason}")
        self.rank = rank
        self.reason = reason


class RankTimeout(RuntimeError):
    """A peer rank did not finish the previous step before the deadline."""

    def __init__(self, ranks, step: int, deadline_s: float):
        super().__init__(f"ranks {sorted(ranks)} did not finish step {step} within "
                         f"{deadline_s:.1f} s")
        self.ranks = sorted(ranks)
        self.step = step


def _is_comm_error(e: BaseException) -> bool:
    """A collective or store operation that ended with an error (a peer that
    closed its connection, or the process group's timeout), as opposed to an
    exception of this rank's own step."""
    try:
        import torch.distributed as dist

        if isinstance(e, dist.DistError):
            return True
    except ImportError:  # torch is optional for the monitor itself
        pass
    if not isinstance(e, RuntimeError):
        return False
    msg = str(e)
    return any(k in msg for k in ("gloo", "NCCL", "Connection closed", "Connection reset",
                                  "timed out", "Timeout", "timeout"))


class RankMonitor:
    """Heartbeats and failure reports of the ranks of one job, in a shared store
    (anything with ``set(key, value)``, ``get(key)`` and ``check([keys])``, such
    as ``torch.distributed.TCPStore``)."""

    def __init__(self, store, rank: int, world_size: int, deadline_s: float = 30.0,
                 prefix: str = "mmn", grace_s: float = 2.0):
        self.store = store
        self.rank = rank
        self.world = world_size
        self.deadline = deadline_s
        self.prefix = prefix
        # how long a rank whose collective failed waits for the peer at fault
        # to publish its failure before it names the cause itself
        self.grace = min(grace_s, deadline_s)
        self.step = 0

    def _key(self, kind: str, rank: int) -> str:
        return f"{self.prefix}/{kind}/{rank}"

    def report_failure(self, reason: str, kind: str = "failed") -> None:
        """kind "failed": this rank is the cause; "lost": it stopped because a
        peer failed or stalled."""
        self.store.set(self._key(kind, self.rank), reason[:1000])

    def _failed_peer(self, include_lost: bool = False):
        """The first peer that reported a failure it caused, else (optionally)
        the first peer that stopped because of another."""
        for kind in ("failed", "lost") if include_lost else ("failed",):
            for r in range(self.world):
                if r != self.rank and self.store.check([self._key(kind, r)]):
                    return r, self.store.get(self._key(kind, r)).decode(errors="replace")
        return None

    def wait_for_peers(self) -> None:
        """Before issuing step ``self.step + 1``: every peer finished
        ``self.step`` (or the job just started). Raises RankFailure or
        RankTimeout instead of letting the next collective block."""
        need = self.step
        t0 = time.monotonic()
        while True:
            failed = self._failed_peer(include_lost=True)
            if failed is not None:
                self.report_failure(f"peer rank {failed[0]} stopped", "lost")
                raise RankFailure(*failed)
            late = []
            for r in range(self.world):
                if r == self.rank or need == 0:
                    continue
                k = self._key("hb", r)
                if not self.store.check([k]) or int(self.store.get(k)) < need:
                    late.append(r)
            if not late:
                return
            if time.monotonic() - t0 > self.deadline:
                raise RankTimeout(late, need, self.deadline)
            time.sleep(0.01)

    def step_done(self) -> None:
        self.step += 1
        self.store.set(self._key("hb", self.rank), str(self.step))

    def _not_started(self, step: int):
        late = []
        for r in range(self.world):
            k = self._key("begin", r)
            if r != self.rank and (not self.store.check([k]) or int(self.store.get(k)) < step):
                late.append(r)
        return late

    @contextlib.contextmanager
    def step_guard(self):
        """Wraps one step: waits for the peers first, publishes a heartbeat after,
        and publishes this rank's failure if the step raises. When the step's
        collective fails (the process group's timeout ended it), the cause is
        named: a peer that reported a failure (RankFailure) or peers that never
        began the step (RankTimeout)."""
        self.wait_for_peers()
        k = self.step + 1
        self.store.set(self._key("begin", self.rank), str(k))
        try:
            yield
        except BaseException as e:  # the peers must learn of any exit
            if isinstance(e, (RankFailure, RankTimeout)):
                self.report_failure(str(e), "lost")
                raise
            comm = _is_comm_error(e)
            failed = self._failed_peer()
            t0 = time.monotonic()
            while comm and failed is None and time.monotonic() - t0 < self.grace:
                # the collective failed because a peer left: it publishes why
                # before its connections close, so give the report a moment
                time.sleep(0.05)
                failed = self._failed_peer()
            if failed is not None:
                self.report_failure(f"peer rank {failed[0]} failed", "lost")
                raise RankFailure(*failed) from e
            if comm:
                late = self._not_started(k)
                if late:
                    self.report_failure(f"peer ranks {late} stalled", "lost")
                    raise RankTimeout(late, k, self.deadline) from e
            # this rank's own step raised: it is the cause
            self.report_failure(f"{type(e).__name__}: {e}")
            raise
        self.step_done()

    @contextlib.contextmanager
    def run(self):
        """Wraps a rank's whole loop: any exit by exception between steps is
        published too."""
        try:
            yield self
        except BaseException as e:
            try:
                if not any(self.store.check([self._key(kind, self.rank)])
                           for kind in ("failed", "lost")):
                    self.report_failure(f"{type(e).__name__}: {e}")
            except Exception:
                # The store is gone (its host process ended): the peers learn of
                # this exit from their collective's timeout instead, and the
                # original exception is what this rank reports.
                pass
            raise
