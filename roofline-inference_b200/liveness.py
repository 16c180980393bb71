"""Host-side liveness of the ranks between steps of a multi-GPU job.

The reference runs every timed unit in a process of its own and, when one
does not come back, writes an exclusion record (gate_timeout, worker_crash,
...) and retries the unit once (agent-test/v3/worker.py:124-141,
run.py:238-261, 347-353).  Its engine is single-device, so it has no peer to
lose mid-job.  Here the ranks of one job check each other on the host before
every step: a rank posts its arrival for step s in the torch.distributed
store and waits, bounded, until every peer has either arrived or announced
that it left.  A rank that leaves between steps -- cleanly (leave()) or by
dying -- is therefore seen by every other rank before any of them enqueues
the step's kernels or collectives, so no GPU spins on a peer that is gone;
the device-side waits (bounded too, rib_set_wait_limit_ns) are the second
line for a peer that dies inside a step.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field


@dataclass
class StepReport:
    """Outcome of one arrival: the peers present, those that announced their
    departure (rank -> the step before which they left) and those that did
    neither within the timeout."""
    step: int
    present: list[int] = field(default_factory=list)
    departed: dict[int, int] = field(default_factory=dict)
    missing: list[int] = field(default_factory=list)

    @property
    def ok(self) -> bool:
        return not self.departed and not self.missing


class StepGuard:
    """Per-rank guard over a torch.distributed store (TCPStore, FileStore,
    or the default group's store).  Every rank calls arrive(s) for the same
    steps in the same order; a rank that stops calls leave(s) first when it
    can."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 5.0, prefix: str = "rib/step",
                 poll_s: float = 0.005):
        if not (0 <= rank < world):
            raise ValueError("rank must be in [0, world)")
        if timeout_s <= 0:
            raise ValueError("timeout_s must be positive")
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.prefix, self.poll_s = timeout_s, prefix, poll_s

    def _arrive_key(self, step: int, rank: int) -> str:
        return f"{self.prefix}/{step}/{rank}"

    def _left_key(self, rank: int) -> str:
        return f"{self.prefix}/left/{rank}"

    def leave(self, step: int) -> None:
        """Announces that this rank takes no part in `step` or any later one."""
        self.store.set(self._left_key(self.rank), str(int(step)))

    def arrive(self, step: int) -> StepReport:
        """Posts this rank's arrival at `step` and waits (at most timeout_s)
        for every peer's arrival or departure notice."""
        self.store.set(self._arrive_key(step, self.rank), "1")
        rep = StepReport(step, present=[self.rank])
        pending = [r for r in range(self.world) if r != self.rank]
        deadline = time.monotonic() + self.timeout_s
        while pending:
            still = []
            for r in pending:
                if self.store.check([self._arrive_key(step, r)]):
                    rep.present.append(r)
                elif self.store.check([self._left_key(r)]):
                    rep.departed[r] = int(self.store.get(self._left_key(r)))
                else:
                    still.append(r)
            pending = still
            if pending and time.monotonic() >= deadline:
                rep.missing = sorted(pending)
                break
            if pending:
                time.sleep(self.poll_s)
        rep.present.sort()
        return rep
