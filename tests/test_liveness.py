"""CPU: ranks that leave a multi-rank job between steps (gloo, world 3).

Failure is made on the host, as the pool requires: one rank announces that
it leaves and exits between steps, or dies between steps without a word.
The survivors must see it through liveness.StepGuard before they issue the
next collective, stop cleanly, and have computed every earlier step right.
The reference's analogue is the v3 harness's exclusion records and one retry
per excluded unit (agent-test/v3/run.py:238-261, 347-353)."""
from __future__ import annotations

import importlib
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, stop_rank, stop_step, steps, q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(root))
    import datetime
    import torch.distributed as dist
    liveness = importlib.import_module("roofline-inference_b200.liveness")
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=30))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    guard = liveness.StepGuard(store, rank, world, timeout_s=1.0)
    sums, report = [], None
    for s in range(steps):
        if rank == stop_rank and s == stop_step:
            if mode == "leave":
                guard.leave(s)
                q.put((rank, "left", s, sums, None))
                return  # no collective in flight; the process exits
            q.put((rank, "died", s, sums, None))
            q.close()
            q.join_thread()  # the test's record of it, flushed before the process dies
            os._exit(0)  # dies without a word to its peers
        rep = guard.arrive(s)
        if not rep.ok:
            report = (rep.step, sorted(rep.departed), rep.missing)
            break
        t = torch.tensor([float(rank + 1) * (s + 1)])
        dist.all_reduce(t)
        sums.append(float(t.item()))
    q.put((rank, "stopped" if report else "done", len(sums), sums, report))
    if rank == 0:  # the store's server stays up until every survivor has read the report
        store.wait([f"rib/done/{r}" for r in range(1, world) if r != stop_rank])
    store.set(f"rib/done/{rank}", "1")
    dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["leave", "die"])
def test_rank_leaves_between_steps(mode):
    world, stop_rank, stop_step, steps = 3, 2, 3, 6
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, stop_rank, stop_step, steps, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, *rest = q.get(timeout=60)
        res[rank] = rest
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[stop_rank][0] == ("left" if mode == "leave" else "died")
    want = [sum(float(r + 1) * (s + 1) for r in range(world)) for s in range(stop_step)]
    for r in range(world):
        if r == stop_rank:
            continue
        status, n, sums, report = res[r]
        assert status == "stopped" and n == stop_step
        assert sums == want  # every step before the departure was right
        step, departed, missing = report
        assert step == stop_step
        if mode == "leave":
            assert departed == [stop_rank] and missing == []
        else:
            assert departed == [] and missing == [stop_rank]


def test_step_guard_all_present_single_process():
    import datetime
    import torch.distributed as dist
    liveness = importlib.import_module("roofline-inference_b200.liveness")
    store = dist.HashStore()
    store.set("rib/step/0/1", "1")
    g = liveness.StepGuard(store, 0, 2, timeout_s=0.2)
    rep = g.arrive(0)
    assert rep.ok and rep.present == [0, 1]
    rep = g.arrive(1)
    assert rep.missing == [1] and not rep.ok
    store.set("rib/step/left/1", "2")
    rep = g.arrive(2)
    assert rep.departed == {1: 2} and rep.missing == []
    with pytest.raises(ValueError):
        liveness.StepGuard(store, 2, 2)
    del datetime
