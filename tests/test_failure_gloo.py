"""Failure detection of the sharded step on the host, with gloo ranks on the
CPU (no GPU is faulted, trapped or hung): a rank that raises, or one that
stalls before a step, turns into RankFailure / RankTimeout on the other ranks
within the process group's short timeout instead of a hang."""
import datetime
import os
import socket
import sys
import time

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WORLD = 3


def _worker(rank, port, q, scenario):
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist

    from magicmindnet_b200.failure import RankFailure, RankMonitor, RankTimeout

    # The store is served by the parent process, so it outlives every rank:
    # a rank that exits first cannot take it down under the others.
    store = dist.TCPStore("127.0.0.1", port, WORLD + 1, False,
                          timeout=datetime.timedelta(seconds=30))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=3))
    mon = RankMonitor(store, rank, WORLD, deadline_s=10.0)
    t0 = time.monotonic()
    outcome = ("done", None)
    try:
        with mon.run():
            for step in range(1, 6):
                if scenario == "stall" and rank == 2 and step == 3:
                    time.sleep(8.0)  # never begins step 3 in time
                    outcome = ("stalled", None)
                    break
                with mon.step_guard():
                    if scenario == "raise" and rank == 1 and step == 3:
                        raise ValueError("injected failure")
                    x = torch.ones(1)
                    dist.all_reduce(x)
    except RankFailure as e:
        outcome = ("RankFailure", e.rank)
    except RankTimeout as e:
        outcome = ("RankTimeout", e.ranks)
    except ValueError:
        outcome = ("ValueError", None)
    q.put((rank, outcome, time.monotonic() - t0))
    q.close()
    q.join_thread()  # the result is sent before the process ends
    os._exit(0)


def _run(scenario):
    import torch.distributed as dist
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    server = dist.TCPStore("127.0.0.1", port, WORLD + 1, True,
                           timeout=datetime.timedelta(seconds=30), wait_for_workers=False)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, port, q, scenario)) for r in range(WORLD)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(WORLD):
        r, outcome, dt = q.get(timeout=120)
        got[r] = (outcome, dt)
    for p in procs:
        p.join(timeout=60)
    del server
    return got


def test_a_rank_that_raises_is_reported_to_the_others():
    got = _run("raise")
    assert got[1][0] == ("ValueError", None)
    for r in (0, 2):
        assert got[r][0] == ("RankFailure", 1), got
        assert got[r][1] < 60.0


def test_a_rank_that_stalls_times_out_on_the_others():
    got = _run("stall")
    assert got[2][0] == ("stalled", None)
    for r in (0, 1):
        assert got[r][0] == ("RankTimeout", [2]), got
        assert got[r][1] < 60.0
