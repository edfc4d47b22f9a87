"""A rank that leaves the group between steps (CPU ranks over gloo, world 2).

Rank 1 finishes step 0 and exits.  With the step heartbeat, rank 0 learns it
on the host before launching step 1 (RankFailure naming rank 1, within the
heartbeat's timeout, no collective in flight); without it, rank 0's next
collective ends with an error instead of blocking."""
import os
import socket
import time
from datetime import timedelta

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _report(q, msg):
    q.put(msg)
    q.close()
    q.join_thread()  # flush to the pipe before os._exit skips interpreter teardown
    os._exit(0)


def _rank_main(rank, world, port, q, use_heartbeat):
    from teenyformers_b200.health import RankFailure, StepHeartbeat
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    hb = StepHeartbeat(dist.distributed_c10d._get_default_store(), rank, world, timeout=2.0)
    t = torch.ones(4)
    for step in range(3):
        if rank == 1 and step == 1:
            os._exit(0)  # leaves between steps, nothing of its own in flight
        t0 = time.monotonic()
        try:
            if use_heartbeat:
                hb.beat(step)
                hb.check(step)
            dist.all_reduce(t)
        except RankFailure as e:
            _report(q, ("rank_failure", rank, step, e.missing, time.monotonic() - t0))
        except Exception as e:  # the collective's own error
            _report(q, ("collective_error", rank, step, type(e).__name__, time.monotonic() - t0))
    _report(q, ("finished", rank, 3, None, 0.0))


def _run(use_heartbeat):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q, use_heartbeat))
             for r in range(2)]
    for p in procs:
        p.start()
    msg = q.get(timeout=60)
    for p in procs:
        p.join(30)
        if p.is_alive():
            p.terminate()
            p.join(10)
    return msg


def test_heartbeat_reports_a_departed_rank_before_the_next_step():
    kind, rank, step, missing, dt = _run(True)
    assert (kind, rank, step, missing) == ("rank_failure", 0, 1, [1])
    assert 1.5 < dt < 10


def test_collective_with_a_departed_rank_errors_instead_of_hanging():
    kind, rank, step, _, dt = _run(False)
    assert (kind, rank, step) == ("collective_error", 0, 1)
    assert dt < 20
