"""Failure detection on the host (no GPU): gloo ranks on the CPU, one of which
leaves between steps.  The survivors must learn of it before their next
launch (PeerWatch over the process group's store raises PeerLost), and a
collective already waiting on the departed rank must end with an error
through the process group's timeout rather than hang."""
import datetime
import os
import time

import pytest
import torch.multiprocessing as mp


def _join_all(ctx, limit_s=60.0):
    """ProcessContext.join returns after any one process ends; wait for all."""
    t_end = time.time() + limit_s
    while not ctx.join(timeout=max(t_end - time.time(), 0.1)):
        if time.time() > t_end:
            for p in ctx.processes:
                if p.is_alive():
                    p.kill()
            raise AssertionError("ranks still running after the limit")


def _init(rank, world, port, timeout_s):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _watch_worker(rank, world, port, leave_after, results):
    from sparsemoe_b200.health import PeerLost, PeerWatch
    dist = _init(rank, world, port, 30)
    w = PeerWatch(PeerWatch.default_store(), rank, world, timeout_s=2.0)
    steps = 0
    try:
        for _ in range(4):
            if rank == world - 1 and steps == leave_after:
                results[rank] = ("left", steps, [])
                os._exit(0)                           # leaves between steps, no teardown
            w.step()
            steps += 1
        results[rank] = ("done", steps, [])
    except PeerLost as e:
        results[rank] = ("peer_lost", steps, e.missing)
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_peer_leaving_between_steps_is_detected_before_the_next_step(world):
    port = 29400 + os.getpid() % 500 + world
    with mp.Manager() as m:
        res = m.dict()
        t0 = time.time()
        ctx = mp.spawn(_watch_worker, args=(world, port, 2, res), nprocs=world, join=False)
        _join_all(ctx)
        res = dict(res)
    assert time.time() - t0 < 60
    assert res[world - 1] == ("left", 2, [])
    for r in range(world - 1):
        status, steps, missing = res[r]
        assert status == "peer_lost" and steps == 2 and missing == [world - 1], res[r]


def _collective_worker(rank, world, port, results):
    import torch
    dist = _init(rank, world, port, 3)
    t = torch.ones(4)
    dist.all_reduce(t)                                # one good step
    if rank == 1:
        results[rank] = "left"
        os._exit(0)
    t0 = time.time()
    try:
        dist.all_reduce(t)                            # the peer is gone: must error, not hang
        results[rank] = ("completed", time.time() - t0)
    except Exception as e:                            # noqa: BLE001 (the backend's error type varies)
        results[rank] = ("error", time.time() - t0, type(e).__name__)


def test_collective_after_a_peer_left_ends_with_an_error():
    port = 29950 + os.getpid() % 40
    with mp.Manager() as m:
        res = m.dict()
        ctx = mp.spawn(_collective_worker, args=(2, port, res), nprocs=2, join=False)
        _join_all(ctx)
        res = dict(res)
    assert res[1] == "left"
    assert res[0][0] == "error" and res[0][1] < 30, res[0]
