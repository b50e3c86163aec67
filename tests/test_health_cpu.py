"""Tensor-parallel group health on CPU ranks (gloo): a rank that stops beating between steps is
detected by the survivors, which plan a smaller group and keep serving on it. No GPU involved."""
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from appcorr_b200.parallel.health import Heartbeat, plan_fallback


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    store = dist.distributed_c10d._get_default_store()
    hb = Heartbeat(store, rank, world, interval=0.05)
    t = torch.ones(1)
    dist.all_reduce(t)                      # one healthy step on the full group
    assert t.item() == world
    if rank == world - 1:                   # this rank leaves between steps
        hb.stop()
        q.put((rank, "left", None))
        time.sleep(3.0)                     # stays alive (store server lives on rank 0) but silent
        return
    deadline = time.monotonic() + 10
    dead = []
    while time.monotonic() < deadline:
        dead = hb.dead_ranks(timeout=0.5)
        if dead:
            break
        time.sleep(0.05)
    alive = [r for r in range(world) if r not in dead]
    plan = plan_fallback(alive, num_heads=32, hidden=4096)
    grp = dist.new_group(ranks=alive, use_local_synchronization=True)
    t = torch.ones(1)
    dist.all_reduce(t, group=grp)           # the survivors keep serving on the re-formed group
    q.put((rank, dead, (plan.tp, plan.dp, t.item())))
    hb.stop()
    time.sleep(0.5)


def test_dead_rank_detected_and_group_reformed():
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, dead, info = q.get(timeout=60)
        res[r] = (dead, info)
    for p in procs:
        p.join(timeout=30)
    assert res[2][0] == "left"
    for r in (0, 1):
        dead, (tp, dp, s) = res[r]
        assert dead == [2]
        assert (tp, dp) == (2, 1) and s == 2.0


def test_plan_fallback_degrees():
    p = plan_fallback([0, 1, 2, 3, 4, 5, 6], num_heads=32, hidden=4096)
    assert (p.tp, p.dp, p.groups, p.idle) == (4, 1, [[0, 1, 2, 3]], [4, 5, 6])
    p = plan_fallback([0, 1, 2, 3, 4, 5, 6, 7], num_heads=32, hidden=4096, max_tp=2)
    assert (p.tp, p.dp) == (2, 4)
    p = plan_fallback([3], num_heads=6, hidden=384)
    assert (p.tp, p.dp, p.groups) == (1, 1, [[3]])
    with pytest.raises(RuntimeError):
        plan_fallback([], 32, 4096)
