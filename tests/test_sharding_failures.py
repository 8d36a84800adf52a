"""Rank failures on the sharded host path, made on the host (gloo ranks on CPU, no GPU):
a rank that leaves between steps, a rank that is late, a rank that sends a corrupted size,
and a collective whose peer is gone.  The survivors must end with a clean error, in bounded
time, never a hang."""
import os
import socket
import sys
import time
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from nexusquant_b200 import sharding as S  # noqa: E402

L, H, PB = 6, 3, 1


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _sizes(plan, corrupt=False):
    comp = [1000 + l for l in plan.quantized]
    prot = [5000 + l for l in plan.protected]
    t = S.local_layer_sizes(plan, comp, prot)
    if corrupt:
        t[plan.layers[0]] = -7
    return t


def _expected(r, l):
    return 5000 + l if l in S.protected_layers(L, PB) else 1000 + l


def _exit(q, code=0):
    """Leave at once, after the queue's feeder thread has delivered what was put."""
    q.close()
    q.join_thread()
    os._exit(code)


def _worker(rank, world, port, q, scenario):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=4))
        store = dist.distributed_c10d._get_default_store()
        plan = S.make_plan(L, H, PB, rank, world)
        # step 0: everyone present
        S.step_checkpoint(store, rank, world, 0, timeout=20)
        table = S.gather_layer_index(_sizes(plan), plan)
        S.validate_index(table, L, H, PB, _expected)
        if scenario == "exit" and rank == world - 1:
            q.put((rank, "left"))
            _exit(q)  # leaves between steps, without joining step 1
        if scenario == "late" and rank == 1:
            time.sleep(1.5)
        t0 = time.monotonic()
        try:
            if scenario != "collective":
                S.step_checkpoint(store, rank, world, 1, timeout=3 if scenario == "exit" else 20)
            elif rank == world - 1:
                q.put((rank, "left"))
                _exit(q)
            table = S.gather_layer_index(_sizes(plan, corrupt=(scenario == "corrupt" and rank == 1)), plan)
            S.validate_index(table, L, H, PB, _expected)
            q.put((rank, "ok"))
        except S.RankFailure as e:
            q.put((rank, f"RankFailure after {time.monotonic() - t0:.1f}s: {e}"))
        except RuntimeError as e:  # the process group's own timeout on a collective
            q.put((rank, f"RuntimeError after {time.monotonic() - t0:.1f}s: {type(e).__name__}"))
        if scenario in ("exit", "collective"):
            _exit(q)  # the group cannot be torn down cleanly without the departed rank
        dist.destroy_process_group()
        _exit(q)
    except Exception as e:
        q.put((rank, f"unexpected {type(e).__name__}: {e}"))
        _exit(q, 1)


def _run(world, scenario):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, scenario)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, st = q.get(timeout=120)
            res[r] = st
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return res


def test_rank_leaving_between_steps_is_named():
    res = _run(3, "exit")
    assert res[2] == "left"
    for r in (0, 1):
        assert res[r].startswith("RankFailure") and "[2]" in res[r] and "step 1" in res[r], res


def test_late_rank_is_waited_for():
    res = _run(3, "late")
    assert all(v == "ok" for v in res.values()), res


def test_corrupted_size_is_rejected_on_every_rank():
    res = _run(3, "corrupt")
    for r in range(3):
        assert res[r].startswith("RankFailure") and "rank 1" in res[r], res


def test_collective_with_a_departed_peer_times_out():
    res = _run(2, "collective")
    assert res[1] == "left"
    assert res[0].startswith("RuntimeError"), res
