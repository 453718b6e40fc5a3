"""Request sharding across ranks (host logic + a 2-rank gloo run on the CPU)."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from nanovllm_dots_b200.sharding import Heartbeat, LeastLoadedSharder, gather_latents


def test_least_loaded_balances_rows():
    s = LeastLoadedSharder(world=2)
    assert s.assign("long", 5000) == 0
    assert s.assign("a", 100) == 1
    assert s.assign("b", 100) == 1
    assert s.assign("c", 100) == 1
    s.grow("a", 17)
    assert s.by_rank(["long", "a", "b", "c"]) == [["long"], ["a", "b", "c"]]
    s.release("long")
    assert s.assign("d", 0) == 0
    assert s.assign("a") == 1          # sticky for the request's whole life


def test_capacity_and_dead_rank():
    s = LeastLoadedSharder(world=3, max_per_rank=1)
    assert [s.assign(i, 10 * i) for i in range(3)] == [0, 1, 2]
    with pytest.raises(RuntimeError):
        s.assign("x")
    lost = s.mark_dead(1)
    assert lost == [1]
    s.max_per_rank = 2
    assert s.assign(1, 10) in (0, 2)
    assert 1 not in [p.rank for p in s.place.values()]


def test_mix_spreads_long_requests():
    g = torch.Generator().manual_seed(4)
    rows = [17 * (int(torch.randint(200, 321, (1,), generator=g)) if i % 4 == 0 else
                  int(torch.randint(0, 61, (1,), generator=g))) for i in range(64)]
    s = LeastLoadedSharder(world=8)
    for i, r in enumerate(rows):
        s.assign(i, r)
    assert max(s.load) < 1.5 * (sum(s.load) / 8)


def _free_port():
    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        return so.getsockname()[1]


def _worker(rank, world, port, fail_rank, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    store = dist.distributed_c10d._get_default_store()
    hb = Heartbeat(store, rank, world, timeout_s=2.0)
    try:
        counts = [3, 2]
        local = torch.full((counts[rank], 16, 64), float(rank))
        hb.beat(0)
        out = gather_latents(local, counts)
        if rank == 0:
            q.put(("gather", out.shape[0], float(out[:3].mean()), float(out[3:].mean())))
        dist.barrier()
        if rank == fail_rank:
            return                      # leaves between ticks, never beats again
        hb.beat(1)
        if rank == 0:
            import time
            time.sleep(2.5)
            hb.beat(2)
            q.put(("stale", hb.stale()))
    finally:
        pass


def test_two_rank_gather_and_heartbeat():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, 1, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
    msgs = {}
    while not q.empty():
        m = q.get()
        msgs[m[0]] = m[1:]
    assert msgs["gather"] == (5, 0.0, 1.0)
    assert msgs["stale"][0] == [1]
