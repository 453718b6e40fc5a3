"""Request sharding of the FM head across the GPUs of one box.

Requests are independent units: each request's FM state (history rows, K/V
pages, g_cond) is private to it (``engine.py:26-29,286-319`` of the reference),
so the head scales by giving every GPU its own ``B200FMHead`` (one process per
GPU) and pinning each request to one GPU for its whole life.  The data path has
no collective; the only cross-rank traffic is the optional gather of the output
latents (128 KiB per GPU per tick at 64 requests) to the rank that owns the
engine, and a heartbeat in the rendezvous store for failure detection.

``LeastLoadedSharder`` is the placement policy: a new request goes to the rank
with the smallest load, where load is the rows of K/V the rank streams per tick
(the attention bytes, which dominate a tick), so short and long requests mix
across GPUs (75 % short, 25 % long prefixes).
"""
from __future__ import annotations

import dataclasses
import time

import torch
import torch.distributed as dist


@dataclasses.dataclass
class Placement:
    rank: int
    rows: int


class LeastLoadedSharder:
    """Host-side placement of requests on ranks (pure bookkeeping)."""

    def __init__(self, world: int, stride: int = 17, max_per_rank: int | None = None):
        if world < 1:
            raise ValueError("world must be >= 1")
        self.world = world
        self.stride = stride
        self.max_per_rank = max_per_rank
        self.place: dict[object, Placement] = {}
        self.load = [0] * world
        self.count = [0] * world
        self.dead: set[int] = set()

    def _cost(self, rows: int) -> int:
        return rows + 2 * self.stride

    def assign(self, rid, rows: int = 0) -> int:
        if rid in self.place:
            return self.place[rid].rank
        live = [r for r in range(self.world) if r not in self.dead
                and (self.max_per_rank is None or self.count[r] < self.max_per_rank)]
        if not live:
            raise RuntimeError("no rank can take another FM request")
        r = min(live, key=lambda k: (self.load[k], self.count[k], k))
        self.place[rid] = Placement(r, rows)
        self.load[r] += self._cost(rows)
        self.count[r] += 1
        return r

    def grow(self, rid, rows: int) -> None:
        """A request's cache grew by ``rows`` (one tick graduates a patch)."""
        p = self.place[rid]
        p.rows += rows
        self.load[p.rank] += rows

    def release(self, rid) -> None:
        p = self.place.pop(rid, None)
        if p is not None:
            self.load[p.rank] -= self._cost(p.rows)
            self.count[p.rank] -= 1

    def by_rank(self, rids) -> list[list]:
        out = [[] for _ in range(self.world)]
        for rid in rids:
            out[self.place[rid].rank].append(rid)
        return out

    def mark_dead(self, rank: int) -> list:
        """Take a rank out of service; return its requests, which lose their
        cache and must be re-placed (and re-prefilled) on the survivors."""
        self.dead.add(rank)
        lost = [rid for rid, p in self.place.items() if p.rank == rank]
        for rid in lost:
            self.release(rid)
        return lost


class Heartbeat:
    """Per-rank liveness in the process group's store: each rank bumps
    ``fm_hb/<rank>`` once per tick; the scheduling rank checks, before it
    dispatches a tick, that every rank's beat is recent.  A rank that raised,
    exited or stopped ticking is reported without any GPU-side wait."""

    def __init__(self, store: dist.Store, rank: int, world: int, timeout_s: float = 5.0):
        self.store, self.rank, self.world, self.timeout_s = store, rank, world, timeout_s

    def beat(self, tick: int) -> None:
        self.store.set(f"fm_hb/{self.rank}", f"{tick}:{time.time():.6f}")

    def stale(self) -> list[int]:
        now = time.time()
        bad = []
        for r in range(self.world):
            try:
                self.store.wait([f"fm_hb/{r}"], _td(self.timeout_s))
                _, ts = self.store.get(f"fm_hb/{r}").decode().split(":")
                if now - float(ts) > self.timeout_s:
                    bad.append(r)
            except Exception:
                bad.append(r)
        return bad


def _td(s: float):
    import datetime
    return datetime.timedelta(seconds=s)


def gather_latents(local: torch.Tensor, counts: list[int], dst: int = 0):
    """Gather every rank's [n_r, lp, ld] output on ``dst`` (concatenated in rank
    order).  Pads to the largest n_r so one all_gather serves every rank."""
    world = dist.get_world_size()
    m = max(counts)
    buf = local.new_zeros((m,) + tuple(local.shape[1:]))
    buf[: local.shape[0]] = local
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf)
    if dist.get_rank() != dst:
        return None
    return torch.cat([p[:c] for p, c in zip(parts, counts)], dim=0)
