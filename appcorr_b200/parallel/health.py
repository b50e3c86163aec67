"""Tensor-parallel group health: host-side heartbeats, failure detection and re-forming the group.

The reference is single-GPU and has no multi-process failure handling beyond its socket retries;
this module covers the multi-GPU serving group of this build. Everything here runs on the host:

    Heartbeat      every rank bumps a counter under `hb/<rank>` in the torch.distributed store
                   from a daemon thread; a rank whose counter has not moved for `timeout` seconds
                   (on the observer's clock) is considered dead.
    check_group    combines the heartbeat view with the device error word of the peer-memory
                   collectives (a bounded wait that expired reports a missing peer without a hang).
    plan_fallback  the largest tensor-parallel degree the surviving ranks can still serve
                   (a power of two that divides the heads and the hidden size), with the remaining
                   ranks as data-parallel replicas.
    reform_group   a new process group over the survivors (only the survivors take part).

A rank leaves only between steps, with none of its kernels in flight; the survivors learn of it on
the host before their next launch, tear down the peer mappings (TPComm.close) and rebuild.
"""
from __future__ import annotations

import threading
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import torch.distributed as dist


class Heartbeat:
    def __init__(self, store: "dist.Store", rank: int, world: int, interval: float = 0.2, prefix: str = "hb"):
        self.store, self.rank, self.world = store, rank, world
        self.interval, self.prefix = interval, prefix
        self._count = 0
        self._stop = threading.Event()
        self._seen: Dict[int, tuple] = {}       # rank -> (last value, local time it changed)
        self._beat()
        self._thread = threading.Thread(target=self._run, name=f"heartbeat-{rank}", daemon=True)
        self._thread.start()

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def _beat(self) -> None:
        self._count += 1
        self.store.set(self._key(self.rank), str(self._count))

    def _run(self) -> None:
        while not self._stop.wait(self.interval):
            try:
                self._beat()
            except Exception:  # the store itself went away: stop beating
                return

    def stop(self) -> None:
        self._stop.set()
        self._thread.join(timeout=2 * self.interval + 1)

    def observe(self) -> Dict[int, float]:
        """Seconds since each peer's heartbeat last changed (0 for this rank)."""
        now = time.monotonic()
        ages: Dict[int, float] = {}
        for r in range(self.world):
            if r == self.rank:
                ages[r] = 0.0
                continue
            try:
                val = self.store.get(self._key(r)).decode() if self.store.check([self._key(r)]) else None
            except Exception:
                val = None
            last = self._seen.get(r)
            if last is None or last[0] != val:  # first sight, or the counter moved
                self._seen[r] = (val, now)
                ages[r] = 0.0
            else:
                ages[r] = now - last[1]
        return ages

    def dead_ranks(self, timeout: float) -> List[int]:
        return sorted(r for r, age in self.observe().items() if age > timeout)


@dataclass
class FallbackPlan:
    alive: List[int]
    tp: int
    dp: int
    groups: List[List[int]] = field(default_factory=list)  # tensor-parallel groups (global ranks)
    idle: List[int] = field(default_factory=list)          # survivors left out of every group


def plan_fallback(alive: Sequence[int], num_heads: int, hidden: int, max_tp: Optional[int] = None) -> FallbackPlan:
    """Largest power-of-two TP degree <= len(alive) (and <= max_tp) that divides the heads and the
    hidden size; the survivors form len(alive) // tp replicas of that degree."""
    alive = sorted(alive)
    if not alive:
        raise RuntimeError("no surviving ranks")
    tp = 1
    limit = min(len(alive), max_tp or len(alive))
    while tp * 2 <= limit and num_heads % (tp * 2) == 0 and hidden % (tp * 2) == 0:
        tp *= 2
    dp = len(alive) // tp
    groups = [alive[i * tp:(i + 1) * tp] for i in range(dp)]
    return FallbackPlan(alive=alive, tp=tp, dp=dp, groups=groups, idle=alive[dp * tp:])


def check_group(hb: Heartbeat, timeout: float, comm=None) -> List[int]:
    """Dead peers by heartbeat; a device-side collective timeout (TPComm.check raising) with no
    heartbeat casualty is reported as an unknown peer (-1) so the caller still re-forms."""
    dead = hb.dead_ranks(timeout)
    if comm is not None:
        try:
            comm.check()
        except RuntimeError:
            if not dead:
                dead = [-1]
    return dead


def reform_group(alive: Sequence[int], backend: Optional[str] = None):
    """Process group over the survivors; only the survivors call this."""
    return dist.new_group(ranks=sorted(alive), backend=backend, use_local_synchronization=True)
