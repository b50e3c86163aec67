"""Host shared-memory broadcast ring (csrc/runtime/shm_ring.cpp): one producer, several consumer
processes, wrap-around, bounded waits, and a detached (dead) consumer no longer blocking."""
import multiprocessing as mp
import os
import uuid

import pytest


def _ring():
    from appcorr_b200 import _runtime

    return _runtime


def _consumer(name, cid, n, q):
    R = _ring()
    r = R.ShmRing(name, create=False)
    got = []
    for _ in range(n):
        b = r.pop(cid, 10.0)
        if b is None:
            break
        got.append(b)
    q.put((cid, [len(b) for b in got], [b[:8] for b in got]))
    r.release()


def test_broadcast_ring_three_consumers_with_wraparound():
    R = _ring()
    name = f"/appcorr_test_{os.getpid()}_{uuid.uuid4().hex[:8]}"
    ring = R.ShmRing(name, 1 << 14, 3, True)   # 16 KiB: the 40 records below wrap several times
    try:
        ctx = mp.get_context("spawn")
        q = ctx.Queue()
        procs = [ctx.Process(target=_consumer, args=(name, c, 40, q)) for c in range(3)]
        for p in procs:
            p.start()
        sizes = [(i * 977) % 3000 + 1 for i in range(40)]
        for i, s in enumerate(sizes):
            payload = (b"%08d" % i) + bytes([i % 251]) * (s - 8 if s > 8 else 0)
            assert ring.push(payload[:max(s, 8)], 10.0)
        res = sorted(q.get(timeout=60) for _ in procs)
        for p in procs:
            p.join(timeout=30)
        for cid, lens, heads in res:
            assert lens == [max(s, 8) for s in sizes], cid
            assert heads == [b"%08d" % i for i in range(40)]
    finally:
        ring.unlink()


def test_full_ring_times_out_until_a_dead_consumer_is_detached():
    R = _ring()
    name = f"/appcorr_test_{os.getpid()}_{uuid.uuid4().hex[:8]}"
    ring = R.ShmRing(name, 1 << 12, 2, True)
    try:
        ok = 0
        while ring.push(b"x" * 1000, 0.05):   # nobody reads: fills up, then the push times out
            ok += 1
        assert ok == 4
        reader = R.ShmRing(name, create=False)
        assert reader.pop(0, 1.0) == b"x" * 1000   # consumer 0 alive and reading
        assert not ring.push(b"y" * 1000, 0.05)    # consumer 1 (dead) still pins the space
        ring.detach(1)
        assert ring.push(b"y" * 1000, 0.05)        # no longer waited for
        assert reader.pop(0, 0.01) == b"x" * 1000
        ring.close()
        for _ in range(3):
            reader.pop(0, 0.01)
        assert reader.pop(0, 0.01) is None         # closed and drained
        reader.release()
    finally:
        ring.unlink()
