"""Host request router over replicas: slot-table logic in-process, and the tick protocol
over two gloo ranks on CPU (fake engines, no GPU)."""
from __future__ import annotations

import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from tests.conftest import load_pkg

load_pkg()                                            # spawned ranks import this module afresh
import z2b.replicas as RP  # noqa: E402


def test_least_loaded_admission_and_reuse():
    t = RP.SlotTable(3, 2)
    picks = []
    for _ in range(6):
        r = t.pick()
        picks.append((r, t.take(r)))
    assert picks == [(0, 0), (1, 0), (2, 0), (0, 1), (1, 1), (2, 1)]
    assert t.pick() is None
    t.give_back(1, 1)
    t.give_back(1, 0)
    assert t.pick() == 1 and t.take(1) == 0


def test_router_single_process_serves_every_request_once():
    reqs = RP.poisson_requests(40, 0.5, (8, 32), (3, 20), seed=1)
    eng = RP.FakeEngine(4)
    ticks, frames, done = RP.serve(eng, reqs, 4)
    assert sorted(done) == list(range(40))
    assert frames == sum(r.gen_frames for r in reqs)


def test_dispatch_partitions_the_arrivals():
    reqs = RP.poisson_requests(101, 2.0, (32, 256), (300, 1500), seed=4)
    parts = [RP.dispatch(reqs, 4, r) for r in range(4)]
    ids = sorted(x.rid for p in parts for x in p)
    assert ids == list(range(101))
    assert max(len(p) for p in parts) - min(len(p) for p in parts) <= 1
    for p in parts:                                   # each replica's queue stays in arrival order
        assert [x.arrival_tick for x in p] == sorted(x.arrival_tick for x in p)


def test_local_admission_waits_for_arrivals_and_free_slots():
    reqs = [RP.Request(0, 10, 5, 0), RP.Request(1, 10, 2, 0), RP.Request(2, 10, 3, 3), RP.Request(3, 10, 1, 4)]
    eng = RP.FakeEngine(2)
    admitted = []
    orig = eng.admit

    def admit(rid, slot, p, g):
        admitted.append((len(admitted), rid, slot))
        orig(rid, slot, p, g)

    eng.admit = admit
    ticks, frames, done = RP.serve_local(eng, reqs, 2)
    assert [a[1:] for a in admitted] == [(0, 0), (1, 1), (2, 1), (3, 0)]
    assert done == [1, 0, 2, 3] and frames == 11


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


FORBIDDEN = ("broadcast_object_list", "all_gather_object", "barrier", "broadcast", "all_gather", "send", "recv")


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    saved = {nm: getattr(dist, nm) for nm in FORBIDDEN + ("all_reduce",)}
    try:
        reqs = RP.poisson_requests(60, 1.5, (32, 256), (5, 40), seed=7)
        eng = RP.FakeEngine(4)
        seen = []
        orig = eng.admit

        def admit(rid, slot, p, g):
            seen.append(rid)
            orig(rid, slot, p, g)

        eng.admit = admit

        def forbid(name):
            def f(*a, **k):
                raise AssertionError(f"collective {name} while serving")
            return f

        reduces = []

        def all_reduce(*a, **k):
            reduces.append(1)
            return saved["all_reduce"](*a, **k)

        for nm in FORBIDDEN:                          # a replica never waits for another
            setattr(dist, nm, forbid(nm))
        dist.all_reduce = all_reduce
        try:
            ticks, frames, done = RP.serve(eng, reqs, 4)
        finally:
            for nm, f in saved.items():
                setattr(dist, nm, f)
        q.put((rank, ticks, frames, sorted(seen), sorted(done), sum(r.gen_frames for r in reqs), len(reduces)))
    except Exception as e:                            # report instead of hanging the parent
        q.put((rank, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_split_the_streams():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r = q.get(timeout=120)
        assert len(r) > 2, r
        res[r[0]] = r
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (_, t0, f0, s0, d0, total, n0), (_, t1, f1, s1, d1, _, n1) = res[0], res[1]
    assert n0 == n1 == 2                              # the totals' reductions after serving, nothing else
    assert t0 == t1                                   # the reduced longest tick count
    assert not set(s0) & set(s1)                      # each stream on one replica
    assert sorted(s0 + s1) == list(range(60)) == sorted(d0 + d1)
    assert f0 == f1 == total                          # the reduced frame total


