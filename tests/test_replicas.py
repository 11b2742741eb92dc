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


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        reqs = RP.poisson_requests(60, 1.5, (32, 256), (5, 40), seed=7)
        eng = RP.FakeEngine(4)
        seen = []
        orig = eng.admit

        def admit(rid, slot, p, g):
            seen.append(rid)
            orig(rid, slot, p, g)

        eng.admit = admit
        ticks, frames, done = RP.serve(eng, reqs, 4)
        q.put((rank, ticks, frames, sorted(seen), done, sum(r.gen_frames for r in reqs)))
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
        res[r[0]] = r
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (_, t0, f0, s0, done, total), (_, t1, f1, s1, _, _) = res[0], res[1]
    assert t0 == t1                                   # ranks took the same ticks
    assert not set(s0) & set(s1)                      # each stream on one replica
    assert sorted(s0 + s1) == list(range(60)) == sorted(done)
    assert f0 + f1 == total and f0 > 0 and f1 > 0     # both replicas did work


@pytest.mark.gpu
def test_router_drives_a_gpu_replica(tiny_path):
    """The router's admissions and retirements through a real replica (one GPU, tiny
    model): prompts packed into decode steps, every request generates its frames."""
    import z2b.runtime as R
    m = R.Model(tiny_path)
    ctx = R.BatchCtx(m, 3, 512)
    try:
        reqs = RP.poisson_requests(8, 0.7, (5, 40), (2, 12), seed=3)
        eng = RP.Z2BEngine(ctx, m.hp, 3)
        ticks, frames, done = RP.serve(eng, reqs, 3)
        assert sorted(done) == list(range(8))
        assert frames == sum(r.gen_frames for r in reqs)
    finally:
        ctx.close()
        m.close()
