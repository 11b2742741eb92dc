"""Host request router over independent per-GPU replicas (multi-GPU = replicas only).

The model fits one B200 and streams are independent, so N GPUs run N replicas, one
process and one batch context each, with no collective on the decode path. This module
is the host side that turns arriving requests into slot admissions on those replicas,
the role the reference's single worker loop plays for one device
(src/server.cpp:1034-1275: admit into a free slot, step all active slots, retire
finished streams).

Dispatch: a request goes to a replica when it arrives, by its arrival order (request i to
replica i mod N), so every replica can compute its own queue from the arrival stream and
no message passes between replicas while they serve. Each replica then runs the
reference's admission policy locally: arrived requests wait in a FIFO and take the
lowest free slot (Router over one replica's SlotTable). A replica never waits for
another; the only collective is one reduction of the totals after serving.
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass

import numpy as np


@dataclass
class Request:
    rid: int
    prompt_len: int
    gen_frames: int
    arrival_tick: float = 0                           # tick, or seconds for wall-clock arrivals


def poisson_requests(n, rate_per_tick, prompt_range, gen_range, seed=0, whole_ticks=True):
    """n requests with exponential inter-arrival times (Poisson arrivals at
    rate_per_tick), prompt lengths and generation lengths uniform in the given
    inclusive ranges. Arrival times are whole ticks, or (whole_ticks=False) real
    values, e.g. seconds for a rate per second."""
    g = np.random.default_rng(seed)
    t = np.cumsum(g.exponential(1.0 / rate_per_tick, n))
    return [Request(i, int(g.integers(prompt_range[0], prompt_range[1] + 1)),
                    int(g.integers(gen_range[0], gen_range[1] + 1)), int(t[i]) if whole_ticks else float(t[i]))
            for i in range(n)]


class SlotTable:
    """Free slots of every replica; least-loaded admission."""

    def __init__(self, n_replicas: int, slots_per_replica: int):
        self.free = [list(range(slots_per_replica - 1, -1, -1)) for _ in range(n_replicas)]
        self.slots = slots_per_replica

    def pick(self):
        best = max(range(len(self.free)), key=lambda r: (len(self.free[r]), -r))
        return best if self.free[best] else None

    def take(self, replica: int) -> int:
        return self.free[replica].pop()

    def give_back(self, replica: int, slot: int):
        self.free[replica].append(slot)
        self.free[replica].sort(reverse=True)        # lowest slot index is reused first

    def busy(self) -> int:
        return sum(self.slots - len(f) for f in self.free)


class Router:
    """Rank-0 state: arrival queue, pending FIFO and the slot table."""

    def __init__(self, requests, n_replicas, slots_per_replica):
        self.arrivals = sorted(requests, key=lambda r: (r.arrival_tick, r.rid))
        self.next_arrival = 0
        self.pending = deque()
        self.table = SlotTable(n_replicas, slots_per_replica)
        self.owner = {}                               # rid -> (replica, slot)
        self.done = []

    def tick(self, now: int):
        """Admissions for this tick: one list of (rid, slot, prompt_len, gen_frames) per replica."""
        while self.next_arrival < len(self.arrivals) and self.arrivals[self.next_arrival].arrival_tick <= now:
            self.pending.append(self.arrivals[self.next_arrival])
            self.next_arrival += 1
        out = [[] for _ in self.table.free]
        while self.pending:
            r = self.table.pick()
            if r is None:
                break
            req = self.pending.popleft()
            slot = self.table.take(r)
            self.owner[req.rid] = (r, slot)
            out[r].append((req.rid, slot, req.prompt_len, req.gen_frames))
        return out

    def retire(self, finished_per_replica):
        for r, fin in enumerate(finished_per_replica):
            for rid in fin:
                rr, slot = self.owner.pop(rid)
                assert rr == r, "a replica reported a stream it does not own"
                self.table.give_back(r, slot)
                self.done.append(rid)

    def all_done(self) -> bool:
        return self.next_arrival == len(self.arrivals) and not self.pending and not self.owner


class FakeEngine:
    """A replica without a GPU: one frame per active stream per step (for host tests)."""

    def __init__(self, n_slots: int):
        self.left = {}
        self.slot_of = {}
        self.n_slots = n_slots
        self.frames = 0

    def admit(self, rid, slot, prompt_len, gen_frames):
        assert slot not in self.slot_of.values() and 0 <= slot < self.n_slots
        self.left[rid] = gen_frames
        self.slot_of[rid] = slot

    def step(self):
        fin = []
        for rid in list(self.left):
            self.left[rid] -= 1
            self.frames += 1
            if self.left[rid] == 0:
                fin.append(rid)
                del self.left[rid], self.slot_of[rid]
        return fin


class Z2BEngine:
    """A replica on this process's GPU: admissions are packed into the next decode step
    as prompt rows (synthetic ids: the prompt builder is not on this path), decode
    streams feed back their sampled frame, greedy sampling on the device."""

    def __init__(self, ctx, hp, n_slots: int, seed: int = 0, max_rows: int = 4096):
        self.ctx, self.hp, self.n_slots = ctx, hp, n_slots
        self.g = np.random.default_rng(seed)
        self.streams = {}                              # rid -> dict(slot, n_past, left, rows)
        self.frames = 0
        self.max_rows = max_rows                       # rows one step may carry (prompts wait beyond it)

    def admit(self, rid, slot, prompt_len, gen_frames):
        from . import runtime as R
        self.ctx.slot_reset(slot, R.Sampling(greedy=True))
        rows = self.g.integers(0, self.hp.codebook_size, (prompt_len, 10)).astype(np.int32)
        rows[:, 9] = self.g.integers(0, self.hp.text_vocab, prompt_len)
        self.streams[rid] = dict(slot=slot, n_past=0, left=gen_frames, rows=rows)

    def step(self):
        from . import runtime as R
        if not self.streams:
            return []
        rids, descs, rows, n_rows = [], [], [], 0
        for rid in sorted(self.streams, key=lambda r: self.streams[r]["slot"]):
            s = self.streams[rid]
            if n_rows > 0 and n_rows + len(s["rows"]) > self.max_rows and len(s["rows"]) > 1:
                continue                               # this prompt waits for a later step
            rids.append(rid)
            descs.append((s["slot"], s["n_past"], len(s["rows"]), R.WANT_SAMPLE))
            rows.append(s["rows"])
            n_rows += len(s["rows"])
        codes, _ = self.ctx.step(descs, np.concatenate(rows), want_logits=False)
        fin = []
        for i, rid in enumerate(rids):
            s = self.streams[rid]
            s["n_past"] += len(s["rows"])
            s["rows"] = np.r_[codes[i], self.hp.text_vocab][None].astype(np.int32)
            s["left"] -= 1
            self.frames += 1
            if s["left"] == 0:
                fin.append(rid)
                del self.streams[rid]
        return fin


def dispatch(requests, n_replicas: int, replica: int):
    """The requests replica `replica` serves: every n_replicas-th arrival, in arrival order."""
    order = sorted(requests, key=lambda r: (r.arrival_tick, r.rid))
    return [r for i, r in enumerate(order) if i % n_replicas == replica]


class Replica:
    """One replica's serving loop: per tick, admit the arrived requests into free slots
    (FIFO, lowest slot first), step the engine, retire the finished streams. clock(tick)
    gives the arrival time a tick has reached (default: the tick itself)."""

    def __init__(self, engine, requests, slots, clock=None):
        self.engine = engine
        self.router = Router(requests, 1, slots)
        self.clock = clock or (lambda t: t)
        self.ticks = 0

    def tick(self):
        for a in self.router.tick(self.clock(self.ticks))[0]:
            self.engine.admit(*a)
        self.router.retire([self.engine.step()])
        self.ticks += 1

    def done(self) -> bool:
        return self.router.all_done()


def serve_local(engine, requests, slots, clock=None, max_ticks=1_000_000):
    """Serve `requests` on one replica until all are done. Returns (ticks, frames, rids in
    retirement order)."""
    rep = Replica(engine, requests, slots, clock)
    while rep.ticks < max_ticks and not rep.done():
        rep.tick()
    return rep.ticks, engine.frames, rep.router.done


def serve(engine, requests, slots_per_replica, max_ticks=1_000_000):
    """Run the request set to completion over all ranks of the default process group
    (or this process alone without one): each rank serves its dispatched share with no
    communication, then one all-reduce sums the frames and takes the longest tick count.
    Returns (max ticks, total frames, rids this rank retired)."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1
    rank = dist.get_rank() if world > 1 else 0
    mine = dispatch(requests, world, rank)
    ticks, frames, done = serve_local(engine, mine, slots_per_replica, max_ticks=max_ticks)
    if world > 1:
        t = torch.tensor([ticks, frames], dtype=torch.int64)
        red = [t.clone(), t.clone()]
        dist.all_reduce(red[0], op=dist.ReduceOp.MAX)
        dist.all_reduce(red[1], op=dist.ReduceOp.SUM)
        ticks, frames = int(red[0][0]), int(red[1][1])
    return ticks, frames, done
