"""Text-to-PCM serving on one GPU: the server's request path without its HTTP layer.

Mirrors the worker loop of src/server.cpp:1034-1275 on this library's calls:
  - admission: the request's text becomes prompt rows (z2b_build_prompt) in a free slot, and
    its rows ride in the next batched step with the other streams' decode rows. A cloned
    voice (a speaker embedding) gets the speaker slot row; all rows but the last are
    prefilled with the speaker projected into that row (z2b_slot_prefill_spk, as the
    reference's admission prefill), and the last row rides in the next step, whose device
    sampler draws the first frame. An emotion request with a CFG scale other than 1 also
    takes a twin slot, prefilled with the speaker but without the emotion delta; the twin
    steps on the same rows and its logits guide the stream's sampling,
    u + scale * (c - u) (src/server.cpp:1064-1099, 1125-1142), on the device;
  - each step: one z2b_step over every active stream (device sampling), then per stream
    zonos2_slot_sample's bookkeeping (z2b_slot_after_frame: EOS frame, countdown,
    max_frames, next input row), the frame appended to the stream's codes;
  - audio: streaming requests emit DAC windows on the server's cadence as frames arrive,
    and every request's tail (or whole buffered decode) goes out when its slot finishes;
    all pending windows of all requests are decoded in one batched GPU DAC call per step
    (streaming.DacBatcher), not one window per DAC lane thread.
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field

import numpy as np

from .streaming import DacBatcher, PcmStream, StreamCfg


@dataclass
class TtsRequest:
    rid: int
    text: str
    max_frames: int = 1500
    stream: bool = True                 # False: one buffered decode at the end
    fade_out_ms: float = 0.0
    sampling: object = None             # runtime.Sampling; None: greedy
    speaker: object = None              # [spk_dim] f32 speaker embedding (cloned voice), or None
    emotion_delta: object = None        # [n_embd] f32 added to the speaker row, or None
    emotion_cfg_scale: float = 1.0      # with emotion_delta: CFG against an unconditional twin

    def use_cfg(self) -> bool:
        return self.emotion_delta is not None and self.emotion_cfg_scale != 1.0


@dataclass
class _Job:
    req: TtsRequest
    slot: object                        # runtime.Slot
    rows: np.ndarray                    # rows fed in the next step
    pcm: PcmStream
    chunks: list = field(default_factory=list)
    twin: object = None                 # runtime.Slot of the unconditional twin (emotion CFG)


class TtsEngine:
    """Requests in, PCM chunks out. ``ctx`` is a runtime.BatchCtx (or anything with its
    slot_reset / step calls), ``dac`` a dac.Dac (or anything with decode_windows)."""

    def __init__(self, ctx, hp, dac, n_slots: int, cfg: StreamCfg | None = None):
        self.ctx, self.hp, self.n_slots = ctx, hp, n_slots
        self.cfg = cfg or StreamCfg(n_codebooks=hp.n_codebooks)
        self.batcher = DacBatcher(dac)
        self.jobs: dict[int, _Job] = {}
        self.queue: deque[TtsRequest] = deque()
        self.done: dict[int, dict] = {}     # rid -> codes, eos_frame, pcm (or error)
        self.frames = 0

    def submit(self, req: TtsRequest) -> None:
        self.queue.append(req)

    def _admit(self) -> None:
        from . import runtime as R
        used = {j.slot.index for j in self.jobs.values()} | {j.twin.index for j in self.jobs.values() if j.twin}
        free = [s for s in range(self.n_slots) if s not in used]
        while self.queue:
            req = self.queue[0]
            need = 2 if req.use_cfg() else 1
            if req.emotion_delta is not None and req.speaker is None or need > self.n_slots:
                self.queue.popleft()              # cannot be served: finished as failed
                why = "an emotion delta needs a speaker" if req.speaker is None else "CFG needs two slots"
                self.done[req.rid] = dict(error=why, codes=None, eos_frame=-1, chunks=[], pcm=None)
                continue
            if len(free) < need:
                break                             # first come, first served: the head waits
            self.queue.popleft()
            rows, spk_pos = R.build_prompt(self.hp, req.text, add_speaker_slot=req.speaker is not None)
            slots = [free.pop(0) for _ in range(need)]
            s = R.Slot(index=slots[0])
            self.ctx.slot_reset(slots[0], req.sampling or R.Sampling(greedy=True))
            twin = None
            if req.speaker is not None:
                self.ctx.slot_prefill(slots[0], rows[:-1], spk=req.speaker, spk_pos=spk_pos,
                                      spk_emotion_delta=req.emotion_delta)
                s.n_past = len(rows) - 1
                if need == 2:
                    twin = R.Slot(index=slots[1], n_past=len(rows) - 1)
                    self.ctx.slot_reset(slots[1], R.Sampling(greedy=True))
                    self.ctx.slot_prefill(slots[1], rows[:-1], spk=req.speaker, spk_pos=spk_pos)
                rows = rows[-1:]
            self.jobs[req.rid] = _Job(req, s, rows, PcmStream(self.cfg), twin=twin)

    def step(self) -> list[int]:
        """Admit queued requests into free slots, run one batched step, hand out audio.
        Returns the requests that finished in this step."""
        from . import runtime as R
        self._admit()
        if not self.jobs:
            return []
        order = sorted(self.jobs.values(), key=lambda j: j.slot.index)
        descs, rows, at = [], [], []
        for j in order:
            at.append(len(descs))
            if j.twin is None:
                descs.append((j.slot.index, j.slot.n_past, len(j.rows), R.WANT_SAMPLE, -1, 1.0))
                rows.append(j.rows)
            else:                                       # the twin's desc follows, logits only
                descs.append((j.slot.index, j.slot.n_past, len(j.rows), R.WANT_SAMPLE, len(descs) + 1,
                              j.req.emotion_cfg_scale))
                descs.append((j.twin.index, j.twin.n_past, len(j.rows), R.WANT_LOGITS, -1, 1.0))
                rows += [j.rows, j.rows]
        codes, _ = self.ctx.step(descs, np.concatenate(rows), want_logits=False)
        finished = []
        for i, j in zip(at, order):
            s = j.slot
            s.n_past += len(j.rows)
            if j.twin is not None:
                j.twin.n_past += len(j.rows)
            frame = np.asarray(codes[i][: self.hp.n_codebooks], np.int32)
            R.slot_after_sample(self.hp, s, frame, j.req.max_frames)
            j.pcm.push(frame)
            self.frames += 1
            j.rows = np.asarray(s.next_ids, np.int32)[None]
            if j.req.stream:
                for w in j.pcm.ready_windows():
                    self.batcher.submit(j.req.rid, w)
            if s.done:
                if j.req.stream:
                    w = j.pcm.final_window(s.eos_frame)
                else:                                   # buffered: one decode of [0, end)
                    nf = len(j.pcm.codes)
                    end = s.eos_frame if 0 <= s.eos_frame < nf else nf
                    w = (j.pcm.snapshot(nf), 0, end, 0, 0) if end > 0 else None
                self.batcher.submit(j.req.rid, w, j.req.fade_out_ms, self.cfg.sample_rate)
                finished.append(j.req.rid)
        for rid, pcm in self.batcher.flush():
            self.jobs[rid].chunks.append(pcm)
        for rid in finished:
            j = self.jobs.pop(rid)
            self.done[rid] = dict(codes=np.asarray(j.pcm.codes, np.int32).reshape(-1, self.hp.n_codebooks),
                                  eos_frame=j.slot.eos_frame, chunks=j.chunks,
                                  pcm=np.concatenate(j.chunks) if j.chunks else np.zeros(0, np.float32))
        return finished

    def run(self, max_steps: int = 1_000_000) -> dict[int, dict]:
        """Step until every submitted request has finished."""
        n = 0
        while (self.queue or self.jobs) and n < max_steps:
            self.step()
            n += 1
        return self.done


def serve_tts(engine: TtsEngine, requests: list[TtsRequest], max_steps: int = 1_000_000) -> dict:
    """Serve `requests` over every rank of the default process group (or this process alone
    without one), one engine per GPU: request i (in rid order) goes to rank i mod N, each rank
    serves its share with no communication, then one all-reduce takes the longest step count
    and another sums the frames and PCM samples. Returns those totals and this rank's results."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1
    rank = dist.get_rank() if world > 1 else 0
    for i, r in enumerate(sorted(requests, key=lambda r: r.rid)):
        if i % world == rank:
            engine.submit(r)
    steps = 0
    while (engine.queue or engine.jobs) and steps < max_steps:
        engine.step()
        steps += 1
    pcm = sum(d["pcm"].size for d in engine.done.values() if d.get("pcm") is not None)
    out = {"steps": steps, "frames": engine.frames, "pcm_samples": pcm, "done": engine.done}
    if world > 1:
        mx = torch.tensor([steps], dtype=torch.int64)
        tot = torch.tensor([engine.frames, pcm], dtype=torch.int64)
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
        out.update(steps=int(mx[0]), frames=int(tot[0]), pcm_samples=int(tot[1]))
    return out
