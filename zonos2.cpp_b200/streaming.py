"""Streaming PCM for many streams through the batched GPU DAC decoder.

Host side of the server's audio path (src/server.cpp:913-1008): as a stream's codec frames
arrive, each complete block of frames becomes a DAC window with conv context on both sides
(stream_submit_ready), and at the stream's end the rest becomes a tail window with no right
context, faded out (submit_finalize, apply_fade). The reference hands every window to a DAC
lane thread that decodes it alone; here ``DacBatcher`` collects the pending windows of all
streams and decodes them in one ``Dac.decode_windows`` call, which decodes each window bit
for bit as it would alone.

With the context at least the decoder's receptive field (the reference's default 24 frames;
16 suffice), a stream's chunks joined end to end equal one decode of the whole stream up to
its end frame, sample for sample (before the fade).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np


@dataclass
class StreamCfg:
    n_codebooks: int = 9
    block: int = 40           # frames per streamed PCM block (src/server.cpp:105)
    ctx: int = 24             # conv-context frames each side (src/server.cpp:106)
    fade_out_ms: float = 0.0  # fade of the last chunk (the request's fade_out_ms)
    sample_rate: int = 44100


@dataclass
class PcmStream:
    """One request's frames and the frames already emitted as PCM."""
    cfg: StreamCfg
    codes: list = field(default_factory=list)   # frames, each n_codebooks ids
    emitted: int = 0
    finished: bool = False

    def push(self, frames) -> None:
        for f in np.asarray(frames, np.int32).reshape(-1, self.cfg.n_codebooks):
            self.codes.append(f)

    def snapshot(self, n):
        """The first n frames as an [n][n_codebooks] array (a copy: the stream keeps growing)."""
        return np.asarray(self.codes[:n], np.int32).reshape(n, self.cfg.n_codebooks)

    def ready_windows(self) -> list[tuple]:
        """Windows that can be decoded now (stream_submit_ready): while a full block plus the right
        context plus the shear lookahead (n_codebooks - 1 frames) is generated, output frames
        [emitted, H - ctx - shear) with ctx frames of context each side."""
        c = self.cfg
        H, shear = len(self.codes), c.n_codebooks - 1
        out = []
        while H - self.emitted >= c.block + c.ctx + shear:
            f_hi = H - c.ctx - shear
            out.append((self.snapshot(H), self.emitted, f_hi, c.ctx, c.ctx))
            self.emitted = f_hi
        return out

    def final_window(self, eos_frame: int = -1):
        """The tail (submit_finalize): output frames [emitted, end) with no right context, end the
        EOS frame when it lies inside the generated frames, else their count. None if empty."""
        self.finished = True
        nf = len(self.codes)
        end = eos_frame if 0 <= eos_frame < nf else nf
        if end <= self.emitted:
            return None
        w = (self.snapshot(nf), self.emitted, end, self.cfg.ctx, 0)
        self.emitted = end
        return w


def apply_fade(pcm: np.ndarray, fade_ms: float, sample_rate: int) -> np.ndarray:
    """Raised-cosine fade over the last fade_ms of pcm (src/server.cpp:475-483), in f32."""
    if fade_ms <= 0 or pcm.size == 0:
        return pcm
    n = min(pcm.size, int(fade_ms * 0.001 * sample_rate))
    if n <= 0:
        return pcm
    i = np.arange(n, dtype=np.float32)
    t = i / np.float32(n)
    g = np.float32(0.5) * (np.float32(1.0) + np.cos(np.float32(math.pi) * t).astype(np.float32))
    out = pcm.copy()
    out[pcm.size - n:] *= g
    return out


class DacBatcher:
    """Pending windows of many streams, decoded together in one batched call per flush.

    ``decoder`` is anything with ``decode_windows(windows) -> list of arrays`` (a ``z2b.dac.Dac``)."""

    def __init__(self, decoder):
        self.decoder = decoder
        self.pending: list[tuple] = []           # (stream id, window, fade_ms, sample_rate)

    def submit(self, sid, window, fade_ms: float = 0.0, sample_rate: int = 44100) -> None:
        if window is not None:
            self.pending.append((sid, window, fade_ms, sample_rate))

    def flush(self) -> list[tuple]:
        """Decode every pending window in one call; returns [(stream id, pcm chunk)] in
        submission order (so each stream's chunks stay ordered)."""
        if not self.pending:
            return []
        pcm = self.decoder.decode_windows([p[1] for p in self.pending])
        out = [(sid, apply_fade(x, fade, sr)) for (sid, _, fade, sr), x in zip(self.pending, pcm)]
        self.pending = []
        return out
