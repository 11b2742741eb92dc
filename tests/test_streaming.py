"""Streaming PCM (zonos2.cpp_b200/streaming.py): the server's block / context / shear cadence
(src/server.cpp:976-1008), the tail window and fade, and the property that a stream's chunks
joined end to end equal one decode of the stream up to its end frame. On the CPU the oracle
decodes the windows; the GPU test runs the same streams through the batched GPU decoder."""
from __future__ import annotations

import numpy as np
import pytest

from oracle.dac_oracle import DacOracle


class _OracleDecoder:
    def __init__(self, o):
        self.o = o

    def decode_windows(self, ws):
        return [self.o.decode_window(*w) for w in ws]


def _reference_cadence(H_steps, block, ctx, shear):
    """The reference's loop (stream_submit_ready) over growing H: (f_lo, f_hi) per window."""
    emitted, out = 0, []
    for H in H_steps:
        while H - emitted >= block + ctx + shear:
            f_hi = H - ctx - shear
            out.append((emitted, f_hi))
            emitted = f_hi
    return out, emitted


def _run(decoder, streams, eos, cfg, seed=0):
    """Feed each stream's frames in random increments, flushing the batcher after every round;
    returns the joined PCM per stream and the (f_lo, f_hi, Rc) of every window."""
    import z2b.streaming as ST
    g = np.random.default_rng(seed)
    ps = [ST.PcmStream(cfg) for _ in streams]
    b = ST.DacBatcher(decoder)
    pos = [0] * len(streams)
    chunks = {i: [] for i in range(len(streams))}
    wins = {i: [] for i in range(len(streams))}
    while any(p < len(s) for p, s in zip(pos, streams)):
        for i, s in enumerate(streams):
            if pos[i] < len(s):
                n = int(g.integers(1, 12))
                ps[i].push(s[pos[i]:pos[i] + n])
                pos[i] += n
                for w in ps[i].ready_windows():
                    wins[i].append((w[1], w[2], w[4]))
                    b.submit(i, w)
        for sid, pcm in b.flush():
            chunks[sid].append(pcm)
    for i in range(len(streams)):
        w = ps[i].final_window(eos[i])
        if w is not None:
            wins[i].append((w[1], w[2], w[4]))
        b.submit(i, w, cfg.fade_out_ms, cfg.sample_rate)
    for sid, pcm in b.flush():
        chunks[sid].append(pcm)
    return [np.concatenate(chunks[i]) if chunks[i] else np.zeros(0, np.float32) for i in range(len(streams))], wins


@pytest.fixture(scope="module")
def small_dac(model_dir):
    import z2b.synth as S
    return S.cached_dac("dac_small", 0, model_dir)


def _streams(lengths, seed):
    g = np.random.default_rng(seed)
    return [g.integers(0, 1024, (n, 9)).astype(np.int32) for n in lengths]


def test_cadence_matches_reference():
    import z2b.streaming as ST
    cfg = ST.StreamCfg()
    g = np.random.default_rng(3)
    frames = g.integers(0, 1024, (300, 9)).astype(np.int32)
    p = ST.PcmStream(cfg)
    H_steps, got, H = [], [], 0
    while H < len(frames):
        n = int(g.integers(1, 30))
        p.push(frames[H:H + n])
        H = min(H + n, len(frames))
        H_steps.append(H)
        got += [(w[1], w[2]) for w in p.ready_windows()]
    ref, emitted = _reference_cadence(H_steps, 40, 24, 8)
    assert got == ref and p.emitted == emitted
    assert emitted > 250
    q = ST.PcmStream(cfg, codes=list(p.codes), emitted=p.emitted)
    assert q.final_window(250) is None                   # an EOS before the emitted frames: no tail
    tail = p.final_window(-1)
    assert (tail[1], tail[2], tail[3], tail[4]) == (emitted, 300, 24, 0)
    assert p.final_window(-1) is None                     # nothing left


def test_joined_chunks_equal_whole_decode(small_dac):
    import z2b.streaming as ST
    o = DacOracle(small_dac)
    cfg = ST.StreamCfg()
    streams = _streams((150, 97, 64), 5)
    eos = [120, -1, 70]                                  # an EOS inside, none, one past the frames
    pcm, wins = _run(_OracleDecoder(o), streams, eos, cfg)
    for i, s in enumerate(streams):
        end = eos[i] if 0 <= eos[i] < len(s) else len(s)
        whole = o.decode(s, eos=end)
        assert pcm[i].shape == whole.shape, i
        assert np.abs(pcm[i] - whole).max() <= 1e-6, (i, np.abs(pcm[i] - whole).max())
        assert any(rc == 24 for _, _, rc in wins[i][:-1]) or len(wins[i]) == 1
        assert wins[i][-1][2] == 0                        # the tail has no right context


def test_fade():
    import z2b.streaming as ST
    a = np.ones(1000, np.float32)
    f = ST.apply_fade(a, 10.0, 44100)                    # 441 samples
    assert np.array_equal(f[:559], a[:559]) and f[559] == 1.0 and 0 < f[-1] < 1e-4
    assert np.all(np.diff(f[559:]) <= 0)
    assert ST.apply_fade(a, 0.0, 44100) is a


@pytest.mark.gpu
def test_gpu_joined_chunks_equal_whole_decode(small_dac):
    """The same streams through the batched GPU decoder: the joined chunks equal the GPU's own
    whole-stream decode bit for bit, and the oracle's within the DAC parity bar."""
    import z2b.dac as D
    import z2b.streaming as ST
    from tests.util import cos
    d = D.Dac(small_dac)
    o = DacOracle(small_dac)
    cfg = ST.StreamCfg()
    streams = _streams((150, 97, 64), 5)
    eos = [120, -1, 70]
    pcm, _ = _run(d, streams, eos, cfg)
    for i, s in enumerate(streams):
        end = eos[i] if 0 <= eos[i] < len(s) else len(s)
        whole = d.decode(s, eos=end)
        assert np.array_equal(pcm[i], whole), i
        assert cos(pcm[i], o.decode(s, eos=end)) >= 0.9999
    d.close()
