"""Text-to-PCM serving (zonos2.cpp_b200/serving.py), the server's worker loop without HTTP.

On the CPU a scripted step context stands in for the GPU backbone and the DAC oracle decodes
the windows: prompt rows come from the prompt builder, the EOS frame and countdown follow
zonos2_slot_sample (through z2b_slot_after_frame), and each request's PCM, streamed or
buffered, equals one decode of its codes up to the EOS frame. The GPU test serves real
requests through the backbone and the GPU DAC and checks the same, bit for bit, plus that a
request's frames do not depend on the other requests in its steps."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle.dac_oracle import DacOracle
from tests.conftest import load_pkg

load_pkg()                                            # spawned ranks import this module afresh


class _OracleDecoder:
    def __init__(self, o):
        self.o = o

    def decode_windows(self, ws):
        return [self.o.decode_window(*w) for w in ws]


class _ScriptedCtx:
    """Step context whose sampled frames are scripted per admission (the n-th slot_reset):
    random codes, with an end-of-audio code at codebook `eoa_cb` of frame `eoa_at[n]` (or
    never)."""

    def __init__(self, hp, eoa_at, eoa_cb=3, seed=0):
        self.hp, self.eoa_at, self.eoa_cb = hp, eoa_at, eoa_cb
        self.g = np.random.default_rng(seed)
        self.frame, self.eoa, self.adm = {}, {}, {}
        self.fed = []                      # rows fed, per admission
        self.n_admitted = 0

    def slot_reset(self, slot, sampling):
        self.frame[slot] = 0
        self.eoa[slot] = self.eoa_at.get(self.n_admitted, -1)
        self.adm[slot] = self.n_admitted
        self.fed.append([])
        self.n_admitted += 1

    def slot_prefill(self, slot, ids, spk=None, spk_pos=0, spk_emotion_delta=None):
        self.fed[self.adm[slot]].append(("prefill", np.asarray(ids).copy(), spk_pos, spk_emotion_delta is not None))
        return None

    def step(self, descs, rows, want_logits=False):
        out, r = [], 0
        for d in descs:
            slot, n_new = d[0], d[2]
            self.fed[self.adm[slot]].append(rows[r:r + n_new].copy())
            r += n_new
            f = self.g.integers(0, 1024, self.hp.n_codebooks).astype(np.int32)
            if self.frame[slot] == self.eoa[slot]:
                f[self.eoa_cb] = self.hp.eoa_id
            self.frame[slot] += 1
            out.append(f)
        return np.stack(out), None


def _hp():
    import z2b.runtime as R
    hp = R.HParams()
    hp.n_codebooks, hp.codebook_size, hp.audio_vocab, hp.eoa_id, hp.audio_pad_id, hp.text_vocab = 9, 1024, 1026, 1024, 1025, 519
    return hp


@pytest.fixture(scope="module")
def small_dac(model_dir):
    import z2b.synth as S
    return S.cached_dac("dac_small", 0, model_dir)


def test_serving_with_scripted_backbone(small_dac):
    import z2b.runtime as R
    import z2b.serving as SV
    hp = _hp()
    o = DacOracle(small_dac)
    ctx = _ScriptedCtx(hp, eoa_at={0: 70, 1: 5})
    eng = SV.TtsEngine(ctx, hp, _OracleDecoder(o), n_slots=2)
    reqs = [SV.TtsRequest(0, "First request.", max_frames=200),
            SV.TtsRequest(1, "Second, buffered.", max_frames=200, stream=False),
            SV.TtsRequest(2, "Third waits for a slot.", max_frames=90, fade_out_ms=5.0)]
    for q in reqs:
        eng.submit(q)
    done = eng.run()
    assert sorted(done) == [0, 1, 2]
    for q in reqs:
        d = done[q.rid]
        codes, eos = d["codes"], d["eos_frame"]
        nf = len(codes)
        if q.rid == 2:
            assert eos == -1 and nf == 90                         # no EOS: max_frames ends it
        else:                                                     # EOS at codebook 3 of frame k
            k = {0: 70, 1: 5}[q.rid]
            assert eos == k - 3 and nf == k + hp.n_codebooks + 1
        end = eos if 0 <= eos < nf else nf
        whole = o.decode(codes, eos=end)
        if q.fade_out_ms:
            import z2b.streaming as ST
            whole = ST.apply_fade(whole, q.fade_out_ms, 44100)
        assert d["pcm"].shape == whole.shape, q.rid
        assert np.abs(d["pcm"] - whole).max() <= 1e-6, q.rid
        if q.stream and nf >= 72:                                 # block + context + shear
            assert len(d["chunks"]) > 1                          # streamed in blocks
    # the first rows of each admission are the prompt builder's rows of its request, then
    # one row per step: the previous frame and the text pad
    for n, q in enumerate(reqs):
        assert np.array_equal(ctx.fed[n][0], R.build_prompt(hp, q.text)[0])
        assert all(len(x) == 1 and x[0, 9] == hp.text_vocab for x in ctx.fed[n][1:])


def test_speaker_request_prefills_then_steps():
    """A cloned-voice request: the speaker slot row first, all prompt rows but the last prefilled
    with the speaker at that row, the last row fed by the next step at n_past = rows - 1."""
    import z2b.runtime as R
    import z2b.serving as SV
    hp = _hp()

    class _Null:
        def decode_windows(self, ws):
            return [np.zeros((w[2] - w[1]) * 4, np.float32) for w in ws]

    ctx = _ScriptedCtx(hp, eoa_at={})

    seen = []
    orig = ctx.step

    def step(descs, rows, want_logits=False):
        seen.append(list(descs))
        return orig(descs, rows, want_logits)

    ctx.step = step
    eng = SV.TtsEngine(ctx, hp, _Null(), n_slots=1)
    eng.submit(SV.TtsRequest(0, "cloned", max_frames=5, speaker=np.ones(128, np.float32)))
    eng.run()
    full, spk_pos = R.build_prompt(hp, "cloned", add_speaker_slot=True)
    kind, pre, pos, has_delta = ctx.fed[0][0]
    assert kind == "prefill" and spk_pos == pos == 0 and np.array_equal(pre, full[:-1]) and not has_delta
    assert np.array_equal(ctx.fed[0][1], full[-1:])
    assert seen[0][0][1:3] == (len(full) - 1, 1)              # n_past, n_new of the first step


def test_emotion_cfg_takes_a_twin_slot():
    """Emotion CFG (scale != 1): the primary slot prefilled with speaker + delta, a twin slot
    with the speaker only; every step carries the twin's desc right after the primary's, the
    primary pointing at it with the scale, the twin asking for logits only, both on the same
    rows. A request that cannot be served is finished as failed."""
    import z2b.runtime as R
    import z2b.serving as SV
    hp = _hp()

    class _Null:
        def decode_windows(self, ws):
            return [np.zeros((w[2] - w[1]) * 4, np.float32) for w in ws]

    ctx = _ScriptedCtx(hp, eoa_at={})
    seen = []
    orig = ctx.step

    def step(descs, rows, want_logits=False):
        seen.append((list(descs), rows.copy()))
        return orig(descs, rows, want_logits)

    ctx.step = step
    eng = SV.TtsEngine(ctx, hp, _Null(), n_slots=3)
    spk, delta = np.ones(128, np.float32), np.ones(256, np.float32)
    eng.submit(SV.TtsRequest(0, "happy", max_frames=4, speaker=spk, emotion_delta=delta, emotion_cfg_scale=2.5))
    eng.submit(SV.TtsRequest(1, "plain", max_frames=4))
    eng.submit(SV.TtsRequest(2, "no speaker", max_frames=4, emotion_delta=delta, emotion_cfg_scale=2.0))
    done = eng.run()
    assert done[2]["error"] and done[2]["pcm"] is None
    assert len(done[0]["codes"]) == 4 and len(done[1]["codes"]) == 4
    assert ctx.fed[0][0][3] and not ctx.fed[1][0][3]      # primary with the delta, twin without
    descs, rows = seen[0]
    assert [d[0] for d in descs] == [0, 1, 2]              # primary, twin, then request 1's slot
    assert descs[0][3] == R.WANT_SAMPLE and descs[0][4] == 1 and descs[0][5] == 2.5
    assert descs[1][3] == R.WANT_LOGITS and descs[1][1] == descs[0][1] and descs[1][2] == descs[0][2] == 1
    assert np.array_equal(rows[0], rows[1])
    for descs, rows in seen[1:]:
        assert descs[1][1] == descs[0][1] and np.array_equal(rows[0], rows[1])


def test_eos_frame_follows_slot_sample():
    """EOS at codebook c of frame k sets eos_frame k - c and ends the stream n_codebooks
    frames later (the countdown of zonos2_slot_sample)."""
    import z2b.serving as SV
    hp = _hp()

    class _Null:
        def decode_windows(self, ws):
            return [np.zeros((w[2] - w[1]) * 4, np.float32) for w in ws]

    for k, c in ((40, 3), (2, 5)):
        ctx = _ScriptedCtx(hp, eoa_at={0: k}, eoa_cb=c)
        eng = SV.TtsEngine(ctx, hp, _Null(), n_slots=1)
        eng.submit(SV.TtsRequest(0, "x", max_frames=500))
        d = eng.run()[0]
        assert d["eos_frame"] == max(0, k - c)
        assert len(d["codes"]) == k + hp.n_codebooks + 1


class _NullDecoder:
    def decode_windows(self, ws):
        return [np.zeros((w[2] - w[1]) * 4, np.float32) for w in ws]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


FORBIDDEN = ("broadcast_object_list", "all_gather_object", "barrier", "broadcast", "all_gather", "send", "recv")


def _tts_worker(rank, world, port, q):
    import z2b.serving as SV
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    saved = {nm: getattr(dist, nm) for nm in FORBIDDEN}
    try:
        hp = _hp()
        ctx = _ScriptedCtx(hp, eoa_at={}, seed=rank)
        eng = SV.TtsEngine(ctx, hp, _NullDecoder(), n_slots=3)

        def forbid(name):
            def f(*a, **k):
                raise AssertionError(f"collective {name} while serving")
            return f

        for nm in FORBIDDEN:                          # a replica never waits for another
            setattr(dist, nm, forbid(nm))
        reqs = [SV.TtsRequest(i, f"request {i}", max_frames=5 + i) for i in range(11)]
        try:
            r = SV.serve_tts(eng, reqs)
        finally:
            for nm, f in saved.items():
                setattr(dist, nm, f)
        q.put((rank, r["steps"], r["frames"], r["pcm_samples"], sorted(r["done"]),
               sum(len(d["codes"]) for d in r["done"].values())))
    except Exception as e:                            # report instead of hanging the parent
        q.put((rank, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_split_the_requests():
    """Two replicas: each request served once, on rank rid mod 2, with no collective while
    serving; the reduced frame total is every request's frame count."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tts_worker, args=(r, 2, port, q)) for r in range(2)]
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
    (_, s0, f0, p0, d0, n0), (_, s1, f1, p1, d1, n1) = res[0], res[1]
    assert d0 == list(range(0, 11, 2)) and d1 == list(range(1, 11, 2))
    assert s0 == s1 and f0 == f1 == n0 + n1 == sum(5 + i for i in range(11))
    assert p0 == p1 == f0 * 4                             # the null decoder's 4 samples per frame


@pytest.mark.gpu
def test_gpu_serving_end_to_end(model_dir, small_dac):
    import z2b.dac as D
    import z2b.runtime as R
    import z2b.serving as SV
    import z2b.synth as S
    m = R.Model(S.cached("tiny", directory=model_dir))
    dac = D.Dac(small_dac)
    texts = ["Hello there.", "A second, longer request for the batch.", "Third."]

    def serve(idx, n_slots):
        ctx = R.BatchCtx(m, n_slots, 512)
        eng = SV.TtsEngine(ctx, m.hp, dac, n_slots=n_slots)
        for i in idx:
            eng.submit(SV.TtsRequest(i, texts[i], max_frames=120, stream=i != 1))
        done = eng.run()
        ctx.close()
        return done

    together = serve([0, 1, 2], 2)                     # request 2 waits for a free slot
    # a cloned voice: the speaker changes the frames, and batching does not
    spk = np.random.default_rng(4).standard_normal(m.hp.spk_dim).astype(np.float32)

    def serve_spk(extra):
        ctx = R.BatchCtx(m, 2, 512)
        eng = SV.TtsEngine(ctx, m.hp, dac, n_slots=2)
        eng.submit(SV.TtsRequest(9, texts[0], max_frames=60, speaker=spk))
        if extra:
            eng.submit(SV.TtsRequest(8, texts[1], max_frames=60))
        done = eng.run()
        ctx.close()
        return done[9]

    a, b = serve_spk(False), serve_spk(True)
    assert np.array_equal(a["codes"], b["codes"])
    assert not np.array_equal(a["codes"], together[0]["codes"][:60])

    # emotion CFG against a twin: the scale changes the frames; batching does not
    delta = np.random.default_rng(5).standard_normal(m.hp.n_embd).astype(np.float32)

    def serve_cfg(scale, extra):
        ctx = R.BatchCtx(m, 3, 512)
        eng = SV.TtsEngine(ctx, m.hp, dac, n_slots=3)
        eng.submit(SV.TtsRequest(7, texts[0], max_frames=60, speaker=spk, emotion_delta=delta,
                                 emotion_cfg_scale=scale))
        if extra:
            eng.submit(SV.TtsRequest(6, texts[2], max_frames=60))
        done = eng.run()
        ctx.close()
        return done[7]["codes"]

    c1, c3, c3b = serve_cfg(1.0, False), serve_cfg(3.0, False), serve_cfg(3.0, True)
    assert np.array_equal(c3, c3b)
    assert not np.array_equal(c1, c3)
    for i in range(3):
        d = together[i]
        nf = len(d["codes"])
        end = d["eos_frame"] if 0 <= d["eos_frame"] < nf else nf
        assert np.array_equal(d["pcm"], dac.decode(d["codes"], eos=end)), i
        alone = serve([i], 1)[i]
        assert np.array_equal(alone["codes"], d["codes"]), i   # batch-invariant frames
    dac.close()
    m.close()
