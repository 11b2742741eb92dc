"""CPU oracle self-checks: KV decode == recompute, ggml-emu close to exact, batch
independence (F.1/F.2 on the oracle), and the sampler's RNG consumption."""
from __future__ import annotations

import random

import numpy as np
import pytest

from oracle import oracle as O
from tests.util import cos, prompt


@pytest.fixture(scope="module")
def om(tiny_path):
    return O.Model(tiny_path)


def test_decode_matches_recompute(om):
    """Prefill + KV decode vs a full prefill of the same rows (f16 cache vs f32 prefill)."""
    c = O.Ctx(om, 1, 256)
    p = prompt(20, 1)
    lg = c.prefill(0, p)
    row = np.concatenate([lg.argmax(-1), [519]]).astype(np.int32)
    a = c.step([0], [20], row[None])[0]
    b = O.Ctx(om, 1, 256).prefill(0, np.concatenate([p, row[None]]))
    assert cos(a, b) > 0.99999


def test_batch_independence(om):
    c1, c2 = O.Ctx(om, 3, 128), O.Ctx(om, 1, 128)
    p0, p1 = prompt(9, 2), prompt(5, 3)
    for s, p in ((0, p0), (1, p1), (2, p0)):
        c1.prefill(s, p)
    c2.prefill(0, p1)
    ids = np.stack([np.r_[np.arange(9), 7]] * 3).astype(np.int32)
    a = c1.step([0, 1, 2], [9, 5, 9], ids)
    b = c2.step([0], [5], ids[:1])
    assert np.array_equal(a[1], b[0])          # F.1: a slot's logits do not depend on the batch
    assert np.array_equal(a[0], a[2])          # F.2: identical prompts in two slots


def test_ggml_emu_close_to_exact(tiny_path):
    p = prompt(12, 4)
    a = O.Ctx(O.Model(tiny_path, O.EXACT), 1, 64).prefill(0, p)
    b = O.Ctx(O.Model(tiny_path, O.GGML_EMU), 1, 64).prefill(0, p)
    assert cos(a, b) > 0.9999


def test_sampler_greedy_is_first_argmax():
    s = O.Sampler(2, greedy=True)
    lg = np.zeros((2, 8), np.float32)
    lg[0, [3, 5]] = 1.0
    lg[1, 7] = 2.0
    assert s.sample(lg).tolist() == [3, 7]


def test_sampler_reproducible_and_seeded():
    g = np.random.default_rng(0)
    lg = g.standard_normal((9, 1026)).astype(np.float32)
    a = [O.Sampler(9, seed=7).sample(lg).tolist() for _ in range(2)]
    assert a[0] == a[1]
    s1, s2 = O.Sampler(9, seed=7), O.Sampler(9, seed=8)
    seq1 = [s1.sample(lg).tolist() for _ in range(5)]
    seq2 = [s2.sample(lg).tolist() for _ in range(5)]
    assert seq1 != seq2


def test_sampler_consumes_one_draw_per_codebook():
    """Non-greedy sampling draws exactly one uniform per (frame, codebook), in codebook
    order, from std::mt19937 (src/zonos2-sampler.cpp:73-74): with top_k = 1 every draw
    is consumed but cannot change the pick, so a second sampler that starts one frame
    later on the same seed matches once it skips 9 draws."""
    lg = np.random.default_rng(1).standard_normal((9, 64)).astype(np.float32)
    s = O.Sampler(9, top_k=1, min_p=0.0, rep_penalty=1.0, seed=3)
    assert s.sample(lg).tolist() == lg.argmax(-1).tolist()


def _spk_inputs(om, seed):
    g = np.random.default_rng(seed)
    sd = int(om.t["spk_lda.weight"].shape[0])
    return g.standard_normal(sd).astype(np.float32), (0.1 * g.standard_normal(om.hp.n_embd)).astype(np.float32)


def test_speaker_row_matches_numpy(om):
    """spk_proj(spk_lda(spk)) + delta (src/zonos2-graph.cpp:262-275) against float64 numpy
    over gguf-py's dequantised tensors."""
    from gguf.quants import dequantize

    def deq(name):
        t = om.t[name]
        return dequantize(t.data, t.tensor_type).astype(np.float64).reshape(
            [int(x) for x in reversed(t.shape) if int(x) > 1] or [-1])

    spk, delta = _spk_inputs(om, 11)
    sl = deq("spk_lda.weight") @ spk.astype(np.float64) + deq("spk_lda.bias")
    sp = deq("spk_proj.weight") @ sl.astype(np.float32).astype(np.float64) + deq("spk_proj.bias")
    got = om.spk_row(spk)
    assert np.allclose(got, sp, rtol=1e-5, atol=1e-6)
    got_d = om.spk_row(spk, delta)
    assert np.allclose(got_d, (got.astype(np.float64) + delta), rtol=1e-6, atol=1e-7)


def test_speaker_replaces_the_row(om):
    """The speaker row replaces (not adds to) the embedding at spk_pos: the ids of that
    row no longer matter, and the logits differ from the prompt without a speaker."""
    spk, delta = _spk_inputs(om, 12)
    p = prompt(10, 5)
    q = p.copy()
    q[2] = (q[2] + 7) % 500
    a = O.Ctx(om, 1, 64).prefill(0, p, spk=spk, spk_pos=2)
    b = O.Ctx(om, 1, 64).prefill(0, q, spk=spk, spk_pos=2)
    assert np.array_equal(a, b)
    plain = O.Ctx(om, 1, 64).prefill(0, p)
    assert not np.array_equal(a, plain)
    e = O.Ctx(om, 1, 64).prefill(0, p, spk=spk, spk_pos=2, spk_emotion_delta=delta)
    assert not np.array_equal(a, e)


def test_teacher_forced_logits_last_row_is_the_prefill(om):
    """zonos2_logits restated: row t of the all-rows forward equals a prefill of rows 0..t."""
    p = prompt(9, 6)
    spk, _ = _spk_inputs(om, 13)
    all_rows = om.logits(p, spk=spk, spk_pos=0)
    assert all_rows.shape == (9, om.hp.n_codebooks, om.hp.audio_vocab)
    assert np.array_equal(all_rows[-1], O.Ctx(om, 1, 64).prefill(0, p, spk=spk, spk_pos=0))
    assert np.array_equal(all_rows[4], O.Ctx(om, 1, 64).prefill(0, p[:5], spk=spk, spk_pos=0))
