"""Speaker injection in prefill (zonos2_batch_slot_prefill's spk / spk_pos /
spk_emotion_delta, src/zonos2-graph.cpp:262-292, 703-760) on the GPU against the oracle:
the projected speaker row replaces the embedding of one prompt row before emb_norm, and
the KV it leaves behind serves the following decode steps."""
from __future__ import annotations

import numpy as np
import pytest

import z2b.runtime as R
from oracle import oracle as O
from tests.util import cos, max_abs_rel, prompt

pytestmark = pytest.mark.gpu
COS_MIN, MAR_MAX = 0.9999, 1e-2


@pytest.fixture(scope="module")
def tiny(tiny_path):
    m = R.Model(tiny_path)
    yield m
    m.close()


def _inputs(hp, seed):
    g = np.random.default_rng(seed)
    return (g.standard_normal(hp.spk_dim).astype(np.float32),
            (0.1 * g.standard_normal(hp.n_embd)).astype(np.float32))


def test_speaker_prefill_and_decode_parity(tiny, tiny_path):
    hp = tiny.hp
    spk, delta = _inputs(hp, 31)
    pa, pb = prompt(40, 21), prompt(7, 22)
    ctx = R.BatchCtx(tiny, 2, 128)
    for s in (0, 1):
        ctx.slot_reset(s, R.Sampling(greedy=True))
    ga = ctx.slot_prefill(0, pa, spk=spk, spk_pos=0)
    gb = ctx.slot_prefill(1, pb, spk=spk, spk_pos=5, spk_emotion_delta=delta)
    oc = O.Ctx(O.Model(tiny_path, O.EXACT), 2, 128)
    oa = oc.prefill(0, pa, spk=spk, spk_pos=0)
    ob = oc.prefill(1, pb, spk=spk, spk_pos=5, spk_emotion_delta=delta)
    for g, o in ((ga, oa), (gb, ob)):
        assert cos(g, o) >= COS_MIN, cos(g, o)
        assert max_abs_rel(g, o) <= MAR_MAX
    # three decode steps over the speaker-conditioned caches, teacher-forced
    past = [40, 7]
    rows = np.stack([np.r_[ga.argmax(-1), hp.text_vocab], np.r_[gb.argmax(-1), hp.text_vocab]]).astype(np.int32)
    for _ in range(3):
        _, lg = ctx.step([(0, past[0], 1, R.WANT_LOGITS), (1, past[1], 1, R.WANT_LOGITS)], rows)
        ref = oc.step([0, 1], past, rows)
        for i in range(2):
            assert cos(lg[i], ref[i]) >= COS_MIN, (i, cos(lg[i], ref[i]))
            assert max_abs_rel(lg[i], ref[i]) <= MAR_MAX
        rows = np.stack([np.r_[lg[i].argmax(-1), hp.text_vocab] for i in range(2)]).astype(np.int32)
        past = [p + 1 for p in past]
    ctx.close()


def test_speaker_row_replaces_the_embedding(tiny, tiny_path):
    """The ids of row spk_pos no longer matter (bit for bit); the speaker changes the
    logits; a one-row speaker prefill is not captured into the decode graphs."""
    hp = tiny.hp
    spk, _ = _inputs(hp, 32)
    p = prompt(12, 23)
    q = p.copy()
    q[3] = (q[3] + 5) % 500
    ctx = R.BatchCtx(tiny, 3, 64)
    for s in range(3):
        ctx.slot_reset(s, R.Sampling(greedy=True))
    a = ctx.slot_prefill(0, p, spk=spk, spk_pos=3)
    b = ctx.slot_prefill(1, q, spk=spk, spk_pos=3)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    assert not np.array_equal(a, ctx.slot_prefill(2, p))
    # one-row prefill (T equals the descriptor count, the decode-graph shape) with a speaker,
    # then a plain one-row decode step, which must not inherit the speaker row
    one = R.BatchCtx(tiny, 1, 64)
    one.slot_reset(0, R.Sampling(greedy=True))
    s0 = one.slot_prefill(0, p[:1], spk=spk, spk_pos=0)
    row = np.r_[s0.argmax(-1), hp.text_vocab].astype(np.int32)[None]
    _, d1 = one.step([(0, 1, 1, R.WANT_LOGITS)], row)
    oc = O.Ctx(O.Model(tiny_path, O.EXACT), 1, 64)
    os0 = oc.prefill(0, p[:1], spk=spk, spk_pos=0)
    assert cos(s0, os0) >= COS_MIN
    od1 = oc.step([0], [1], row)[0]
    assert cos(d1[0], od1) >= COS_MIN, cos(d1[0], od1)
    assert max_abs_rel(d1[0], od1) <= MAR_MAX
    for c in (ctx, one):
        c.close()


def test_speaker_pos_outside_prompt_is_an_error(tiny):
    hp = tiny.hp
    spk, _ = _inputs(hp, 33)
    ctx = R.BatchCtx(tiny, 1, 64)
    ctx.slot_reset(0, R.Sampling(greedy=True))
    with pytest.raises(R.Z2BError) as e:
        ctx.slot_prefill(0, prompt(6, 24), spk=spk, spk_pos=6)
    assert e.value.rc == 1 and "spk_pos" in str(e.value)          # Z2B_ERR_ARG
    ctx.close()


def test_negative_speaker_pos_means_no_speaker(tiny, tiny_path):
    """As the reference (src/zonos2-graph.cpp:36-37, 716): a speaker with spk_pos < 0 is
    not injected, so the prefill equals a plain prefill bit for bit; the same holds for the
    teacher-forced logits entry point."""
    hp = tiny.hp
    spk, delta = _inputs(hp, 34)
    p = prompt(7, 25)
    ctx = R.BatchCtx(tiny, 2, 64)
    for s in (0, 1):
        ctx.slot_reset(s, R.Sampling(greedy=True))
    a = ctx.slot_prefill(0, p, spk=spk, spk_pos=-1, spk_emotion_delta=delta)
    b = ctx.slot_prefill(1, p)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    la = tiny.logits(p, spk=spk, spk_pos=-3)
    lb = tiny.logits(p)
    assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
    ctx.close()
