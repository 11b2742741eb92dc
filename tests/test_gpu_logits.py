"""Teacher-forced logits (zonos2_logits, src/zonos2-graph.cpp:457-473) through the decode
kernels: every row against the oracle, the last row bit-identical to a prefill of the same
rows, with and without a speaker row, across the 512-row step boundary."""
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


@pytest.fixture(scope="module")
def tiny_oracle(tiny_path):
    return O.Model(tiny_path, O.EXACT)


def _check_rows(g, o):
    assert g.shape == o.shape
    worst = min(cos(g[t], o[t]) for t in range(g.shape[0]))
    assert worst >= COS_MIN, worst
    assert max(max_abs_rel(g[t], o[t]) for t in range(g.shape[0])) <= MAR_MAX


def test_logits_every_row_and_last_row_is_prefill(tiny, tiny_oracle):
    p = prompt(40, 31)
    g = tiny.logits(p)
    _check_rows(g, tiny_oracle.logits(p))
    ctx = R.BatchCtx(tiny, 1, 64)
    ctx.slot_reset(0, R.Sampling(greedy=True))
    last = ctx.slot_prefill(0, p)
    ctx.close()
    assert np.array_equal(g[-1].view(np.uint32), last.view(np.uint32))


def test_logits_with_speaker(tiny, tiny_oracle):
    hp = tiny.hp
    rng = np.random.default_rng(41)
    spk = rng.standard_normal(hp.spk_dim).astype(np.float32)
    delta = (0.1 * rng.standard_normal(hp.n_embd)).astype(np.float32)
    p = prompt(24, 32)
    g = tiny.logits(p, spk=spk, spk_pos=1, spk_emotion_delta=delta)
    _check_rows(g, tiny_oracle.logits(p, spk=spk, spk_pos=1, spk_emotion_delta=delta))
    ctx = R.BatchCtx(tiny, 1, 64)
    ctx.slot_reset(0, R.Sampling(greedy=True))
    last = ctx.slot_prefill(0, p, spk=spk, spk_pos=1, spk_emotion_delta=delta)
    ctx.close()
    assert np.array_equal(g[-1].view(np.uint32), last.view(np.uint32))
    with pytest.raises(R.Z2BError):
        tiny.logits(p, spk=spk, spk_pos=24)


def test_logits_across_step_boundary(tiny, tiny_oracle):
    """600 rows run as a 512-row step and an 88-row step over the slot's cache."""
    p = prompt(600, 33)
    g = tiny.logits(p)
    o = tiny_oracle.logits(p)
    _check_rows(g[[0, 255, 511, 512, 513, 599]], o[[0, 255, 511, 512, 513, 599]])
    assert cos(g.ravel(), o.ravel()) >= COS_MIN
