"""ZONOS2-scale (config 2: d 2048, 28 MoE layers, E 32 top-4, ff 1408, 16x128 / 4 KV,
Q4_K attention and gate/up, F16 down, Q8_0 head/router, Q6_K embeddings) on the GPU:
oracle parity on a short teacher-forced decode, and batch-16 properties at full size."""
from __future__ import annotations

import numpy as np
import pytest

import z2b.runtime as R
import z2b.synth as S
from oracle import oracle as O
from tests.util import cos, max_abs_rel, prompt, run_gpu, run_oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def z2_path(model_dir):
    return S.cached("zonos2", directory=model_dir)


@pytest.fixture(scope="module")
def z2(z2_path):
    m = R.Model(z2_path)
    yield m
    m.close()


def _flips(a, b, L, n, k):
    a, b = a.reshape(L, n, k), b.reshape(L, n, k)
    return sum(set(a[l, t].tolist()) != set(b[l, t].tolist()) for l in range(L) for t in range(n))


def test_config2_decode_parity(z2, z2_path):
    """Teacher-forced against the oracle in exact mode. At 28 MoE layers a near-tie in a
    router's top-k can flip under any rounding change (the reference notes the same for
    the real model); the emulated reference CPU arithmetic (ggml-emu) flips ~7% of the
    (token, layer) decisions vs exact on this model. So: every step whose routing matches
    meets cos >= 0.9999 and max-abs-rel <= 1e-2; the GPU's flip rate stays <= 1% and
    below the emulated reference path's own."""
    prompts = [prompt(16, 80), prompt(24, 81), prompt(40, 82), prompt(9, 83)]
    n, steps = len(prompts), 4
    g = run_gpu(R, z2, prompts, steps, capture_sel=True)
    ox = run_oracle(O, O.Model(z2_path, O.EXACT), prompts, g["fed"], capture_sel=True)
    oe = run_oracle(O, O.Model(z2_path, O.GGML_EMU), prompts, g["fed"], capture_sel=True)
    flips_gpu = flips_emu = 0
    checked = 0
    for s in range(steps):
        fg = _flips(g["sel"][s], ox["sel"][s], 28, n, 4)
        flips_gpu += fg
        flips_emu += _flips(oe["sel"][s], ox["sel"][s], 28, n, 4)
        if fg == 0:
            checked += 1
            for i in range(n):
                assert cos(g["logits"][s, i], ox["logits"][s, i]) >= 0.9999
                assert max_abs_rel(g["logits"][s, i], ox["logits"][s, i]) <= 1e-2
        for i in range(n):
            assert cos(g["logits"][s, i], ox["logits"][s, i]) >= 0.999
    total = steps * 28 * n
    assert checked >= steps // 2
    assert flips_gpu / total <= 0.01, (flips_gpu, total)
    assert flips_gpu <= flips_emu, (flips_gpu, flips_emu)


def test_config2_batch16(z2):
    prompts = [prompt(8 + 2 * i, 90 + i) for i in range(16)]
    g = run_gpu(R, z2, prompts, 4)
    assert np.isfinite(g["logits"]).all()
    solo = run_gpu(R, z2, [prompts[5]], 4)
    assert np.array_equal(solo["logits"][:, 0].view(np.uint32), g["logits"][:, 5].view(np.uint32))
