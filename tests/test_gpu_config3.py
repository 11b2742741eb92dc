"""Config 3 shapes (ZONOS2 backbone at Q6_K and at Q8_0, mixed prefill + decode steps) on
the GPU. Parity against the oracle on a 4-layer cut of the model with a mixed batch the
oracle finishes in seconds; at batch 64 (60 decode streams + 4 new prompts per step) the
batch-invariance property of the reference's --batch-test (src/main.cpp:255-268)."""
from __future__ import annotations

import numpy as np
import pytest

import z2b.runtime as R
import z2b.synth as S
from oracle import oracle as O
from tests.util import cos, max_abs_rel, prompt

pytestmark = pytest.mark.gpu


def _model(model_dir, preset, layers):
    return S.cached(preset, directory=model_dir, n_layer=layers, expert_used=[4] * layers)


def _mixed_run(model, n_dec, dec_lens, new_lens, steps, seed):
    """n_dec streams prefilled with dec_lens rows, then `steps` mixed steps: every decode
    stream feeds its last frame, and len(new_lens[s]) new streams are admitted with
    their prompt rows in the same step. Returns per-step (descs, ids, logits, codes)."""
    hp = model.hp
    n_new_total = sum(len(x) for x in new_lens)
    ctx = R.BatchCtx(model, n_dec + n_new_total, max(dec_lens + [max(x) for x in new_lens if x]) + steps + 8)
    past, last = [], []
    for i in range(n_dec):
        ctx.slot_reset(i, R.Sampling(greedy=True))
        lg = ctx.slot_prefill(i, prompt(dec_lens[i], seed + i))
        past.append(dec_lens[i])
        last.append(np.r_[lg.argmax(-1), hp.text_vocab].astype(np.int32))
    out = []
    nxt = n_dec
    for s in range(steps):
        descs, rows, new_prompts = [], [], []
        for i in range(n_dec):
            descs.append((i, past[i], 1, R.WANT_SAMPLE))
            rows.append(last[i][None])
        for j, n in enumerate(new_lens[s]):
            p = prompt(n, seed + 1000 + 10 * s + j)
            ctx.slot_reset(nxt, R.Sampling(greedy=True))
            descs.append((nxt, 0, n, R.WANT_SAMPLE))
            rows.append(p)
            new_prompts.append((nxt, p))
            nxt += 1
        ids = np.concatenate(rows)
        codes, lg = ctx.step(descs, ids)
        out.append(dict(descs=descs, ids=ids, logits=lg, codes=codes, new=new_prompts,
                        dec_ids=np.stack([last[i] for i in range(n_dec)]), past=list(past)))
        for i in range(n_dec):
            past[i] += 1
            last[i] = np.r_[codes[i], hp.text_vocab].astype(np.int32)
    ctx.close()
    return out


@pytest.mark.parametrize("preset", ["zonos2_q6k", "zonos2_q8"])
def test_config3_mixed_step_parity(model_dir, preset):
    path = _model(model_dir, preset, 4)
    m = R.Model(path)
    try:
        n_dec = 10
        dec_lens = [int(x) for x in np.random.default_rng(5).integers(16, 48, n_dec)]
        new_lens = [[20, 33], [17], [40, 25]]
        run = _mixed_run(m, n_dec, dec_lens, new_lens, 3, seed=300)
    finally:
        m.close()
    om = O.Model(path, O.EXACT)
    oc = O.Ctx(om, n_dec + 5, 64 + 8)
    for i in range(n_dec):
        oc.prefill(i, prompt(dec_lens[i], 300 + i))
    worst = 1.0
    for st in run:
        ref_dec = oc.step(list(range(n_dec)), st["past"], st["dec_ids"])
        ref = list(ref_dec) + [oc.prefill(slot, p) for slot, p in st["new"]]
        for i, r in enumerate(ref):
            c = cos(st["logits"][i], r)
            worst = min(worst, c)
            assert c >= 0.9999, (preset, i, c)
            assert max_abs_rel(st["logits"][i], r) <= 1e-2
    assert worst >= 0.9999


def test_config3_batch64_invariance(model_dir):
    """60 decode streams + 4 new prompts per step at 8 layers (Q6_K): every decode
    stream's logits in the mixed batch equal, bit for bit, the same stream decoded alone.
    The prompt rows' routes run on the tensor-core GEMM while decode rows stay on the
    GEMV, so a decode row's arithmetic never depends on what else the step carries."""
    path = _model(model_dir, "zonos2_q6k", 8)
    m = R.Model(path)
    try:
        g = np.random.default_rng(9)
        dec_lens = [int(x) for x in g.integers(128, 512, 60)]
        new_lens = [[int(x) for x in g.integers(32, 512, 4)] for _ in range(2)]
        run = _mixed_run(m, 60, dec_lens, new_lens, 2, seed=700)
        assert all(np.isfinite(st["logits"]).all() for st in run)
        for k in (3, 41):
            solo = _mixed_run(m, 1, [dec_lens[k]], [[], []], 2, seed=700 + k)
            for s in range(2):
                assert np.array_equal(solo[s]["logits"][0].view(np.uint32), run[s]["logits"][k].view(np.uint32))
    finally:
        m.close()


@pytest.mark.parametrize("preset", ["zonos2", "zonos2_q6k", "zonos2_q8"])
def test_long_prompt_tensor_core_path_parity(model_dir, preset):
    """A 512-row prompt in one step: every route of a prompt row runs on the tcgen05
    grouped GEMM (about 64 tokens per expert, so several 64-token tiles per expert and
    partial last tiles): the prompt's last-row logits against the oracle."""
    path = _model(model_dir, preset, 4)
    m = R.Model(path)
    try:
        ctx = R.BatchCtx(m, 1, 600)
        p = prompt(512, 4242)
        ctx.slot_reset(0, R.Sampling(greedy=True))
        lg = ctx.slot_prefill(0, p)
        ctx.close()
    finally:
        m.close()
    oc = O.Ctx(O.Model(path, O.EXACT), 1, 600)
    ref = oc.prefill(0, p)
    assert cos(lg, ref) >= 0.9999, cos(lg, ref)
    assert max_abs_rel(lg, ref) <= 1e-2
