"""End-to-end parity of the B200 decode step against the CPU oracle (teacher-forced:
the oracle is fed exactly the rows the GPU fed itself), plus the reference's batch
self-consistency checks F.1 / F.2 (src/main.cpp:255-268)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import z2b.runtime as R
from oracle import oracle as O
from tests.util import argmax_agree, cos, max_abs_rel, prompt, run_gpu, run_oracle

pytestmark = pytest.mark.gpu

# config 1 workload: 4 streams, prompt lengths {17, 40, 5, 63}, seed 0, 32 greedy steps
LENS = [17, 40, 5, 63]
COS_MIN, MAR_MAX = 0.9999, 1e-2


@pytest.fixture(scope="module")
def tiny(tiny_path):
    m = R.Model(tiny_path)
    yield m
    m.close()


@pytest.fixture(scope="module")
def tiny_oracle(tiny_path):
    return O.Model(tiny_path)


@pytest.fixture(scope="module")
def config1(tiny, tiny_oracle):
    prompts = [prompt(n, i) for i, n in enumerate(LENS)]
    g = run_gpu(R, tiny, prompts, 32, capture_sel=True)
    o = run_oracle(O, tiny_oracle, prompts, g["fed"], capture_sel=True)
    return prompts, g, o


def test_config1_prefill_logits(config1):
    _, g, o = config1
    for i in range(len(LENS)):
        assert cos(g["pre"][i], o["pre"][i]) >= COS_MIN
        assert max_abs_rel(g["pre"][i], o["pre"][i]) <= MAR_MAX


def test_config1_decode_logits(config1):
    _, g, o = config1
    worst_cos, worst_mar = 1.0, 0.0
    for s in range(32):
        for i in range(len(LENS)):
            worst_cos = min(worst_cos, cos(g["logits"][s, i], o["logits"][s, i]))
            worst_mar = max(worst_mar, max_abs_rel(g["logits"][s, i], o["logits"][s, i]))
    assert worst_cos >= COS_MIN, worst_cos
    assert worst_mar <= MAR_MAX, worst_mar
    assert argmax_agree(g["logits"], o["logits"]) > 0.97       # models/compare.py logits bar


def test_config1_greedy_codes_are_argmax(config1):
    _, g, _ = config1
    assert np.array_equal(g["codes"], g["logits"].argmax(-1))


def test_config1_router_topk_agreement(config1, tiny):
    """Router top-k id sets agree with the oracle on >= 99.9% of (token, layer)."""
    _, g, o = config1
    L, k = tiny.hp.n_layer, max(tiny.hp.expert_used[:tiny.hp.n_layer])
    agree = total = 0
    for s in range(32):
        gs = g["sel"][s].reshape(L, len(LENS), k)
        os_ = o["sel"][s].reshape(L, len(LENS), k)
        for l in range(L):
            for t in range(len(LENS)):
                total += 1
                agree += set(gs[l, t].tolist()) == set(os_[l, t].tolist())
    assert agree / total >= 0.999, (agree, total)


def test_f1_batch_invariance_bitexact(tiny, config1):
    """A stream decoded alone gives bit-identical logits to the same stream in the batch."""
    prompts, g, _ = config1
    solo = run_gpu(R, tiny, [prompts[1]], 32)
    assert np.array_equal(solo["logits"][:, 0].view(np.uint32), g["logits"][:, 1].view(np.uint32))


def test_f2_identical_prompts_identical(tiny):
    p = prompt(23, 9)
    r = run_gpu(R, tiny, [p, prompt(11, 10), p], 16)
    assert np.array_equal(r["codes"][:, 0], r["codes"][:, 2])
    assert np.array_equal(r["logits"][:, 0].view(np.uint32), r["logits"][:, 2].view(np.uint32))


def test_mixed_prefill_and_decode_step(tiny):
    """Prompt rows packed into a decode step (ragged T) leave the decode rows bit-identical
    and produce the same last-row logits as a separate prefill."""
    hp = tiny.hp
    pa, pb = prompt(12, 11), prompt(30, 12)
    ctx = R.BatchCtx(tiny, 2, 128)
    for s in (0, 1):
        ctx.slot_reset(s, R.Sampling(greedy=True))
    la = ctx.slot_prefill(0, pa)
    row = np.r_[la.argmax(-1), hp.text_vocab].astype(np.int32)
    _, mixed = ctx.step([(0, 12, 1, R.WANT_SAMPLE), (1, 0, 30, R.WANT_LOGITS)], np.concatenate([row[None], pb]))
    ref = R.BatchCtx(tiny, 2, 128)
    for s in (0, 1):
        ref.slot_reset(s, R.Sampling(greedy=True))
    ref.slot_prefill(0, pa)
    _, alone = ref.step([(0, 12, 1, R.WANT_SAMPLE)], row[None])
    pb_logits = ref.slot_prefill(1, pb)
    assert np.array_equal(mixed[0].view(np.uint32), alone[0].view(np.uint32))
    assert np.array_equal(mixed[1].view(np.uint32), pb_logits.view(np.uint32))


def test_dummy_fixture_greedy_frames(dummy_path):
    """The reference's CI model (F16, dense + top-1 + top-2 MoE layers, head_dim 16):
    prefill + 8 greedy frames against the oracle."""
    m = R.Model(dummy_path)
    om = O.Model(dummy_path)
    prompts = [prompt(20, 21), prompt(7, 22)]
    g = run_gpu(R, m, prompts, 8)
    o = run_oracle(O, om, prompts, g["fed"])
    for s in range(8):
        for i in range(2):
            assert cos(g["logits"][s, i], o["logits"][s, i]) >= COS_MIN
            assert max_abs_rel(g["logits"][s, i], o["logits"][s, i]) <= MAR_MAX
    m.close()


SAMPLER_CASES = [
    # the reference defaults (src/zonos2.h:197-208): top-k 106, min-p 0.18, repetition penalty
    dict(temperature=1.15, top_k=106, top_p=0.0, min_p=0.18, rep_penalty=1.2, rep_window=50, rep_codebooks=8),
    # top-p after a top-k cut
    dict(temperature=0.9, top_k=40, top_p=0.8, min_p=0.0, rep_penalty=1.0, rep_window=50, rep_codebooks=8),
    # every token a candidate: top-p over the probability order, CDF walk in token order
    dict(temperature=1.3, top_k=0, top_p=0.9, min_p=0.05, rep_penalty=1.1, rep_window=20, rep_codebooks=9),
]


@pytest.mark.parametrize("case", range(len(SAMPLER_CASES)))
def test_device_sampler_matches_reference_sampler(tiny, case):
    """Non-greedy sampling on the device vs the reference sampler restated on the host
    (std::mt19937, same seed) fed the very logits the device sampled from: every code
    agrees. Logit ties order by token id on both sides (the reference's partial_sort
    leaves tie order unspecified)."""
    hp = tiny.hp
    sp = SAMPLER_CASES[case]
    ctx = R.BatchCtx(tiny, 2, 256)
    seeds = (1234 + case, 99 + case)
    for slot, seed in zip((0, 1), seeds):
        ctx.slot_reset(slot, R.Sampling(seed=seed, **sp))
    host = [O.Sampler(hp.n_codebooks, seed=s, **sp) for s in seeds]
    lg0 = [ctx.slot_prefill(s, prompt(10 + s, 30 + s)) for s in (0, 1)]
    nxt = [np.r_[x.argmax(-1), hp.text_vocab] for x in lg0]
    past = [10, 11]
    mism = []
    total = 0
    for step in range(40):
        codes, logits = ctx.step([(0, past[0], 1, R.WANT_SAMPLE), (1, past[1], 1, R.WANT_SAMPLE)],
                                 np.stack(nxt).astype(np.int32))
        for s in (0, 1):
            hc = host[s].sample(logits[s])
            total += hp.n_codebooks
            for cb in np.nonzero(hc != codes[s])[0]:
                mism.append((step, s, int(cb), int(hc[cb]), int(codes[s][cb])))
            nxt[s] = np.r_[codes[s], hp.text_vocab]
            past[s] += 1
    print(f"sampler case {case}: {total - len(mism)}/{total} codes agree")
    assert not mism, mism[:10]


def test_cfg_twin_guidance(tiny):
    """Emotion CFG: guided = u + s * (c - u) (src/zonos2-graph.cpp:917-918), greedy on it."""
    hp = tiny.hp
    ctx = R.BatchCtx(tiny, 2, 64)
    for s in (0, 1):
        ctx.slot_reset(s, R.Sampling(greedy=True))
    ctx.slot_prefill(0, prompt(8, 40))
    ctx.slot_prefill(1, prompt(8, 41))
    ids = np.stack([prompt(1, 42)[0], prompt(1, 42)[0]])
    codes, lg = ctx.step([(0, 8, 1, R.WANT_SAMPLE, 1, 2.5), (1, 8, 1, R.WANT_LOGITS)], ids)
    guided = lg[1] + np.float32(2.5) * (lg[0] - lg[1])
    assert np.array_equal(codes[0], guided.argmax(-1))


def test_expert_mask(tiny_path, tiny_oracle):
    m = R.Model(tiny_path)
    keep = {0: [0, 1, 2], 2: [5, 6, 7]}
    m.set_expert_mask(keep)
    tiny_oracle.set_expert_mask(keep)
    prompts = [prompt(9, 50), prompt(14, 51)]
    g = run_gpu(R, m, prompts, 4, capture_sel=True)
    o = run_oracle(O, tiny_oracle, prompts, g["fed"])
    tiny_oracle.set_expert_mask({})
    L, k = m.hp.n_layer, 2
    for s in range(4):
        sel = g["sel"][s].reshape(L, 2, k)
        assert set(sel[0].ravel()) <= set(keep[0]) and set(sel[2].ravel()) <= set(keep[2])
        for i in range(2):
            assert cos(g["logits"][s, i], o["logits"][s, i]) >= COS_MIN
    m.close()


def test_bad_ids_report_device_error(tiny):
    """An out-of-range id is caught by the embedding kernel's bounds check and reported
    as Z2B_ERR_DEVICE; the context stays usable."""
    ctx = R.BatchCtx(tiny, 1, 64)
    ctx.slot_reset(0)
    bad = prompt(4, 60)
    bad[2, 3] = 5000
    with pytest.raises(R.Z2BError) as e:
        ctx.slot_prefill(0, bad)
    assert e.value.rc == 6
    ok = ctx.slot_prefill(0, prompt(4, 61))
    assert np.isfinite(ok).all()


def test_decode_loop_matches_stepping(tiny):
    """The device-resident loop (fed back on the device) leaves the same state as stepping
    through the public call one step at a time."""
    hp = tiny.hp
    prompts = [prompt(6, 70), prompt(9, 71), prompt(3, 72)]
    a, b = R.BatchCtx(tiny, 3, 64), R.BatchCtx(tiny, 3, 64)
    first = []
    for i, p in enumerate(prompts):
        for c in (a, b):
            c.slot_reset(i, R.Sampling(greedy=True))
        lg = a.slot_prefill(i, p)
        b.slot_prefill(i, p)
        first.append(np.r_[lg.argmax(-1), hp.text_vocab])
    first = np.stack(first).astype(np.int32)
    past = [len(p) for p in prompts]
    a.decode_loop([(i, past[i]) for i in range(3)], first, 5)
    a.sync()
    nxt = first
    for s in range(5):
        codes, _ = b.step([(i, past[i] + s, 1, R.WANT_SAMPLE) for i in range(3)], nxt)
        nxt = np.concatenate([codes, np.full((3, 1), hp.text_vocab, np.int32)], 1)
    ca, la = a.step([(i, past[i] + 5, 1, R.WANT_SAMPLE) for i in range(3)], nxt)
    cb, lb = b.step([(i, past[i] + 5, 1, R.WANT_SAMPLE) for i in range(3)], nxt)
    assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))


def test_step_logits_view(tiny):
    """z2b_step_logits (zonos2_batch_slot_logits) after a z2b_step given no out_logits: the
    per-desc host view equals, bit for bit, the logits a second context returned through
    out_logits; descs without Z2B_WANT_LOGITS and out-of-range indices have none; with
    readback off and no out_logits there is no view."""
    hp = tiny.hp
    prompts = [prompt(9, 300), prompt(14, 301), prompt(4, 302)]
    a, b = R.BatchCtx(tiny, 3, 64), R.BatchCtx(tiny, 3, 64)
    rows = []
    for i, p in enumerate(prompts):
        for c in (a, b):
            c.slot_reset(i, R.Sampling(greedy=True))
        rows.append(np.r_[a.slot_prefill(i, p).argmax(-1), hp.text_vocab])
        b.slot_prefill(i, p)
    ids = np.stack(rows).astype(np.int32)
    past = [len(p) for p in prompts]
    for s in range(3):
        descs = [(0, past[0] + s, 1, R.WANT_SAMPLE), (1, past[1] + s, 1, 0), (2, past[2] + s, 1, R.WANT_LOGITS)]
        ca, la = a.step(descs, ids)
        cb, _ = b.step(descs, ids, want_logits=False)
        assert np.array_equal(ca[0], cb[0])
        for i in (0, 2):
            v = b.step_logits(i)
            assert v is not None and np.array_equal(v.view(np.uint32), la[i].view(np.uint32))
        assert b.step_logits(1) is None and b.step_logits(3) is None and b.step_logits(-1) is None
        ids = np.concatenate([ca[:1], ca[:1], ca[:1]], 0)
        ids = np.concatenate([ids, np.full((3, 1), hp.text_vocab, np.int32)], 1).astype(np.int32)
    b.set_logits_readback(False)
    b.step([(0, past[0] + 3, 1, R.WANT_SAMPLE)], ids[:1], want_logits=False)
    assert b.step_logits(0) is None
    a.close()
    b.close()


def test_set_sampling_after_prefill_keeps_the_stream(tiny):
    """z2b_set_slot_sampling after a prefill (the shim's device-sampling opt-in) samples
    exactly as a stream whose sampler was set before its prefill, and keeps its KV."""
    hp = tiny.hp
    sp = R.Sampling(seed=77, temperature=1.1, top_k=50, min_p=0.1)
    p = prompt(12, 310)
    a, b = R.BatchCtx(tiny, 1, 64), R.BatchCtx(tiny, 1, 64)
    a.slot_reset(0, sp)
    la = a.slot_prefill(0, p)
    b.slot_reset(0, R.Sampling(greedy=True))
    lb = b.slot_prefill(0, p)
    b.set_sampling(0, sp)
    assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
    ids = np.r_[la.argmax(-1), hp.text_vocab][None].astype(np.int32)
    for s in range(6):
        ca, ga = a.step([(0, 12 + s, 1, R.WANT_SAMPLE)], ids)
        cb, gb = b.step([(0, 12 + s, 1, R.WANT_SAMPLE)], ids)
        assert np.array_equal(ca, cb) and np.array_equal(ga.view(np.uint32), gb.view(np.uint32))
        ids = np.r_[ca[0], hp.text_vocab][None].astype(np.int32)
    a.close()
    b.close()
