"""Test helpers: seeded prompts and the reference's comparison metrics
(models/compare.py:24-41) plus the max-abs-relative bound used for logits."""
from __future__ import annotations

import numpy as np


def prompt(n, seed, text_vocab=519):
    """n input rows: 9 audio ids uniform in [0, 1024), text id uniform in [0, text_vocab]."""
    g = np.random.default_rng(seed)
    a = g.integers(0, 1024, (n, 10))
    a[:, 9] = g.integers(0, text_vocab + 1, n)
    return a.astype(np.int32)


def cos(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30))


def max_abs_rel(a, b):
    """max |a - b| / max |b|: the logits tolerance (<= 1e-2) of the parity bar."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / (np.abs(b).max() + 1e-30))


def argmax_agree(a, b):
    return float((np.asarray(a).argmax(-1) == np.asarray(b).argmax(-1)).mean())


def run_gpu(R, model, prompts, steps, sampling=None, cap_extra=8, capture_sel=False):
    """Prefill each prompt into its own slot, then `steps` batched decode steps where every
    stream is fed its previous frame (device-sampled) + the text pad. Returns dict with
    prefill logits, per-step logits [steps][n][ncb][av], codes, fed ids and router ids."""
    import ctypes
    hp = model.hp
    n = len(prompts)
    ctx = R.BatchCtx(model, n, max(len(p) for p in prompts) + steps + cap_extra)
    pre, slots, fed, sels, logits, codes_all = [], [], [], [], [], []
    for i, p in enumerate(prompts):
        ctx.slot_reset(i, sampling or R.Sampling(greedy=True))
        lg = ctx.slot_prefill(i, p)
        pre.append(lg)
        s = R.Slot(index=i, n_past=len(p))
        R.slot_after_sample(hp, s, lg.argmax(-1), 10 ** 9)
        slots.append(s)
    for _ in range(steps):
        descs = [(s.index, s.n_past, 1, R.WANT_SAMPLE) for s in slots]
        ids = np.array([s.next_ids for s in slots], np.int32)
        fed.append(ids)
        codes, lg = ctx.step(descs, ids)
        logits.append(lg)
        codes_all.append(codes)
        if capture_sel:
            L = R.lib()
            L.z2b_debug_last_sel.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
            need = L.z2b_debug_last_sel(ctx.h, None, 0)
            buf = np.empty(need, np.int32)
            L.z2b_debug_last_sel(ctx.h, buf.ctypes.data, need)
            sels.append(buf)
        for i, s in enumerate(slots):
            s.n_past += 1
            R.slot_after_sample(hp, s, codes[i], 10 ** 9)
    ctx.close()
    return dict(pre=np.stack(pre), logits=np.stack(logits) if logits else None, codes=np.stack(codes_all) if codes_all else None,
                fed=np.stack(fed) if fed else None, sel=sels)


def run_oracle(O, om, prompts, fed, capture_sel=False):
    """Teacher-forced oracle: same prompts, then the GPU's fed rows at each step."""
    n = len(prompts)
    c = O.Ctx(om, n, max(len(p) for p in prompts) + len(fed) + 8)
    pre = np.stack([c.prefill(i, p) for i, p in enumerate(prompts)])
    past = [len(p) for p in prompts]
    logits, sels = [], []
    for ids in fed:
        logits.append(c.step(list(range(n)), past, ids))
        if capture_sel:
            sels.append(c.last_sel())
        past = [x + 1 for x in past]
    return dict(pre=pre, logits=np.stack(logits) if logits else None, sel=sels)


def run_gpu_filled(R, model, ctx_lens, steps, seed, capture_sel=False):
    """Streams whose KV of positions [0, ctx_lens[i]) comes from the hash fill (seed + i),
    then `steps` batched greedy decode steps starting from a random row each. Returns
    per-step logits [steps][n][ncb][av], the fed rows and, optionally, router ids."""
    hp = model.hp
    n = len(ctx_lens)
    ctx = R.BatchCtx(model, n, max(ctx_lens) + steps + 8)
    for i, L in enumerate(ctx_lens):
        ctx.slot_reset(i, R.Sampling(greedy=True))
        ctx.fill_kv(i, int(L), seed + i)
    ids = np.stack([prompt(1, seed + 500 + i)[0] for i in range(n)]).astype(np.int32)
    past = [int(L) for L in ctx_lens]
    fed, logits, sels = [], [], []
    for s in range(steps):
        fed.append(ids)
        codes, lg = ctx.step([(i, past[i] + s, 1, R.WANT_SAMPLE) for i in range(n)], ids)
        logits.append(lg)
        if capture_sel:
            sels.append(ctx.last_sel().reshape(hp.n_layer, n, -1))
        ids = np.concatenate([codes, np.full((n, 1), hp.text_vocab, np.int32)], 1).astype(np.int32)
    ctx.close()
    return dict(logits=np.stack(logits), fed=np.stack(fed), sel=sels)


def run_oracle_filled(O, om, ctx_lens, fed, seed):
    """The oracle over the same hash-filled contexts, teacher-forced with the GPU's rows."""
    n = len(ctx_lens)
    c = O.Ctx(om, n, max(ctx_lens) + len(fed) + 8)
    for i, L in enumerate(ctx_lens):
        c.hash_fill(i, int(L), seed + i)
    past = [int(L) for L in ctx_lens]
    logits, sels = [], []
    for s, ids in enumerate(fed):
        logits.append(c.step(list(range(n)), [p + s for p in past], ids))
        sels.append(c.last_sel().reshape(-1, n, int(max(om.expert_used))))
    return dict(logits=np.stack(logits), sel=sels)


def topk_set_flips(a, b):
    """Per (layer, token) whether the sets of router ids differ: a, b [L][n][k]."""
    a, b = np.sort(np.asarray(a), -1), np.sort(np.asarray(b), -1)
    return (a != b).any(-1)
