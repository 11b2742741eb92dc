"""One process driving a model and a context on each of two GPUs (the layout of one
context per GPU behind a host router): every kernel's per-device set-up (the dynamic
shared memory opt-ins) holds on the second device, and both devices give bit-identical
results for the same inputs. Skipped with fewer than two GPUs. No peer memory is used."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import z2b.runtime as R
from tests.util import prompt

pytestmark = pytest.mark.gpu


def _device_count():
    try:
        cu = ctypes.CDLL("libcuda.so.1")
    except OSError:
        return 0
    if cu.cuInit(0) != 0:
        return 0
    n = ctypes.c_int(0)
    return n.value if cu.cuDeviceGetCount(ctypes.byref(n)) == 0 else 0


@pytest.mark.skipif(_device_count() < 2, reason="needs two GPUs")
def test_contexts_on_two_devices_in_one_process(tiny_path):
    hp = None
    out = []
    models = [R.Model(tiny_path, dev) for dev in (0, 1)]
    ctxs = [R.BatchCtx(m, 2, 64) for m in models]
    prompts = [prompt(13, 200), prompt(6, 201)]
    for m, c in zip(models, ctxs):
        hp = m.hp
        rows = []
        for i, p in enumerate(prompts):
            c.slot_reset(i, R.Sampling(greedy=True))
            rows.append(np.r_[c.slot_prefill(i, p).argmax(-1), hp.text_vocab])
        ids = np.stack(rows).astype(np.int32)
        past = [len(p) for p in prompts]
        logits = []
        for s in range(3):
            codes, lg = c.step([(0, past[0] + s, 1, R.WANT_SAMPLE), (1, past[1] + s, 1, R.WANT_SAMPLE)], ids)
            logits.append(lg)
            ids = np.concatenate([codes, np.full((2, 1), hp.text_vocab, np.int32)], 1)
        out.append(np.stack(logits))
    assert np.isfinite(out[0]).all()
    assert np.array_equal(out[0].view(np.uint32), out[1].view(np.uint32))
    for c in ctxs:
        c.close()
    for m in models:
        m.close()
