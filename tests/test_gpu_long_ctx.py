"""Decode over long contexts against the oracle: paged split-K attention across many KV
pages and page boundaries (src/zonos2-graph.cpp:139-153). The contexts are filled with
the same integer-hash values on the GPU (z2b_debug_fill_kv) and in the oracle
(hash_fill), so no prefill of thousands of rows is needed on the CPU. 4-layer cuts of the
ZONOS2 shapes: Q4_K (config 2, contexts U[64, 2048] and U[128, 4096]) and the config-3
types Q6_K and Q8_0 (contexts of 1024 rows and more)."""
from __future__ import annotations

import numpy as np
import pytest

import z2b.runtime as R
import z2b.synth as S
from oracle import oracle as O
from tests.util import cos, max_abs_rel, run_gpu_filled, run_oracle_filled, topk_set_flips

pytestmark = pytest.mark.gpu

COS_MIN, MAR_MAX = 0.9999, 1e-2


def _check(g, o, steps, n):
    checked = 0
    for s in range(steps):
        flips = topk_set_flips(g["sel"][s], o["sel"][s])          # [L][n]
        for i in range(n):
            c, m = cos(g["logits"][s, i], o["logits"][s, i]), max_abs_rel(g["logits"][s, i], o["logits"][s, i])
            assert c >= 0.999, (s, i, c)
            if not flips[:, i].any():                               # routing identical for this token
                checked += 1
                assert c >= COS_MIN and m <= MAR_MAX, (s, i, c, m)
    return checked


@pytest.mark.parametrize("preset,lo,hi", [("zonos2", 64, 2048), ("zonos2", 128, 4096),
                                          ("zonos2_q6k", 1024, 4096), ("zonos2_q8", 1024, 4096)])
def test_long_context_decode_vs_oracle(model_dir, preset, lo, hi):
    path = S.cached(preset, directory=model_dir, n_layer=4, expert_used=[4] * 4)
    g_rng = np.random.default_rng(hi + lo)
    lens = [int(x) for x in g_rng.integers(lo, hi + 1, 4)]
    lens[0] = hi                                                      # the longest context of the range
    lens[1] = max(lo, 2 * 256 + 1)                                    # one row past a page boundary
    steps, seed = 3, 40 + lo
    m = R.Model(path)
    try:
        g = run_gpu_filled(R, m, lens, steps, seed, capture_sel=True)
    finally:
        m.close()
    o = run_oracle_filled(O, O.Model(path, O.EXACT), lens, g["fed"], seed)
    checked = _check(g, o, steps, len(lens))
    print(f"{preset} ctx {lens}: {checked}/{steps * len(lens)} (step, stream) pairs with identical routing "
          f"checked at cos >= {COS_MIN}, max-abs-rel <= {MAR_MAX}")
    assert checked >= steps * len(lens) // 2
