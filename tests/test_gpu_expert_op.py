"""The isolated MoE expert op (config 4 of the benchmark set: E 32, d 2048, ff 1408, Q4_K
gate/up, F16 down, top-4 routing skewed by a Zipf(1.1) bias) through z2b_expert_op,
against a float32 numpy restatement over gguf-py's dequantised weights, at every token
count of the config-4 sweep (T = 16, 64, 256, 1024, 4096) plus 320. The experts with >= 9
routes take the tcgen05 GEMM from T = 64 (T = 16 runs on the tile GEMV only);
at 1024 and 4096 the most-loaded experts span several token tiles, the last one partial."""
from __future__ import annotations

import numpy as np
import pytest

import z2b.runtime as R
import z2b.synth as S

pytestmark = pytest.mark.gpu

GEMM_MIN = 9                                   # z2b_expert_op's default GEMV / GEMM threshold


def routing(T, E, k, seed):
    """Router logits N(0, 1) + Zipf(s = 1.1) per-expert bias, softmax, top-k; route
    weight = the selected probability (no renormalisation, as the model)."""
    g = np.random.default_rng(seed)
    bias = np.log(1.0 / np.arange(1, E + 1) ** 1.1)
    logits = g.standard_normal((T, E)) + bias[g.permutation(E)]
    p = np.exp(logits - logits.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    sel = np.argsort(-p, 1, kind="stable")[:, :k].astype(np.int32)
    return sel, np.take_along_axis(p, sel, 1).astype(np.float32)


_W = {}


def _weights(path):
    if path not in _W:
        from gguf import GGUFReader
        from gguf.quants import dequantize
        rd = GGUFReader(path)
        t = {tt.name: tt for tt in rd.tensors}
        _W.clear()
        _W[path] = {n: dequantize(t[f"blk.0.ffn_{n}_exps.weight"].data,
                                  t[f"blk.0.ffn_{n}_exps.weight"].tensor_type).astype(np.float32)
                    for n in ("gate", "up", "down")}
    return _W[path]


def reference(path, x, sel, w):
    W = _weights(path)
    out = np.zeros_like(x)
    for e in np.unique(sel):
        rows, cols = np.nonzero(sel == e)
        xe = x[rows]
        gt = xe @ W["gate"][e].T
        y = (gt / (1.0 + np.exp(-gt))) * (xe @ W["up"][e].T)
        out[rows] += w[rows, cols][:, None] * (y @ W["down"][e].T)
    return out


@pytest.mark.parametrize("T", [16, 64, 256, 320, 1024, 4096])
def test_expert_op_vs_float32(model_dir, T):
    path = S.cached("zonos2", directory=model_dir, n_layer=1, expert_used=[4])
    m = R.Model(path)
    try:
        ctx = R.BatchCtx(m, 16, 64)
        x = np.random.default_rng(T).standard_normal((T, m.hp.n_embd)).astype(np.float32)
        sel, w = routing(T, m.hp.n_expert, 4, seed=T + 1)
        out, _, nbytes, n_gemm = ctx.expert_op(0, x, sel, w)
        ctx.close()
    finally:
        m.close()
    counts = np.bincount(sel.ravel(), minlength=m.hp.n_expert)
    expected = int((counts >= GEMM_MIN).sum()) if T >= 64 else 0   # the op launches the GEMM from 64 rows
    assert n_gemm == expected                  # the loaded experts took the tensor-core path
    if T >= 64:
        assert n_gemm > 0
    ref = reference(path, x, sel, w)
    a, b = out.astype(np.float64), ref.astype(np.float64)
    c = (a * b).sum(1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1))
    print(f"T {T}: {n_gemm} experts on the tcgen05 GEMM, worst token cos {c.min():.7f}")
    assert c.min() >= 0.9999, (int(c.argmin()), c.min())
    assert np.abs(out - ref).max() / np.abs(ref).max() <= 1e-2


@pytest.mark.parametrize("gemm_min", [1, 1 << 30])
def test_expert_op_forced_path(model_dir, gemm_min):
    """The threshold of z2b_set_expert_gemm_min: 1 sends every expert (down to 1-route ones,
    a 16-wide MMA over a single route) to the tcgen05 GEMM, 2^30 every expert to the tile
    GEMV (up to ~40 routes, three 16-token passes); both match the float32 reference."""
    path = S.cached("zonos2", directory=model_dir, n_layer=1, expert_used=[4])
    m = R.Model(path)
    T = 96
    try:
        ctx = R.BatchCtx(m, 16, 64)
        ctx.set_expert_gemm_min(gemm_min)
        x = np.random.default_rng(5).standard_normal((T, m.hp.n_embd)).astype(np.float32)
        sel, w = routing(T, m.hp.n_expert, 4, seed=6)
        out, _, _, n_gemm = ctx.expert_op(0, x, sel, w)
        with pytest.raises(RuntimeError):
            ctx.set_expert_gemm_min(0)
        ctx.close()
    finally:
        m.close()
    assert n_gemm == (len(np.unique(sel)) if gemm_min == 1 else 0)
    ref = reference(path, x, sel, w)
    a, b = out.astype(np.float64), ref.astype(np.float64)
    c = (a * b).sum(1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1))
    print(f"gemm_min {gemm_min}: {n_gemm} experts on the tcgen05 GEMM, worst token cos {c.min():.7f}")
    assert c.min() >= 0.9999, (int(c.argmin()), c.min())
    assert np.abs(out - ref).max() / np.abs(ref).max() <= 1e-2
