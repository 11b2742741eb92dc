"""Kernel-level parity on the GPU: device block decode bit-exact against gguf-py's golden
vectors, tile GEMV against an fp32 reference of the same op, and the device packer and
expert permutation bit-exact against their definitions."""
from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest

import z2b.runtime as R
from tests.util import cos, max_abs_rel

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = np.load(os.path.join(HERE, "golden", "blocks.npz"))
TYPES = ["q8_0", "q4_k", "q6_k", "f16"]


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("name", TYPES)
@pytest.mark.parametrize("from_tiles", [True, False])
def test_device_dequant_bitexact(name, from_tiles):
    qt, rows, k = (int(x) for x in GOLD[f"{name}_meta"])
    if from_tiles and name == "q8_0" and k % 128:
        pytest.skip("no tile layout")
    out = R.test_dequant(qt, rows, k, GOLD[f"{name}_raw"], from_tiles)
    assert np.array_equal(_bits(out), _bits(GOLD[f"{name}_f32"]))


@pytest.mark.parametrize("name", TYPES)
@pytest.mark.parametrize("n_tok", [1, 3, 8, 16, 21])
def test_gemv_vs_fp32(name, n_tok):
    """Tile GEMV (f16 weights/activations on mma.sync, f32 accumulate) vs x @ W^T in fp32."""
    qt, rows, k = (int(x) for x in GOLD[f"{name}_meta"])
    w = GOLD[f"{name}_f32"]
    x = np.random.default_rng(n_tok).standard_normal((n_tok, k)).astype(np.float16)
    y = R.test_gemv(qt, rows, k, GOLD[f"{name}_raw"], x)
    ref = x.astype(np.float32) @ w.T
    assert cos(y, ref) > 0.99999
    assert max_abs_rel(y, ref) < 2e-3


def test_pack_prefix_sum_bitexact():
    """Ragged packing: single-row descs take tokens [0, T_dec) in desc order, then the rows of
    each prompt chunk follow in desc order (token of row r of a chunk: T_dec + prefix of
    the chunks' rows + r) with position n_past + r; descs with an output flag get output
    rows in desc order (their last token)."""
    L = R.lib()
    L.z2b_test_pack.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int] + [ctypes.c_void_p] * 4
    g = np.random.default_rng(5)
    for trial in range(20):
        n = int(g.integers(1, 40))
        d = np.zeros((n, 4), np.int32)
        d[:, 0] = g.permutation(64)[:n]
        d[:, 1] = g.integers(0, 3000, n)
        d[:, 2] = np.where(g.random(n) < 0.3, g.integers(1, 60, n), 1)
        d[:, 3] = g.random(n) < 0.8
        T = int(d[:, 2].sum())
        ts, tp, to = (np.empty(T, np.int32) for _ in range(3))
        ot = np.empty(max(int(d[:, 3].sum()), 1), np.int32)
        assert L.z2b_test_pack(d.ctypes.data, n, T, ts.ctypes.data, tp.ctypes.data, to.ctypes.data, ot.ctypes.data) == 0
        dec = d[:, 2] == 1
        t_dec = int(dec.sum())
        start = np.where(dec, np.cumsum(dec) - 1, t_dec + np.cumsum(np.where(dec, 0, d[:, 2])) - d[:, 2])
        es = np.full(T, -1, np.int32)
        ep = np.full(T, -1, np.int32)
        for i in range(n):
            es[start[i]:start[i] + d[i, 2]] = d[i, 0]
            ep[start[i]:start[i] + d[i, 2]] = d[i, 1] + np.arange(d[i, 2])
        orow = np.cumsum(d[:, 3]) - 1
        eo = np.full(T, -1, np.int32)
        eot = []
        for i in range(n):
            if d[i, 3]:
                eo[start[i] + d[i, 2] - 1] = orow[i]
                eot.append(start[i] + d[i, 2] - 1)
        assert np.array_equal(ts, es) and np.array_equal(tp, ep) and np.array_equal(to, eo)
        assert np.array_equal(ot[:len(eot)], np.array(eot, np.int32))


@pytest.mark.parametrize("E,k,T", [(32, 4, 16), (8, 2, 4), (32, 4, 300), (4, 1, 7), (256, 8, 64)])
def test_route_permutation_bitexact(E, k, T):
    """Given router ids, routes are sorted by (expert, token, rank) and every route's
    position is recorded (token->expert permutation + segment offsets)."""
    L = R.lib()
    L.z2b_test_route.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                 ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    g = np.random.default_rng(E * 100 + T)
    z = 1.0 / np.arange(1, E + 1) ** 1.1                 # Zipf-skewed load
    sel = np.stack([g.choice(E, k, replace=False, p=z / z.sum()) for _ in range(T)]).astype(np.int32)
    w = g.random((T, k)).astype(np.float32)
    seg = np.empty(E + 1, np.int32)
    tok = np.empty(T * k, np.int32)
    pos = np.empty(T * k, np.int32)
    assert L.z2b_test_route(sel.ctypes.data, w.ctypes.data, T, k, E, seg.ctypes.data, tok.ctypes.data, pos.ctypes.data) == 0
    order = sorted(range(T * k), key=lambda r: (sel.ravel()[r], r))
    exp_tok = np.array([r // k for r in order], np.int32)
    exp_pos = np.empty(T * k, np.int32)
    exp_pos[order] = np.arange(T * k)
    counts = np.bincount(sel.ravel(), minlength=E)
    assert np.array_equal(seg, np.concatenate([[0], np.cumsum(counts)]).astype(np.int32))
    assert np.array_equal(tok, exp_tok) and np.array_equal(pos, exp_pos)


def test_bounded_wait_gives_up_and_reports():
    """The kernels' mbarrier wait on a phase nothing completes: it stops after its poll
    limit, sets DERR_WAIT_TIMEOUT and returns; the context keeps working afterwards."""
    L = R.lib()
    L.z2b_test_wait_timeout.argtypes = [ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    err, out, ns = ctypes.c_uint32(7), ctypes.c_uint32(7), ctypes.c_uint64(0)
    assert L.z2b_test_wait_timeout(64, ctypes.byref(err), ctypes.byref(out), ctypes.byref(ns)) == 0
    assert out.value == 2 and err.value == 1
    print(f"bounded wait: 64 polls gave up after {ns.value / 1e3:.1f} us")
    assert ns.value < 5e9
    # the device is still usable: a kernel test right after succeeds
    test_pack_prefix_sum_bitexact()
