"""The allocation-free segment builder (z2b_route_segments_noalloc): against the
allocating entry point (z2b_test_route) on the same router ids, two calls in a row; its
size limit; and that calls after the first leave the device's free memory unchanged.
Collected last so it also runs after every other GPU test."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import z2b.runtime as R

pytestmark = pytest.mark.gpu

ARGS = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
MAX_ROUTES = 16384          # Z2B_NOALLOC_MAX_ROUTES


def _lib():
    L = R.lib()
    L.z2b_test_route.argtypes = ARGS
    L.z2b_route_segments_noalloc.argtypes = ARGS
    L.z2b_last_error.restype = ctypes.c_char_p
    return L


def _ids(E, k, T, seed):
    g = np.random.default_rng(seed)
    z = 1.0 / np.arange(1, E + 1) ** 1.1
    sel = np.stack([g.choice(E, k, replace=False, p=z / z.sum()) for _ in range(T)]).astype(np.int32)
    sel[g.random(T) < 0.1] = -1                         # padding tokens route nowhere
    return sel, g.random((T, k)).astype(np.float32)


def _call(fn, sel, w, E):
    T, k = sel.shape
    seg = np.full(E + 1, 7, np.int32)
    tok = np.full(T * k, 7, np.int32)
    pos = np.full(T * k, 7, np.int32)
    rc = fn(sel.ctypes.data, w.ctypes.data, T, k, E, seg.ctypes.data, tok.ctypes.data, pos.ctypes.data)
    return rc, seg, tok, pos


@pytest.mark.parametrize("E,k,T", [(32, 4, 16), (256, 8, 2048)])
def test_noalloc_matches_allocating_entry_point(E, k, T):
    L = _lib()
    for call in range(2):                               # two calls in a row reuse the scratch
        sel, w = _ids(E, k, T, seed=1000 * call + T)
        rc0, *ref = _call(L.z2b_test_route, sel, w, E)
        rc1, *got = _call(L.z2b_route_segments_noalloc, sel, w, E)
        assert rc0 == 0 and rc1 == 0, L.z2b_last_error()
        (seg0, tok0, pos0), (seg1, tok1, pos1) = ref, got
        n_routed = int((sel >= 0).sum())
        assert seg0[-1] == n_routed
        assert np.array_equal(seg0, seg1)
        # route_tok past the routed count is written by neither entry point
        assert np.array_equal(tok0[:n_routed], tok1[:n_routed])
        assert np.array_equal(pos0, pos1)


def test_noalloc_rejects_sizes_beyond_the_limit():
    L = _lib()
    sel, w = _ids(8, 2, MAX_ROUTES // 2 + 1, seed=5)
    rc, *_ = _call(L.z2b_route_segments_noalloc, sel, w, 8)
    assert rc == 1                                       # Z2B_ERR_ARG
    assert b"Z2B_NOALLOC_MAX_ROUTES" in L.z2b_last_error()


def _free_device_bytes():
    """cuMemGetInfo on the calling thread's current (primary) context."""
    cu = ctypes.CDLL("libcuda.so.1")
    free, total = ctypes.c_size_t(), ctypes.c_size_t()
    assert cu.cuMemGetInfo_v2(ctypes.byref(free), ctypes.byref(total)) == 0
    return free.value


def test_noalloc_calls_allocate_nothing():
    """After the first call (which does the per-device set-up), further calls do not change
    the device's free memory."""
    L = _lib()
    sel, w = _ids(64, 8, 1024, seed=11)
    rc, *first = _call(L.z2b_route_segments_noalloc, sel, w, 64)
    assert rc == 0, L.z2b_last_error()
    before = _free_device_bytes()
    for i in range(4):
        rc, *again = _call(L.z2b_route_segments_noalloc, sel, w, 64)
        assert rc == 0, L.z2b_last_error()
        assert all(np.array_equal(a, b) for a, b in zip(first, again))
    assert _free_device_bytes() == before
