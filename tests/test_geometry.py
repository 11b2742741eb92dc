"""Launch geometry of the tile GEMV (host logic, no GPU): shared memory within the SM at
the intended blocks per SM, and, for the projections, the layout of each warp's shared
activation slice: every 16-byte unit written once and inside the slice, every fragment
read finding the token and K position it needs, and the 8 lanes of each quarter-warp
reading 8 distinct bank groups."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import z2b.build as B

GT = {"Q4_K": 12, "Q6_K": 14, "Q8_0": 8, "F16": 1}
SM_BYTES, BLOCK_RESERVED, MAX_BLOCK = 233472, 1024, 232448


def _geom(type_id, k, nmat, ntg):
    L = ctypes.CDLL(B.LIB)
    out = np.zeros(7, np.int32)
    rc = L.z2b_test_gemv_geometry(ctypes.c_uint32(type_id), ctypes.c_int64(k), nmat, ntg,
                                  out.ctypes.data_as(ctypes.c_void_p))
    assert rc == 0
    return dict(zip(["nw", "ns", "sb", "smem", "cps", "x_rs", "cpw"], out.tolist()))


CASES = ([(t, k) for t in ("Q4_K", "Q6_K", "Q8_0") for k in (256, 1024, 2048, 4096)]
         + [("F16", k) for k in (256, 512, 1408, 2048)])


@pytest.mark.parametrize("wt,k", CASES)
@pytest.mark.parametrize("nmat,ntg,want", [(1, 2, 2), (2, 2, 2), (2, 1, 2), (1, 1, 3)])
def test_shared_memory_fits(wt, k, nmat, ntg, want):
    g = _geom(GT[wt], k, nmat, ntg)
    assert 1 <= g["ns"] <= 4 and g["nw"] >= 1
    assert g["smem"] <= MAX_BLOCK
    if g["x_rs"]:
        assert nmat == 1 and ntg == 2
        assert want * (g["smem"] + BLOCK_RESERVED) <= SM_BYTES   # staging never costs a block per SM


@pytest.mark.parametrize("wt,k", CASES)
def test_projection_activation_slice_layout(wt, k):
    g = _geom(GT[wt], k, 1, 2)
    rs = g["x_rs"]
    if rs == 0:
        pytest.skip("activations read into registers for this shape")
    steps = {12: 16, 14: 16, 8: 8}.get(GT[wt])
    if steps is None:                   # F16: steps from the tile geometry (16 k per step)
        steps = 4 if k % 64 == 0 else (2 if k % 32 == 0 else 1)
    KC, KS = 16 * steps, steps
    QU, QSB = KC // 32, (KC // 32 + 1) * 16
    cpw, NTG = g["cpw"], 2
    size = 8 * NTG * rs
    written = {}
    upr = cpw * 4 * QU
    for i in range(8 * NTG * upr):
        n, u = divmod(i, upr)
        cc, w = divmod(u, 4 * QU)
        qq, uu = divmod(w, QU)
        off = n * rs + cc * 4 * QSB + qq * QSB + uu * 16
        assert 0 <= off and off + 16 <= size
        assert off not in written
        written[off] = (n, cc * KC + w * 8)
    for nt in range(NTG):
        for cc in range(cpw):
            for s in range(0, KS, 2):
                groups = [set() for _ in range(4)]
                for lane in range(32):
                    r8, q = lane >> 2, lane & 3
                    off = (nt * 8 + r8) * rs + q * QSB + cc * 4 * QSB + (s // 2) * 16
                    assert written[off] == (nt * 8 + r8, cc * KC + q * (KC // 4) + 4 * s)
                    groups[lane // 8].add((off // 16) % 8)
                assert all(len(gr) == 8 for gr in groups)
