"""Golden block vectors for the dequantisation pins (writes tests/golden/blocks.npz).

For each storage type the file holds raw GGUF blocks whose bytes are random (every bit of
the scale and quant fields varies) except for the f16 scale fields, which are set to
finite values, plus the f32 values gguf-py 0.19.0 decodes them to
(gguf.quants.dequantize, the third-party reference for the block formats used by
zonos2.cpp's loader). Tests compare the oracle, the host repack and the device decode
against these arrays bit for bit.

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import os

import numpy as np
from gguf import GGMLQuantizationType as Q
from gguf.quants import dequantize

HERE = os.path.dirname(os.path.abspath(__file__))


def blocks(qt, rows, k, rng):
    if qt == Q.F16:
        return rng.standard_normal((rows, k)).astype(np.float16).view(np.uint8).reshape(rows, -1)
    per = {Q.Q8_0: (32, 34), Q.Q4_K: (256, 144), Q.Q6_K: (256, 210)}[qt]
    nb = k // per[0]
    b = rng.integers(0, 256, (rows, nb, per[1]), dtype=np.uint8)
    scale = lambda n: (rng.uniform(1e-4, 2e-2, n)).astype(np.float16).view(np.uint8).reshape(-1, 2)
    if qt == Q.Q8_0:
        b[:, :, 0:2] = scale(rows * nb).reshape(rows, nb, 2)
    elif qt == Q.Q4_K:
        b[:, :, 0:2] = scale(rows * nb).reshape(rows, nb, 2)
        b[:, :, 2:4] = scale(rows * nb).reshape(rows, nb, 2)
    else:
        b[:, :, 208:210] = scale(rows * nb).reshape(rows, nb, 2)
    return b.reshape(rows, -1)


def main():
    rng = np.random.default_rng(20240601)
    out = {}
    # (rows, k) chosen to cover partial row-tiles (rows % 16 != 0) and several chunks
    for name, qt, rows, k in [("q8_0", Q.Q8_0, 37, 384), ("q4_k", Q.Q4_K, 21, 512), ("q6_k", Q.Q6_K, 19, 512),
                              ("f16", Q.F16, 23, 192)]:
        raw = blocks(qt, rows, k, rng)
        ref = dequantize(raw, qt).reshape(rows, k).astype(np.float32)
        out[f"{name}_raw"] = raw
        out[f"{name}_f32"] = ref
        out[f"{name}_meta"] = np.array([int(qt), rows, k], np.int64)
    np.savez_compressed(os.path.join(HERE, "blocks.npz"), **out)
    print("wrote", os.path.join(HERE, "blocks.npz"))


if __name__ == "__main__":
    main()
