"""Block-format pins (CPU): golden vectors vs gguf-py, oracle dequant, host tile repack."""
from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest
from gguf import GGMLQuantizationType as Q
from gguf.quants import dequantize, quantize

from oracle import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = np.load(os.path.join(HERE, "golden", "blocks.npz"))
TYPES = ["q8_0", "q4_k", "q6_k", "f16"]


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("name", TYPES)
def test_golden_matches_gguf_py(name):
    qt, rows, k = (int(x) for x in GOLD[f"{name}_meta"])
    ref = dequantize(GOLD[f"{name}_raw"], Q(qt)).reshape(rows, k).astype(np.float32)
    assert np.array_equal(_bits(ref), _bits(GOLD[f"{name}_f32"]))


@pytest.mark.parametrize("name", TYPES)
def test_oracle_dequant_bitexact(name):
    qt, rows, k = (int(x) for x in GOLD[f"{name}_meta"])
    out = O.dequant(qt, GOLD[f"{name}_raw"], rows * k).reshape(rows, k)
    assert np.array_equal(_bits(out), _bits(GOLD[f"{name}_f32"]))


def _host_lib():
    import z2b.runtime as R
    return R.lib()


@pytest.mark.parametrize("name", TYPES)
def test_host_repack_roundtrip_bitexact(name):
    """Tile image -> f32 on the host equals gguf-py, including padded partial row-tiles."""
    L = _host_lib()
    qt, rows, k = (int(x) for x in GOLD[f"{name}_meta"])
    raw = np.ascontiguousarray(GOLD[f"{name}_raw"])
    nb = L.z2b_host_tiles_bytes(qt, rows, k)
    assert nb > 0
    tiles = np.zeros(nb, np.uint8)
    assert L.z2b_host_repack(qt, rows, k, raw.ctypes.data, tiles.ctypes.data) == 0
    out = np.zeros((rows, k), np.float32)
    assert L.z2b_host_unpack_tiles(qt, rows, k, tiles.ctypes.data, out.ctypes.data) == 0
    assert np.array_equal(_bits(out), _bits(GOLD[f"{name}_f32"]))


def test_tile_bytes_equal_gguf_bytes():
    """The tile image adds no bytes beyond padding rows to a multiple of 16."""
    L = _host_lib()
    for qt, per_blk, be in [(8, 34, 32), (12, 144, 256), (14, 210, 256), (1, 2, 1)]:
        for rows, k in [(16, 2048), (1408, 2048), (2048, 1408 if qt in (8, 1) else 2048)]:
            assert L.z2b_host_tiles_bytes(qt, rows, k) == ((rows + 15) // 16 * 16) * (k // be) * per_blk


def test_unsupported_shapes_report():
    L = _host_lib()
    assert L.z2b_host_tiles_bytes(12, 16, 1408) == -1     # Q4_K rows must be whole super-blocks
    assert L.z2b_host_tiles_bytes(8, 16, 96) == -1        # Q8_0 tiles need K % 128 == 0


def test_q8_0_encoder_bitexact_with_gguf_py(tmp_path):
    """The synthetic writer's Q8_0 encoder reproduces gguf-py's quantizer byte for byte."""
    import z2b.synth as S
    from gguf import GGUFReader
    p = S.write(str(tmp_path / "q8.gguf"), "tiny", n_layer=1, expert_used=[2])
    r = GGUFReader(p)
    t = next(t for t in r.tensors if t.name == "blk.0.attn_q.weight")
    assert t.tensor_type == Q.Q8_0
    f32 = dequantize(t.data, Q.Q8_0).astype(np.float32)
    # re-quantising the decoded values is a fixed point of gguf-py's Q8_0 quantizer
    again = quantize(f32, Q.Q8_0)
    assert np.array_equal(again.reshape(-1), np.asarray(t.data).reshape(-1))


@pytest.mark.parametrize("qt", [Q.Q4_K, Q.Q6_K])
def test_kquant_encoder_valid(tmp_path, qt):
    """Our Q4_K / Q6_K encoders produce blocks gguf-py decodes close to the source values."""
    import z2b.synth as S
    from gguf import GGUFReader
    preset = "zonos2" if qt == Q.Q4_K else "zonos2_q6k"
    p = S.write(str(tmp_path / "k.gguf"), preset, n_layer=1, expert_used=[4], n_expert=2)
    t = next(t for t in GGUFReader(p).tensors if t.name == "blk.0.attn_q.weight")
    assert t.tensor_type == qt
    x = dequantize(t.data, qt)
    assert np.isfinite(x).all()
    assert 0.018 < float(x.std()) < 0.022            # N(0, 0.02) survives quantisation
