"""DAC decoder on the GPU (include/z2b_dac.h) against the CPU oracle (oracle/dac_o.cpp).

Parity bar: the oracle rounds conv operands to f16 as the reference's CPU graph does; the GPU
also runs the transposed convs in f16 and sums in a different order. The decoder amplifies
single f16 rounding flips: on these synthetic models the reference's own f16 rounding moves
the output by up to 1.7e-2 (mean 1.6e-3, cosine 0.999993) against exact f32 inputs. So the
GPU output must reach cosine >= 0.9999, mean |diff| <= 5e-3 and max |diff| <= 5e-2 against
the oracle. Batching is exact: a window decodes bit for bit the same alone or in a batch.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle.dac_oracle import DacOracle
from tests.util import cos

pytestmark = pytest.mark.gpu

COS_MIN, MEAN_MAX, MAX_MAX = 0.9999, 5e-3, 5e-2


def _codes(n, seed, ncb=9):
    return np.random.default_rng(seed).integers(0, 1024, (n, ncb)).astype(np.int32)


def _check(got, ref, what):
    assert got.shape == ref.shape, what
    assert np.isfinite(got).all(), what
    d = np.abs(got.astype(np.float64) - ref)
    c = cos(got, ref)
    print(f"{what}: cos {c:.7f} mean {d.mean():.2e} max {d.max():.2e}")
    assert c >= COS_MIN and d.mean() <= MEAN_MAX and d.max() <= MAX_MAX, (what, c, d.mean(), d.max())


@pytest.fixture(scope="module")
def paths(model_dir):
    import z2b.synth as S
    return {p: S.cached_dac(p, 0, model_dir) for p in ("dac_tiny", "dac_small", "dac44k")}


@pytest.fixture(scope="module")
def dacs(paths):
    import z2b.dac as D
    ds = {p: D.Dac(path) for p, path in paths.items()}
    yield ds
    for d in ds.values():
        d.close()


@pytest.mark.parametrize("preset,n,eos", [("dac_tiny", 33, -1), ("dac_small", 20, -1), ("dac_small", 20, 13),
                                          ("dac44k", 8, -1)])
def test_decode_matches_oracle(dacs, paths, preset, n, eos):
    d = dacs[preset]
    codes = _codes(n, 7 + n)
    got = d.decode(codes, eos)
    ref = DacOracle(paths[preset]).decode(codes, eos)
    _check(got, ref, f"{preset} decode H={n} eos={eos}")
    assert d.last_launches() == 3 + 7 * len(d.hp.rates[:d.hp.n_rates])


def test_hparams(dacs):
    hp = dacs["dac44k"].hp
    assert (hp.n_codebooks, hp.codebook_size, hp.latent_dim, hp.decoder_dim, hp.hop_length) == (9, 1024, 1024, 1536, 512)
    assert list(hp.rates[:hp.n_rates]) == [8, 8, 4, 2] and hp.samples_per_frame == 512


def test_windows_batch_exact_and_match_oracle(dacs, paths):
    """Streaming windows of several streams (the server's block 40 / context 24 cadence, a
    stream start with less left context, a tail with no right context, one past H) decode in
    one batched call bit for bit as they do alone, and match the oracle's dac_decode_window."""
    d = dacs["dac_small"]
    o = DacOracle(paths["dac_small"])
    streams = [_codes(120, s) for s in range(4)]
    wins = [(streams[0], 0, 40, 24, 24), (streams[1], 40, 80, 24, 24), (streams[2], 70, 120, 24, 0),
            (streams[3], 100, 130, 24, 24), (streams[0], 5, 6, 0, 3)]
    batched = d.decode_windows(wins)
    for w, b in zip(wins, batched):
        alone = d.decode_window(*w)
        assert np.array_equal(alone, b), w[1:]
        _check(b, o.decode_window(*w), f"window {w[1:]}")


def test_window_equals_full_decode_slice(dacs):
    """With context at least the decoder's receptive field, and the right context inside the
    generated codes, the window's samples equal the full decode's (src/dac.h:37-44); on the
    GPU bit for bit. (Context frames at or past H read as pad codes, where the full decode
    ends, so a window whose right context runs past H differs near its end, as in the
    reference; such a window is checked against the oracle above.)"""
    d = dacs["dac_small"]
    codes = _codes(96, 3)
    full = d.decode(codes)
    spf = d.spf
    for f_lo, f_hi in ((20, 60), (0, 16), (56, 72)):
        win = d.decode_window(codes, f_lo, f_hi, 24, 24)
        seg = full[f_lo * spf:f_hi * spf]
        diff = np.abs(win - seg).max()
        print(f"window [{f_lo}, {f_hi}) vs full slice: max {diff:.2e}")
        assert diff <= 1e-6


def test_full_size_streaming_batch(dacs, paths):
    """The real decoder's shapes: 16 streams' windows (40 frames, 24 frames of context each
    side) in one call, one of them checked against the oracle."""
    d = dacs["dac44k"]
    streams = [_codes(200, 100 + s) for s in range(16)]
    wins = [(c, 60, 100, 24, 24) for c in streams]
    out = d.decode_windows(wins)
    assert all(x.shape == (40 * 512,) for x in out)
    assert all(np.isfinite(x).all() for x in out)
    ref = DacOracle(paths["dac44k"]).decode_window(*wins[5])
    _check(out[5], ref, "dac44k window 5 of 16")


def test_errors(dacs):
    import z2b.dac as D
    from z2b.runtime import Z2BError
    d = dacs["dac_small"]
    with pytest.raises(Z2BError):
        d.decode(np.zeros((10, 8), np.int32))            # wrong codebook count
    with pytest.raises(Z2BError):
        d.decode(_codes(10, 1), eos=0)                   # no frames to decode
    assert d.decode_window(_codes(10, 1), 5, 5, 4, 4).size == 0
    with pytest.raises(Z2BError):
        D.Dac("/nonexistent/dac.gguf")
    # the context still decodes after the errors
    assert d.decode(_codes(4, 2)).shape == (4 * d.spf,)
