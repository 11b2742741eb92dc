"""DAC decoder, CPU side: the oracle (oracle/dac_o.cpp) pinned against an independent torch
restatement of the published DAC decoder on synthetic files and, with Z2B_REFERENCE_DIR set to a
reference checkout, on the reference's own CI fixture tests/fixtures/dummy-dac.gguf; the window
semantics of dac_decode / dac_decode_window (src/dac.cpp:260-299); the WAV writer
(src/dac.cpp:318-336); and the C ABI's exports."""
from __future__ import annotations

import os
import re
import struct

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle.dac_oracle import DacOracle, tensor_names
from tests.util import cos

REF_FIXTURE = os.path.join(os.environ.get("Z2B_REFERENCE_DIR", ""), "tests", "fixtures", "dummy-dac.gguf")


def _torch_decode(o: DacOracle, codes, a, b, f16=True):
    """Restatement with torch's conv1d / conv_transpose1d (NCL layout, float64 sums). With f16,
    Conv1d operands are rounded to f16 as the reference's im2col path rounds them; the
    transposed convs stay f32 as its f32 GEMM does."""
    arr = dict(zip(tensor_names(o.n_cb, len(o.rates)), o._arrays))
    c = np.asarray(codes, np.int64)
    H = c.shape[0]
    L = b - a
    idx = np.empty((o.n_cb, L), np.int64)
    for j in range(o.n_cb):
        for l in range(L):
            t = a + l
            v = c[t + j, j] if t + j < H else o.pad_id
            idx[j, l] = min(max(v, 0), 1023)
    z = None
    for j in range(o.n_cb):
        tab = torch.from_numpy(arr[f"quant.{j}.table"].reshape(o.cb_size, o.latent))
        zj = tab[torch.from_numpy(idx[j])]
        z = zj if z is None else z + zj
    z = z + torch.from_numpy(arr["quant.bias"])
    x = z.T.unsqueeze(0)                               # [1, latent, L] f32

    def h16(t):
        return t.to(torch.float16).to(torch.float64) if f16 else t.to(torch.float64)

    def conv(x, name, ic, oc, k, dil):
        w = torch.from_numpy(arr[name + ".weight"].reshape(oc, ic, k))
        bias = torch.from_numpy(arr[name + ".bias"])
        y = F.conv1d(h16(x), h16(w), padding=(k // 2) * dil, dilation=dil)
        return y.to(torch.float32) + bias.view(1, -1, 1)

    def snake(x, name):
        al = torch.from_numpy(arr[name + ".alpha"]).view(1, -1, 1)
        iv = torch.from_numpy(arr[name + ".inv_alpha"]).view(1, -1, 1)
        return x + torch.sin(x * al) ** 2 * iv

    C = o.dec_dim
    x = conv(x, "dec.conv_in", o.latent, C, 7, 1)
    for bi, s in enumerate(o.rates):
        p = f"dec.b{bi}"
        y = snake(x, p + ".snake")
        w = torch.from_numpy(arr[p + ".convt.weight"].reshape(C, C // 2, 2 * s))
        x = F.conv_transpose1d(y.to(torch.float64), w.to(torch.float64), stride=s, padding=s // 2)
        x = x.to(torch.float32) + torch.from_numpy(arr[p + ".convt.bias"]).view(1, -1, 1)
        C //= 2
        for r, d in enumerate((1, 3, 9)):
            q = f"{p}.res{r}"
            u = conv(snake(x, q + ".snake1"), q + ".conv1", C, C, 7, d)
            u = conv(snake(u, q + ".snake2"), q + ".conv2", C, C, 1, 1)
            x = x + u
    x = conv(snake(x, "dec.snake_out"), "dec.conv_out", C, 1, 7, 1)
    return torch.tanh(x).reshape(-1).numpy()


def _codes(n, seed, ncb=9):
    return np.random.default_rng(seed).integers(0, 1024, (n, ncb)).astype(np.int32)


@pytest.fixture(scope="module")
def small_dac(tmp_path_factory):
    import z2b.synth as S
    return S.write_dac(str(tmp_path_factory.mktemp("dac") / "dac_small.gguf"), "dac_small", seed=3)


@pytest.fixture(scope="module")
def tiny_dac(tmp_path_factory):
    import z2b.synth as S
    return S.write_dac(str(tmp_path_factory.mktemp("dac") / "dac_tiny.gguf"), "dac_tiny", seed=5)


@pytest.mark.parametrize("which", ["tiny", "small"])
def test_oracle_matches_torch_restatement(which, tiny_dac, small_dac):
    """Structure pinned at f32 precision (both without the f16 operand rounding), then the
    reference's f16 rounding on: the decoder amplifies single f16 rounding flips, so that
    comparison holds to the size of the rounding's own effect (torch with vs without it
    differs by up to 2.1e-2 on the small model)."""
    path = tiny_dac if which == "tiny" else small_dac
    exact, emu = DacOracle(path, f16=False), DacOracle(path, f16=True)
    codes = _codes(14, 11)
    for a, b in ((0, 14), (3, 9), (10, 20)):            # [10, 20) runs past H: pad codes
        got = exact.frames(codes, a, b)
        ref = _torch_decode(exact, codes, a, b, f16=False)
        assert got.shape == ref.shape == ((b - a) * exact.spf,)
        assert np.abs(got - ref).max() < 2e-5, (which, a, b, np.abs(got - ref).max())
        got16 = emu.frames(codes, a, b)
        ref16 = _torch_decode(emu, codes, a, b, f16=True)
        assert np.abs(got16 - ref16).max() < 3e-2 and cos(got16, ref16) > 0.9999
    assert np.abs(got).max() > 0.05                     # not a degenerate all-zero output


@pytest.mark.skipif(not os.environ.get("Z2B_REFERENCE_DIR") or not os.path.exists(REF_FIXTURE),
                    reason="Z2B_REFERENCE_DIR not set to a reference checkout")
def test_oracle_on_reference_fixture():
    """The reference's own CI DAC file (scripts/make-dummy-dac.py output) decodes identically
    through the oracle and the torch restatement."""
    for f16 in (False, True):
        o = DacOracle(REF_FIXTURE, f16=f16)
        assert (o.n_cb, o.cb_size, o.latent, o.dec_dim, o.rates) == (9, 1024, 8, 16, [2, 2])
        codes = _codes(32, 2)
        got = o.decode(codes)
        ref = _torch_decode(o, codes, 0, 32, f16=f16)
        assert got.shape == (32 * 4,)
        assert np.abs(got - ref).max() < 2e-6


def test_window_semantics(small_dac):
    """dac_decode_window: frames [f_lo - Lc, f_hi + Rc) decoded, [f_lo, f_hi) kept; with enough
    context the samples equal the full decode's (src/dac.h:37-44)."""
    o = DacOracle(small_dac)
    codes = _codes(40, 4)
    full = o.decode(codes)
    win = o.decode_window(codes, 12, 20, 16, 16)
    seg = full[12 * o.spf:20 * o.spf]
    assert win.shape == seg.shape
    assert np.abs(win - seg).max() < 1e-5
    assert o.decode_window(codes, 5, 5, 4, 4).size == 0
    assert o.decode(codes, eos=7).shape == (7 * o.spf,)
    with pytest.raises(ValueError):
        o.decode(codes, eos=0)


def test_wav_bytes_layout():
    import z2b.dac as dac
    a = np.array([0.0, 0.5, -0.5, 1.5, -2.0, 1.0 / 65534], np.float32)
    b = dac.wav_bytes(a, 44100)
    assert len(b) == 44 + 2 * a.size
    assert b[:4] == b"RIFF" and b[8:16] == b"WAVEfmt " and b[36:40] == b"data"
    riff, = struct.unpack("<I", b[4:8])
    fmt = struct.unpack("<IHHIIHH", b[16:36])
    assert riff == 36 + 2 * a.size and fmt == (16, 1, 1, 44100, 88200, 2, 16)
    pcm = np.frombuffer(b[44:], "<i2")
    # clamp to [-1, 1], x 32767, round to nearest even
    assert pcm.tolist() == [0, 16384, -16384, 32767, -32767, 0]


def test_capi_exports():
    import z2b.runtime as R
    lib = R.lib()
    hdr = open(os.path.join(os.path.dirname(__file__), "..", "include", "z2b_dac.h")).read()
    names = re.findall(r"\b(z2b_dac_\w+)\s*\(", hdr)
    assert len(names) >= 8
    for n in names:
        assert hasattr(lib, n), n
