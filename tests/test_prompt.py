"""TTS prompt builder (z2b_build_prompt, host code in libz2b.so) against the CPU restatement
of the reference's zonos2_build_prompt (oracle/prompt_oracle.py): bit-exact rows and speaker
slot position over texts (ASCII, multi-byte UTF-8, empty) and every option the reference's
CLI and server set (speaker slot with clean / noisy background and accurate mode on / off,
speaking rate, quality buckets, no silence), plus the sizing call and the error paths."""
from __future__ import annotations

import ctypes
import itertools

import numpy as np
import pytest

from oracle.prompt_oracle import build_prompt as oracle_prompt


def _hp(ncb=9, tv=519, pad=1025):
    import z2b.runtime as R
    hp = R.HParams()
    hp.n_codebooks, hp.text_vocab, hp.audio_pad_id = ncb, tv, pad
    return hp


TEXTS = ["Hello, world.", "", "ünïcödé — 音声合成 ✓", "a" * 300]


@pytest.mark.parametrize("text", TEXTS)
def test_default_prompt_matches_reference(text):
    import z2b.runtime as R
    got, sp = R.build_prompt(_hp(), text)
    ref, rsp = oracle_prompt(text.encode())
    assert sp == rsp == -1
    assert got.tolist() == ref
    # BOS, bytes, EOS, then 17 silence frames; one default quality row before them
    assert got.shape == (1 + 2 + len(text.encode()) + 17, 10)


def test_options_match_reference():
    import z2b.runtime as R
    hp = _hp()
    text = "Synthesise this."
    for slot, clean, acc, rate, qual, sil in itertools.product(
            (False, True), (True, False), (True, False), (-1, 0, 7), (None, [0, -1, 11], [-1] * 6, [1, 2, 3, 4, 5, 6]),
            (True, False)):
        kw = dict(add_speaker_slot=slot, clean_speaker_background=clean, accurate_mode=acc,
                  speaking_rate_bucket=rate, quality_buckets=qual, prepend_silence=sil)
        got, sp = R.build_prompt(hp, text, **kw)
        ref, rsp = oracle_prompt(text.encode(), **kw)
        assert sp == rsp and got.tolist() == ref, kw


@pytest.mark.parametrize("ncb,tv,pad", [(9, 519, 1025), (4, 600, 77), (12, 519, 1025)])
def test_other_shapes(ncb, tv, pad):
    """Fewer codebooks truncate the sheared silence, more leave the extra codebooks padded."""
    import z2b.runtime as R
    got, _ = R.build_prompt(_hp(ncb, tv, pad), "abc", add_speaker_slot=True)
    ref, _ = oracle_prompt(b"abc", n_codebooks=ncb, text_vocab=tv, audio_pad=pad, add_speaker_slot=True)
    assert got.tolist() == ref


def test_layout_invariants():
    """With the real vocabulary the byte ids end where the conditioning ids begin."""
    import z2b.runtime as R
    got, sp = R.build_prompt(_hp(), bytes([0, 255]), add_speaker_slot=True, speaking_rate_bucket=0)
    text_col = got[:, 9]
    assert sp == 0 and text_col[0] == 519                      # speaker slot: text pad
    assert text_col[1] == 448 + 8 + 60 and text_col[2] == 448 + 8 + 60 + 2   # clean bg, accurate
    assert text_col[3] == 448                                  # speaking rate bucket 0
    bos = list(text_col).index(2)
    assert text_col[bos + 1] == 192 and text_col[bos + 2] == 447 and text_col[bos + 3] == 3


def test_sizing_and_errors():
    import z2b.runtime as R
    L = R.lib()
    hp = _hp()
    o = R.PromptOptions()
    L.z2b_prompt_options_default(ctypes.byref(o))
    n, sp = ctypes.c_int(), ctypes.c_int()
    assert L.z2b_build_prompt(ctypes.byref(hp), b"hi", 2, ctypes.byref(o), None, 0, ctypes.byref(n),
                              ctypes.byref(sp)) == 0
    assert n.value == 1 + 2 + 2 + 17
    small = np.zeros((n.value - 1, 10), np.int32)
    assert L.z2b_build_prompt(ctypes.byref(hp), b"hi", 2, ctypes.byref(o), small.ctypes.data, n.value - 1,
                              ctypes.byref(n), ctypes.byref(sp)) == 1
    assert not small.any()                                     # nothing written
    o.n_quality = 17
    assert L.z2b_build_prompt(ctypes.byref(hp), b"hi", 2, ctypes.byref(o), None, 0, ctypes.byref(n),
                              ctypes.byref(sp)) == 1
    assert b"n_quality" in L.z2b_last_error()
