"""Emotion control (zonos2.cpp_b200/emotion.py) against a literal restatement of the reference's
loops (src/zonos2-emotion.cpp:60-205, 330-358) on synthetic directions directories in all three
spaces (proj, raw, lda) with per-speaker calibration, the error paths, and, with
Z2B_REFERENCE_DIR set to a reference checkout, the reference's own emotion_directions."""
from __future__ import annotations

import json
import math
import os

import numpy as np
import pytest

REF_DIR = os.path.join(os.environ.get("Z2B_REFERENCE_DIR", ""), "emotion_directions")


def _write_dir(path, space, dim, input_dim, seed=0, calibration=True):
    g = np.random.default_rng(seed)
    os.makedirs(path, exist_ok=True)
    dirs = {}
    for name, kind in (("happy", "named"), ("sad", "named"), ("calm", "named"), ("valence", "axis"),
                       ("arousal", "axis")):
        np.save(os.path.join(path, f"{name}.npy"), (g.standard_normal(dim) * 0.05).astype(np.float32))
        dirs[name] = {"file": f"{name}.npy", "kind": kind}
    man = {"dim": dim, "input_dim": input_dim, "space": space, "directions": dirs}
    if space == "lda":
        np.save(os.path.join(path, "w.npy"), (g.standard_normal((dim, input_dim)) * 0.3).astype(np.float32))
        np.save(os.path.join(path, "b.npy"), (g.standard_normal(dim) * 0.1).astype(np.float32))
        np.save(os.path.join(path, "p.npy"), (g.standard_normal((input_dim, dim)) * 0.3).astype(np.float32))
        man["lda"] = {"weight": "w.npy", "bias": "b.npy", "pinv": "p.npy"}
    with open(os.path.join(path, "manifest.json"), "w") as f:
        json.dump(man, f)
    if calibration:
        with open(os.path.join(path, "calibration.json"), "w") as f:
            json.dump({"global_default": 2.0, "default": {"happy": 3.0, "valence": 1.5},
                       "by_speaker": {"spk_a": {"happy": 4.0, "sad": 0.5}}}, f)
    return path


def _ref_apply(d, speaker, sliders, valence, arousal, strength, key):
    """The reference's loops, element by element in f32 with f64 norms and products."""
    f32 = np.float32

    def cal(name):
        if key and name in d.cal_by_speaker.get(key, {}):
            return f32(d.cal_by_speaker[key][name])
        return f32(d.cal_default.get(name, d.cal_global))

    delta = [f32(0)] * d.dim
    asked = False
    for name in sorted(sliders):
        w0 = f32(sliders[name])
        if w0 == 0:
            continue
        vec = d.named.get(name, d.axes.get(name))
        w = f32(w0 * cal(name))
        delta = [f32(delta[i] + f32(w * vec[i])) for i in range(d.dim)]
        asked = True
    for name, w0 in (("valence", f32(valence)), ("arousal", f32(arousal))):
        if w0 == 0:
            continue
        w = f32(w0 * cal(name))
        delta = [f32(delta[i] + f32(w * d.axes[name][i])) for i in range(d.dim)]
        asked = True
    spk = [f32(x) for x in speaker]
    if not asked or f32(strength) == 0:
        return np.array(spk, np.float32), None
    if f32(strength) != 1:
        delta = [f32(x * f32(strength)) for x in delta]

    def norm(v):
        return f32(math.sqrt(sum(float(x) * float(x) for x in v)))

    def rescale(v, target):
        cur = norm(v)
        if cur <= f32(1e-8):
            return v
        s = f32(target / cur)
        return [f32(x * s) for x in v]

    if d.space == "proj":
        return np.array(spk, np.float32), np.array(delta, np.float32)
    if d.space == "raw":
        t = norm(spk)
        return np.array(rescale([f32(spk[i] + delta[i]) for i in range(len(spk))], t), np.float32), None
    W, b, P = d.lda_weight, d.lda_bias, d.lda_pinv
    lda = [f32(float(b[r]) + sum(float(W[r, c]) * float(spk[c]) for c in range(d.input_dim))) for r in range(d.dim)]
    t = norm(lda)
    lda = rescale([f32(lda[r] + delta[r]) for r in range(d.dim)], t)
    raw = [f32(sum(float(P[i, r]) * float(f32(lda[r] - b[r])) for r in range(d.dim))) for i in range(d.input_dim)]
    return np.array(raw, np.float32), None


CASES = [({"happy": 1.0}, 0.0, 0.0, 1.0, ""), ({"happy": 0.5, "sad": -0.25}, 0.3, -0.7, 0.8, "spk_a"),
         ({"calm": 1.0, "happy": 0.0}, 0.0, 0.4, 1.0, "nobody"), ({}, 0.0, 0.0, 1.0, ""),
         ({"sad": 1.0}, 0.0, 0.0, 0.0, "")]


@pytest.mark.parametrize("space,dim,input_dim", [("proj", 32, 32), ("raw", 16, 16), ("lda", 6, 16)])
def test_apply_matches_reference_loops(tmp_path, space, dim, input_dim):
    import z2b.emotion as E
    d = E.load(_write_dir(str(tmp_path / space), space, dim, input_dim, seed=dim))
    spk = np.random.default_rng(1).standard_normal(input_dim).astype(np.float32)
    for sliders, val, aro, strength, key in CASES:
        got_spk, got_delta = E.apply(d, spk, sliders, val, aro, strength, key)
        ref_spk, ref_delta = _ref_apply(d, spk, sliders, val, aro, strength, key)
        assert (got_delta is None) == (ref_delta is None), (space, sliders)
        if ref_delta is not None:
            assert np.abs(got_delta - ref_delta).max() <= 1e-6 * (1 + np.abs(ref_delta).max())
        assert np.abs(got_spk - ref_spk).max() <= 2e-6 * (1 + np.abs(ref_spk).max()), (space, sliders)
    if space == "raw":                                  # the speaker keeps its norm
        s2, _ = E.apply(d, spk, {"happy": 1.0})
        assert abs(np.linalg.norm(s2) - np.linalg.norm(spk)) < 1e-5


def test_calibration_fallbacks(tmp_path):
    import z2b.emotion as E
    d = E.load(_write_dir(str(tmp_path / "c"), "proj", 8, 8))
    assert d.strength("spk_a", "happy") == 4.0          # the speaker's own entry
    assert d.strength("spk_a", "calm") == 2.0           # not there: global default
    assert d.strength("", "happy") == 3.0               # the default table
    nd = E.load(_write_dir(str(tmp_path / "n"), "proj", 8, 8, calibration=False))
    assert not nd.has_calibration and nd.strength("x", "happy") == 1.0


def test_errors(tmp_path):
    import z2b.emotion as E
    d = E.load(_write_dir(str(tmp_path / "e"), "raw", 8, 8))
    with pytest.raises(E.EmotionError):
        E.apply(d, np.ones(8, np.float32), {"furious": 1.0})
    with pytest.raises(E.EmotionError):
        E.apply(d, np.ones(7, np.float32), {"happy": 1.0})      # wrong speaker dim
    with pytest.raises(E.EmotionError):
        E.load(str(tmp_path / "missing"))
    bad = _write_dir(str(tmp_path / "bad"), "raw", 8, 8)
    with open(os.path.join(bad, "manifest.json"), "w") as f:
        json.dump({"dim": 9, "space": "raw", "directions": {"happy": {"file": "happy.npy"}}}, f)
    with pytest.raises(E.EmotionError):
        E.load(bad)                                             # 8-wide vector, dim 9


@pytest.mark.skipif(not os.environ.get("Z2B_REFERENCE_DIR") or not os.path.isdir(REF_DIR),
                    reason="Z2B_REFERENCE_DIR not set to a reference checkout")
def test_reference_directions():
    import z2b.emotion as E
    d = E.load(REF_DIR)
    assert d.space == "proj" and d.dim == 2048
    assert sorted(d.named) == ["angry", "happy", "sad", "surprised"] and sorted(d.axes) == ["arousal", "valence"]
    assert d.strength("", "surprised") == 4.0 and d.strength("", "happy") == 3.0
    spk = np.ones(2048, np.float32)
    s, dl = E.apply(d, spk, {"happy": 1.0})
    assert np.array_equal(s, spk) and np.array_equal(dl, (np.float32(3.0) * d.named["happy"]).astype(np.float32))
