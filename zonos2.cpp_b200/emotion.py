"""Emotion control: a request's emotion sliders turned into what the prefill injects.

Replaces src/zonos2-emotion.cpp (zonos2_emotion_load / zonos2_emotion_apply). A directions
directory holds manifest.json (dim, input_dim, space, one .npy file per direction: named
emotions and the valence / arousal axes), an optional calibration.json (per-speaker and
default strengths) and, for the "lda" space, the LDA weight / bias / pseudo-inverse.

A request's delta is the sum over its sliders of weight x calibrated strength x direction
(sliders in name order, then valence, then arousal), times the overall strength. What it
changes depends on the space:
  - "proj": nothing in the speaker vector; the delta [n_embd] is added to the projected
    speaker row in the prefill (z2b_slot_prefill_spk's spk_emotion_delta), and it is what
    emotion CFG guides against;
  - "raw": the speaker vector plus the delta, rescaled to the speaker's norm;
  - "lda": the speaker vector projected to LDA space, plus the delta, rescaled to the
    projection's norm, mapped back through the pseudo-inverse.
Arithmetic follows the reference: f32 element updates, norms and matrix products summed in
f64 and rounded to f32.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field

import numpy as np


class EmotionError(ValueError):
    pass


@dataclass
class EmotionDirections:
    dim: int = 0
    input_dim: int = 0
    space: str = "raw"
    ref_base_norm: float | None = None
    named: dict = field(default_factory=dict)        # name -> [dim] f32, manifest order
    axes: dict = field(default_factory=dict)         # valence / arousal / kind "axis"
    cal_by_speaker: dict = field(default_factory=dict)
    cal_default: dict = field(default_factory=dict)
    cal_global: float = 1.0
    has_calibration: bool = False
    lda_weight: np.ndarray | None = None             # [dim][input_dim]
    lda_bias: np.ndarray | None = None               # [dim]
    lda_pinv: np.ndarray | None = None               # [input_dim][dim]

    def available(self) -> bool:
        return self.dim > 0 and bool(self.named or self.axes)

    def strength(self, speaker_key: str, emotion: str) -> float:
        """Calibrated strength: the speaker's own entry, else the default's, else the global."""
        if speaker_key and emotion in self.cal_by_speaker.get(speaker_key, {}):
            return float(self.cal_by_speaker[speaker_key][emotion])
        return float(self.cal_default.get(emotion, self.cal_global))


def _vector(path: str, dim: int, name: str) -> np.ndarray:
    try:
        v = np.load(path).astype(np.float32).reshape(-1)
    except Exception as e:
        raise EmotionError(f"failed to load emotion direction '{name}' from {path}") from e
    if v.size != dim:
        raise EmotionError(f"emotion direction '{name}' has dim {v.size}, expected {dim}")
    return v


def load(directory: str) -> EmotionDirections:
    """Read a directions directory (zonos2_emotion_load); raises EmotionError when it is missing
    or invalid."""
    mpath = os.path.join(directory, "manifest.json")
    try:
        with open(mpath) as f:
            man = json.load(f)
    except (OSError, ValueError) as e:
        raise EmotionError(f"no valid emotion directions manifest at {mpath}") from e
    if not isinstance(man, dict):
        raise EmotionError(f"invalid emotion directions manifest at {mpath}")
    d = EmotionDirections(dim=int(man.get("dim", 0)))
    d.input_dim = int(man.get("input_dim", d.dim))
    d.space = str(man.get("space", "raw"))
    if isinstance(man.get("ref_base_norm"), (int, float)):
        d.ref_base_norm = float(man["ref_base_norm"])
    if d.dim <= 0 or d.input_dim <= 0:
        raise EmotionError("emotion manifest has invalid dimensions")
    dirs = man.get("directions")
    if not isinstance(dirs, dict):
        raise EmotionError("emotion manifest has no directions object")
    for name, entry in dirs.items():
        if not isinstance(entry, dict) or not isinstance(entry.get("file"), str):
            raise EmotionError(f"emotion direction '{name}' is missing a file")
        v = _vector(os.path.join(directory, entry["file"]), d.dim, name)
        if entry.get("kind") == "axis" or name in ("valence", "arousal"):
            d.axes[name] = v
        else:
            d.named[name] = v
    if d.space == "lda":
        lda = man.get("lda", {})
        if not isinstance(lda, dict) or not all(k in lda for k in ("weight", "bias", "pinv")):
            raise EmotionError("LDA emotion directions require lda.weight, lda.bias, and lda.pinv")
        d.lda_weight = np.load(os.path.join(directory, lda["weight"])).astype(np.float32)
        d.lda_bias = np.load(os.path.join(directory, lda["bias"])).astype(np.float32).reshape(-1)
        d.lda_pinv = np.load(os.path.join(directory, lda["pinv"])).astype(np.float32)
        if d.lda_weight.ndim != 2 or d.lda_pinv.ndim != 2:
            raise EmotionError("emotion LDA matrices must be 2-D")
    cpath = os.path.join(directory, "calibration.json")
    if os.path.exists(cpath):
        try:
            with open(cpath) as f:
                cal = json.load(f)
        except ValueError:
            cal = None                                   # an invalid calibration is ignored
        if isinstance(cal, dict):
            d.has_calibration = True
            d.cal_global = float(cal.get("global_default", 1.0))
            d.cal_default = {k: float(v) for k, v in (cal.get("default") or {}).items()
                             if isinstance(v, (int, float))}
            for spk, table in (cal.get("by_speaker") or {}).items():
                if isinstance(table, dict):
                    d.cal_by_speaker[spk] = {k: float(v) for k, v in table.items() if isinstance(v, (int, float))}
    if not d.available():
        raise EmotionError("emotion directions hold no direction")
    return d


def _norm(v: np.ndarray) -> np.float32:
    return np.float32(np.sqrt(np.sum(v.astype(np.float64) ** 2)))


def _rescale(v: np.ndarray, target: np.float32) -> np.ndarray:
    cur = _norm(v)
    if cur <= np.float32(1e-8):
        return v
    return (v * np.float32(target / cur)).astype(np.float32)


def delta(d: EmotionDirections, sliders: dict | None = None, valence: float = 0.0, arousal: float = 0.0,
          strength: float = 1.0, speaker_key: str = "") -> np.ndarray | None:
    """The request's combined direction [dim] (f32), or None when it asks for nothing."""
    out = np.zeros(d.dim, np.float32)
    asked = False
    for name in sorted(sliders or {}):
        w0 = np.float32(sliders[name])
        if w0 == 0:
            continue
        vec = d.named.get(name, d.axes.get(name))
        if vec is None:
            raise EmotionError(f"unknown emotion direction '{name}' (available: "
                               f"{', '.join(sorted(d.named) + sorted(d.axes))})")
        out = (out + np.float32(w0 * np.float32(d.strength(speaker_key, name))) * vec).astype(np.float32)
        asked = True
    for name, w0 in (("valence", valence), ("arousal", arousal)):
        w0 = np.float32(w0)
        if w0 == 0:
            continue
        if name not in d.axes:
            raise EmotionError(f"emotion axis '{name}' is not available")
        out = (out + np.float32(w0 * np.float32(d.strength(speaker_key, name))) * d.axes[name]).astype(np.float32)
        asked = True
    if not asked:
        return None
    if np.float32(strength) != 1:
        out = (out * np.float32(strength)).astype(np.float32)
    return out


def apply(d: EmotionDirections, speaker, sliders: dict | None = None, valence: float = 0.0, arousal: float = 0.0,
          strength: float = 1.0, speaker_key: str = ""):
    """zonos2_emotion_apply: (speaker vector to inject, hidden delta or None)."""
    spk = np.asarray(speaker, np.float32).reshape(-1).copy()
    if not d.available():
        raise EmotionError("emotion control requested but no emotion directions are loaded")
    if spk.size == 0:
        return spk, None
    dl = delta(d, sliders, valence, arousal, strength, speaker_key)
    if dl is None or np.float32(strength) == 0:
        return spk, None
    if d.space == "proj":
        return spk, dl
    if d.space == "raw":
        if spk.size != d.input_dim or d.dim != d.input_dim:
            raise EmotionError(f"raw emotion directions require speaker dim {d.input_dim}, got {spk.size}")
        return _rescale((spk + dl).astype(np.float32), _norm(spk)), None
    if d.space == "lda":
        W, b, P = d.lda_weight, d.lda_bias, d.lda_pinv
        if spk.size != d.input_dim:
            raise EmotionError(f"LDA emotion directions require speaker dim {d.input_dim}, got {spk.size}")
        if W.shape != (d.dim, d.input_dim) or P.shape != (d.input_dim, d.dim) or b.size != d.dim:
            raise EmotionError("LDA emotion matrix shapes do not match manifest dimensions")
        lda = (b.astype(np.float64) + W.astype(np.float64) @ spk.astype(np.float64)).astype(np.float32)
        target = _norm(lda)
        lda = _rescale((lda + dl).astype(np.float32), target)
        centered = (lda - b).astype(np.float32)
        return (P.astype(np.float64) @ centered.astype(np.float64)).astype(np.float32), None
    raise EmotionError(f"unsupported emotion direction space '{d.space}'")
