"""ctypes binding of include/z2b_dac.h — the Python host mirror of the reference's DAC API.

Names follow src/dac.h: ``Dac`` (dac_load / dac_free), ``Dac.decode`` (dac_decode),
``Dac.decode_window`` (dac_decode_window), ``Dac.decode_windows`` (the batched form: many
streams' windows in one pass) and ``wav_bytes`` (dac_wav_bytes). Decoding runs on the GPU;
every call raises ``Z2BError`` when the library returns an error, with no fallback path.
"""
from __future__ import annotations

import ctypes

import numpy as np

from .runtime import Z2BError, _check, _ptr, lib


class DacHParams(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("n_codebooks", "codebook_size", "latent_dim", "decoder_dim",
                                               "sample_rate", "hop_length", "audio_pad_id", "n_rates")] + \
               [("rates", ctypes.c_int32 * 8), ("samples_per_frame", ctypes.c_int32)]


class DacWindow(ctypes.Structure):
    _fields_ = [("codes", ctypes.c_void_p)] + [(n, ctypes.c_int32) for n in ("H", "f_lo", "f_hi", "Lc", "Rc")]


class Dac:
    """A DAC decoder GGUF loaded onto one GPU (dac_model)."""

    def __init__(self, path: str, device: int = 0):
        h = ctypes.c_void_p()
        _check(lib().z2b_dac_load(path.encode(), device, ctypes.byref(h)))
        self.h = h
        self.hp = DacHParams()
        _check(lib().z2b_dac_get_hparams(self.h, ctypes.byref(self.hp)))
        self.spf = self.hp.samples_per_frame

    def close(self):
        if self.h:
            lib().z2b_dac_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _codes(self, codes):
        c = np.ascontiguousarray(codes, dtype=np.int32)
        if c.ndim != 2:
            raise ValueError("codes must be [H, n_codebooks]")
        return c

    def decode(self, codes, eos: int = -1) -> np.ndarray:
        """dac_decode: raw codes [H, W] -> shear_up -> truncate at eos -> clamp -> decoder -> tanh."""
        c = self._codes(codes)
        H, W = c.shape
        E = min(eos, H) if eos >= 0 else H
        out = np.empty(max(E, 0) * self.spf, np.float32)
        n = ctypes.c_int64()
        _check(lib().z2b_dac_decode(self.h, _ptr(c), H, W, eos, _ptr(out), out.size, ctypes.byref(n)))
        return out[: n.value]

    def decode_window(self, codes, f_lo: int, f_hi: int, lc: int, rc: int) -> np.ndarray:
        """dac_decode_window: the samples of output frames [f_lo, f_hi), decoded with lc / rc frames
        of context on either side."""
        c = self._codes(codes)
        out = np.empty(max(f_hi - f_lo, 0) * self.spf, np.float32)
        n = ctypes.c_int64()
        _check(lib().z2b_dac_decode_window(self.h, _ptr(c), c.shape[0], f_lo, f_hi, lc, rc, _ptr(out), out.size,
                                           ctypes.byref(n)))
        return out[: n.value]

    def decode_windows(self, windows) -> list[np.ndarray]:
        """Batched decode_window: windows = [(codes, f_lo, f_hi, lc, rc), ...], one pass on the GPU."""
        arrs = [self._codes(w[0]) for w in windows]
        ws = (DacWindow * max(len(windows), 1))()
        total = 0
        for i, (w, a) in enumerate(zip(windows, arrs)):
            ws[i] = DacWindow(a.ctypes.data, a.shape[0], w[1], w[2], w[3], w[4])
            total += max(w[2] - w[1], 0) * self.spf
        out = np.empty(max(total, 1), np.float32)
        ns = np.zeros(max(len(windows), 1), np.int64)
        _check(lib().z2b_dac_decode_windows(self.h, ws, len(windows), _ptr(out), total, _ptr(ns)))
        res, o = [], 0
        for i in range(len(windows)):
            res.append(out[o: o + ns[i]])
            o += ns[i]
        return res

    def last_launches(self) -> int:
        return int(lib().z2b_dac_last_launches(self.h))

    def stream(self) -> int:
        """The decoder's CUDA stream handle (for events around its calls)."""
        return int(lib().z2b_dac_stream(self.h) or 0)

    def conv_flops(self, latent_frames: int) -> int:
        """Algorithmic multiply-add FLOPs (x2) of the decoder's convolutions over a window of
        latent_frames (valid channels only: conv_in, each block's transposed conv and residual
        units, conv_out)."""
        hp = self.hp
        rates = list(hp.rates[:hp.n_rates])
        L, C = latent_frames, hp.decoder_dim
        f = 2 * L * 7 * hp.latent_dim * C
        for s in rates:
            co = C // 2
            f += 2 * (L * s) * (2 * C) * co
            L, C = L * s, co
            f += 3 * (2 * L * 7 * C * C + 2 * L * C * C)
        return f + 2 * L * 7 * C


def wav_bytes(audio, sample_rate: int = 44100) -> bytes:
    """dac_wav_bytes: 16-bit PCM mono RIFF/WAVE image of audio."""
    a = np.ascontiguousarray(audio, dtype=np.float32)
    size = lib().z2b_dac_wav_bytes(_ptr(a), a.size, sample_rate, None, 0)
    if size < 0:
        raise Z2BError(1, "bad audio buffer")
    buf = np.empty(size, np.uint8)
    lib().z2b_dac_wav_bytes(_ptr(a), a.size, sample_rate, _ptr(buf), size)
    return buf.tobytes()
