"""Python wrapper of the DAC CPU oracle (oracle/dac_o.cpp) — TEST INFRASTRUCTURE ONLY.

Only tests/ and bench.py's CPU legs use this module, as the checker or as the timed CPU
restatement; the product path never imports it. Weights come straight from gguf-py's
GGUFReader memory maps (third-party gguf 0.19.0), so the checker shares no loading or
layout code with the product library.

Tensor order handed to o_dac_decode: quant.{0..n-1}.table, quant.bias, dec.conv_in.{weight,
bias}; per block b: dec.b{b}.snake.{alpha, inv_alpha}, dec.b{b}.convt.{weight, bias}, then per
residual unit r: snake1.{alpha, inv_alpha}, conv1.{weight, bias}, snake2.{alpha, inv_alpha},
conv2.{weight, bias}; dec.snake_out.{alpha, inv_alpha}, dec.conv_out.{weight, bias}.

The window semantics restate src/dac.cpp:260-299 (dac_decode: latent frames [0, min(eos, H));
dac_decode_window: frames [max(0, f_lo - Lc), f_hi + Rc), samples of [f_lo, f_hi) kept).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_build", "libdaco.so")


class ODac(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("n_cb", "cb_size", "latent", "dec_dim", "n_blocks", "pad_id", "f16")] + \
               [("rates", ctypes.c_int * 8), ("t", ctypes.POINTER(ctypes.c_void_p))]


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            from . import oracle as _o
            _o.build()
        L = ctypes.CDLL(LIB)
        L.o_dac_decode.argtypes = [ctypes.POINTER(ODac), ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_void_p]
        L.o_dac_decode.restype = ctypes.c_int
        _lib = L
    return _lib


def tensor_names(n_cb: int, n_blocks: int) -> list[str]:
    names = [f"quant.{i}.table" for i in range(n_cb)] + ["quant.bias", "dec.conv_in.weight", "dec.conv_in.bias"]
    for b in range(n_blocks):
        p = f"dec.b{b}"
        names += [f"{p}.snake.alpha", f"{p}.snake.inv_alpha", f"{p}.convt.weight", f"{p}.convt.bias"]
        for r in range(3):
            q = f"{p}.res{r}"
            names += [f"{q}.snake1.alpha", f"{q}.snake1.inv_alpha", f"{q}.conv1.weight", f"{q}.conv1.bias",
                      f"{q}.snake2.alpha", f"{q}.snake2.inv_alpha", f"{q}.conv2.weight", f"{q}.conv2.bias"]
    return names + ["dec.snake_out.alpha", "dec.snake_out.inv_alpha", "dec.conv_out.weight", "dec.conv_out.bias"]


class DacOracle:
    """A DAC GGUF read with gguf-py, decoded on the CPU."""

    def __init__(self, path: str, f16: bool = True):
        """f16: round conv operands to f16 as the reference's CPU graph does (False: exact)."""
        from gguf import GGUFReader
        r = GGUFReader(path)

        def u32(key, dflt):
            f = r.fields.get(key)
            return int(f.parts[f.data[0]][0]) if f is not None else dflt

        self.n_cb = u32("dac.n_codebooks", 9)
        self.cb_size = u32("dac.codebook_size", 1024)
        self.latent = u32("dac.latent_dim", 1024)
        self.dec_dim = u32("dac.decoder_dim", 1536)
        self.sample_rate = u32("dac.sample_rate", 44100)
        self.pad_id = u32("dac.audio_pad_id", 1025)
        f = r.fields.get("dac.decoder_rates")
        self.rates = [int(f.parts[i][0]) for i in f.data] if f is not None else [8, 8, 4, 2]
        self.spf = int(np.prod(self.rates))
        by_name = {t.name: t for t in r.tensors}
        self._arrays = []
        for n in tensor_names(self.n_cb, len(self.rates)):
            t = by_name[n]
            a = np.ascontiguousarray(np.asarray(t.data, dtype=np.float32).reshape(-1))
            self._arrays.append(a)
        self._ptrs = (ctypes.c_void_p * len(self._arrays))(*[a.ctypes.data for a in self._arrays])
        self._m = ODac(self.n_cb, self.cb_size, self.latent, self.dec_dim, len(self.rates), self.pad_id, int(f16),
                       (ctypes.c_int * 8)(*(self.rates + [0] * (8 - len(self.rates)))),
                       ctypes.cast(self._ptrs, ctypes.POINTER(ctypes.c_void_p)))

    def frames(self, codes, a: int, b: int) -> np.ndarray:
        """Decoded audio of latent frames [a, b) of raw codes [H, n_cb]."""
        c = np.ascontiguousarray(codes, dtype=np.int32)
        out = np.empty((b - a) * self.spf, np.float32)
        rc = lib().o_dac_decode(ctypes.byref(self._m), c.ctypes.data, c.shape[0], a, b, out.ctypes.data)
        if rc != 0:
            raise ValueError("o_dac_decode: bad arguments")
        return out

    def decode(self, codes, eos: int = -1) -> np.ndarray:
        H = np.asarray(codes).shape[0]
        E = min(eos, H) if eos >= 0 else H
        if E <= 0:
            raise ValueError("no frames to decode")
        return self.frames(codes, 0, E)

    def decode_window(self, codes, f_lo: int, f_hi: int, lc: int, rc: int) -> np.ndarray:
        if f_hi <= f_lo:
            return np.empty(0, np.float32)
        a, b = max(0, f_lo - lc), f_hi + rc
        full = self.frames(codes, a, b)
        return full[(f_lo - a) * self.spf:(f_hi - a) * self.spf]
