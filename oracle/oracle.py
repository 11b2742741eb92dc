"""Python wrapper of the CPU oracle (oracle/z2o.cpp) — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference legs use
this module, as the checker or as the timed CPU restatement; the product path never
imports it. Weights are handed to the oracle straight from gguf-py's GGUFReader
memory maps (third-party gguf 0.19.0), so the checker shares no parsing, repacking or
dequantisation code with the product library.

Parity of the graph arithmetic is unpinned (see z2o.cpp): the reference's ggml
submodule is absent, so the oracle restates src/zonos2-graph.cpp and the sampler
rather than running them. Dequantisation is pinned bit-exactly to gguf-py.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_build", "libz2o.so")
EXACT, GGML_EMU = 0, 1


def build():
    """Compile the oracle (make -f oracle/Makefile)."""
    subprocess.run(["make", "-s", "-f", os.path.join(HERE, "Makefile")], check=True)
    return LIB


class OTensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("type", ctypes.c_uint32), ("ne0", ctypes.c_int64),
                ("ne1", ctypes.c_int64), ("ne2", ctypes.c_int64)]


class OHparams(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("n_layer", "n_embd", "head_dim", "n_head", "n_head_kv", "n_ff",
                                            "n_codebooks", "audio_vocab", "text_vocab", "eoa_id", "n_ctx_train")] + \
               [(n, ctypes.c_float) for n in ("rope_base", "rms_eps", "qk_eps", "softcap")]


LAYER_NAMES = ["attn_norm.weight", "ffn_norm.weight", "attn_q.weight", "attn_k.weight", "attn_v.weight",
               "attn_output.weight", "attn_temp", "attn_gate.weight", "ffn_up.weight", "ffn_gate.weight",
               "ffn_down.weight", "ffn_gate_exps.weight", "ffn_up_exps.weight", "ffn_down_exps.weight",
               "router_down.weight", "router_down.bias", "router_mlp0.weight", "router_mlp0.bias",
               "router_mlp2.weight", "router_mlp2.bias", "router_mlp4.weight", "router_norm.weight", "router_bias",
               "router_eda_scale"]

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = ctypes.CDLL(LIB)
        P, I, V = ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p
        L.o_model_new.argtypes = [ctypes.POINTER(OHparams), V, V, V, V, V, V, I]
        L.o_model_new.restype = P
        L.o_model_free.argtypes = [P]
        L.o_model_set_mode.argtypes = [P, I]
        L.o_model_set_mask.argtypes = [P, I, V, I]
        L.o_ctx_new.argtypes = [P, I, I]
        L.o_ctx_new.restype = P
        L.o_ctx_free.argtypes = [P]
        L.o_prefill.argtypes = [P, I, V, I, V]
        L.o_model_set_spk.argtypes = [P, V]
        L.o_spk_row.argtypes = [P, V, V, V]
        L.o_prefill_spk.argtypes = [P, I, V, I, V, I, V, V]
        L.o_logits.argtypes = [P, V, I, V, I, V, V]
        L.o_step.argtypes = [P, V, V, V, I, V]
        L.o_last_sel.argtypes = [P, V, I]
        L.o_ctx_fake_fill.argtypes = [P, I, I, ctypes.c_uint32]
        L.o_ctx_hash_fill.argtypes = [P, I, I, ctypes.c_uint32]
        L.o_router.argtypes = [P, I, V, V, I, V, V, V]
        L.o_dequant.argtypes = [ctypes.c_uint32, V, ctypes.c_int64, V]
        L.o_sampler_new.argtypes = [ctypes.c_float, I, ctypes.c_float, ctypes.c_float, ctypes.c_float, I, I,
                                    ctypes.c_uint32, I, I]
        L.o_sampler_new.restype = P
        L.o_sampler_free.argtypes = [P]
        L.o_sample_frame.argtypes = [P, V, I, I, V]
        _lib = L
    return _lib


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def dequant(qtype: int, raw: np.ndarray, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    raw = np.ascontiguousarray(raw)
    lib().o_dequant(qtype, _ptr(raw), n, _ptr(out))
    return out


class Model:
    """zonos2 GGUF restated on the CPU; tensors stay in gguf-py's memory maps."""

    def __init__(self, path: str, mode: int = EXACT):
        from gguf import GGUFReader
        r = GGUFReader(path)
        self.reader = r
        f = {k: v for k, v in r.fields.items()}

        def kv(key):
            fld = f[key]
            return fld.parts[fld.data[0]][0]

        self.t = {t.name: t for t in r.tensors}
        hp = OHparams()
        hp.n_layer = int(kv("zonos2.block_count")); hp.n_embd = int(kv("zonos2.embedding_length"))
        hp.head_dim = int(kv("zonos2.head_dim")); hp.n_head = int(kv("zonos2.attention.head_count"))
        hp.n_head_kv = int(kv("zonos2.attention.head_count_kv")); hp.n_ff = int(kv("zonos2.feed_forward_length"))
        hp.n_codebooks = int(kv("zonos2.n_codebooks")); hp.audio_vocab = int(kv("zonos2.audio_vocab"))
        hp.text_vocab = int(kv("zonos2.text_vocab")); hp.eoa_id = int(kv("zonos2.eoa_id"))
        hp.n_ctx_train = int(kv("zonos2.context_length"))
        hp.rope_base = float(kv("zonos2.rope.freq_base")); hp.rms_eps = float(kv("zonos2.attention.layer_norm_rms_epsilon"))
        hp.qk_eps = float(kv("zonos2.attention.qk_norm_epsilon")); hp.softcap = float(kv("zonos2.logit_softcap"))
        fld = f["zonos2.expert_used_count_per_layer"]
        self.expert_used = np.array([int(fld.parts[i][0]) for i in fld.data], np.int32)
        self.hp = hp

        def ot(name):
            t = self.t.get(name)
            if t is None:
                return OTensor(None, 0, 0, 0, 0)
            shape = [int(x) for x in t.shape] + [1, 1]
            return OTensor(t.data.ctypes.data, int(t.tensor_type), shape[0], shape[1], shape[2])

        self._audio = (OTensor * hp.n_codebooks)(*[ot(f"audio_embd.{i}.weight") for i in range(hp.n_codebooks)])
        self._text, self._on, self._out = ot("text_embd.weight"), ot("output_norm.weight"), ot("output.weight")
        n = hp.n_layer * len(LAYER_NAMES)
        self._layers = (OTensor * n)(*[ot(f"blk.{L}.{nm}") for L in range(hp.n_layer) for nm in LAYER_NAMES])
        self.h = lib().o_model_new(ctypes.byref(hp), ctypes.cast(self._audio, ctypes.c_void_p),
                                   ctypes.addressof(self._text), ctypes.addressof(self._on),
                                   ctypes.addressof(self._out), ctypes.cast(self._layers, ctypes.c_void_p),
                                   _ptr(self.expert_used), mode)
        spk_names = ["spk_lda.weight", "spk_lda.bias", "spk_proj.weight", "spk_proj.bias"]
        self.has_spk = all(nm in self.t for nm in spk_names)
        if self.has_spk:
            self._spk = (OTensor * 4)(*[ot(nm) for nm in spk_names])
            lib().o_model_set_spk(self.h, ctypes.cast(self._spk, ctypes.c_void_p))

    def set_mode(self, mode: int):
        lib().o_model_set_mode(self.h, mode)

    def logits(self, ids, spk=None, spk_pos: int = 0, spk_emotion_delta=None) -> np.ndarray:
        """zonos2_logits: every row's logits [n, ncb, av] of one sequence from position 0."""
        ids = np.ascontiguousarray(ids, np.int32)
        n = ids.shape[0]
        out = np.empty((n, self.hp.n_codebooks, self.hp.audio_vocab), np.float32)
        sp = None if spk is None else np.ascontiguousarray(spk, np.float32)
        dl = None if spk_emotion_delta is None else np.ascontiguousarray(spk_emotion_delta, np.float32)
        rc = lib().o_logits(self.h, _ptr(ids), n, _ptr(sp) if sp is not None else None, int(spk_pos),
                            _ptr(dl) if dl is not None else None, _ptr(out))
        assert rc == 0
        return out

    def spk_row(self, spk, delta=None) -> np.ndarray:
        """The projected speaker row [n_embd] that replaces a prompt row's embedding."""
        spk = np.ascontiguousarray(spk, np.float32)
        delta = None if delta is None else np.ascontiguousarray(delta, np.float32)
        out = np.empty(self.hp.n_embd, np.float32)
        assert lib().o_spk_row(self.h, _ptr(spk), _ptr(delta) if delta is not None else None, _ptr(out)) == 0
        return out

    def router(self, layer: int, res, state_in=None):
        """The router of MoE layer `layer` on residual rows res [n, d] (ffn_norm applied
        inside) and the previous MoE layer's state [n, rd] (None for the first MoE layer):
        returns (sel [n, k], weights [n, k], new state [n, rd])."""
        res = np.ascontiguousarray(res, np.float32)
        n = res.shape[0]
        k = int(self.expert_used[layer])
        rd = int(self.t[f"blk.{layer}.router_down.weight"].shape[1])
        sel = np.empty((n, k), np.int32)
        w = np.empty((n, k), np.float32)
        st = np.empty((n, rd), np.float32)
        si = None if state_in is None else np.ascontiguousarray(state_in, np.float32)
        rc = lib().o_router(self.h, layer, _ptr(res), _ptr(si) if si is not None else None, n, _ptr(sel), _ptr(w),
                            _ptr(st))
        assert rc == 0
        return sel, w, st

    def set_expert_mask(self, keep: dict[int, list[int]]):
        for L in range(self.hp.n_layer):
            if L in keep:
                E = int(self.t[f"blk.{L}.ffn_up_exps.weight"].shape[2])
                m = np.full(E, -np.inf, np.float32)
                m[list(keep[L])] = 0.0
                lib().o_model_set_mask(self.h, L, _ptr(m), E)
            else:
                lib().o_model_set_mask(self.h, L, None, 0)

    def __del__(self):
        if getattr(self, "h", None):
            lib().o_model_free(self.h)
            self.h = None


class Ctx:
    """zonos2_batch_ctx restated: per-slot contiguous f16 KV band of `cap` rows."""

    def __init__(self, model: Model, n_slots: int, cap: int):
        self.model = model
        self.h = lib().o_ctx_new(model.h, n_slots, cap)
        self.nout = model.hp.n_codebooks * model.hp.audio_vocab

    def prefill(self, slot: int, ids, spk=None, spk_pos: int = 0, spk_emotion_delta=None) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.empty(self.nout, np.float32)
        if spk is None:
            rc = lib().o_prefill(self.h, slot, _ptr(ids), ids.shape[0], _ptr(out))
        else:
            spk = np.ascontiguousarray(spk, np.float32)
            dl = None if spk_emotion_delta is None else np.ascontiguousarray(spk_emotion_delta, np.float32)
            rc = lib().o_prefill_spk(self.h, slot, _ptr(ids), ids.shape[0], _ptr(spk), int(spk_pos),
                                     _ptr(dl) if dl is not None else None, _ptr(out))
        assert rc == 0
        return out.reshape(self.model.hp.n_codebooks, -1)

    def step(self, slots, n_past, ids) -> np.ndarray:
        slots = np.ascontiguousarray(slots, np.int32)
        n_past = np.ascontiguousarray(n_past, np.int32)
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.empty((len(slots), self.nout), np.float32)
        rc = lib().o_step(self.h, _ptr(slots), _ptr(n_past), _ptr(ids), len(slots), _ptr(out))
        assert rc == 0
        return out.reshape(len(slots), self.model.hp.n_codebooks, -1)

    def last_sel(self) -> np.ndarray:
        n = lib().o_last_sel(self.h, None, 0)
        out = np.empty(max(n, 1), np.int32)
        lib().o_last_sel(self.h, _ptr(out), n)
        return out[:n]

    def fake_fill(self, slot: int, n: int, seed: int = 0):
        lib().o_ctx_fake_fill(self.h, slot, n, seed)

    def hash_fill(self, slot: int, n: int, seed: int = 0):
        """KV of positions [0, n) from the integer hash the GPU's z2b_debug_fill_kv uses."""
        lib().o_ctx_hash_fill(self.h, slot, n, seed)

    def __del__(self):
        if getattr(self, "h", None):
            lib().o_ctx_free(self.h)
            self.h = None


class Sampler:
    """zonos2_sampler restated (std::mt19937 + uniform_real_distribution<double>)."""

    def __init__(self, n_codebooks, temperature=1.15, top_k=106, top_p=0.0, min_p=0.18, rep_penalty=1.2,
                 rep_window=50, rep_codebooks=8, seed=0, greedy=False):
        self.ncb = n_codebooks
        self.h = lib().o_sampler_new(temperature, top_k, top_p, min_p, rep_penalty, rep_window, rep_codebooks,
                                     seed, 1 if greedy else 0, n_codebooks)

    def sample(self, logits: np.ndarray) -> np.ndarray:
        logits = np.ascontiguousarray(logits, np.float32)
        codes = np.empty(self.ncb, np.int32)
        lib().o_sample_frame(self.h, _ptr(logits), self.ncb, logits.shape[-1], _ptr(codes))
        return codes

    def __del__(self):
        if getattr(self, "h", None):
            lib().o_sampler_free(self.h)
            self.h = None
