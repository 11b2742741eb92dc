"""ctypes binding of include/z2b.h — the Python host mirror of the reference batch API.

Names follow src/zonos2.h: ``Model`` (zonos2_model_load / _free), ``BatchCtx``
(zonos2_batch_init / _free, zonos2_batch_slot_prefill, zonos2_batch_step,
zonos2_batch_slot_logits) and ``Slot`` (zonos2_slot, with the per-frame EOS logic of
zonos2_slot_sample, src/zonos2-graph.cpp:843-870). Sampling itself runs on the device.
Every call raises ``Z2BError`` when the library returns an error; there is no fallback
path — without libz2b.so and a CUDA device nothing here works.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, field

import numpy as np

from .build import LIB

NCOL = 10
WANT_LOGITS = 1
WANT_SAMPLE = 3


class Z2BError(RuntimeError):
    def __init__(self, rc, msg):
        super().__init__(f"z2b error {rc}: {msg}")
        self.rc = rc


class HParams(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint32) for n in ("n_layer", "n_embd", "head_dim", "n_head", "n_head_kv", "n_ff",
                                                "n_expert", "n_ctx_train")] + \
               [(n, ctypes.c_float) for n in ("rope_freq_base", "rms_eps", "qk_norm_eps", "logit_softcap")] + \
               [(n, ctypes.c_uint32) for n in ("n_codebooks", "codebook_size", "audio_vocab", "eoa_id",
                                                "audio_pad_id", "text_vocab", "spk_dim", "spk_lda_dim",
                                                "router_dim")] + \
               [("expert_used", ctypes.c_int32 * 128), ("weight_bytes", ctypes.c_uint64)]


class Sampling(ctypes.Structure):
    """zonos2_sampling (src/zonos2.h:197-208) with the reference defaults."""
    _fields_ = [("temperature", ctypes.c_float), ("top_k", ctypes.c_int32), ("top_p", ctypes.c_float),
                ("min_p", ctypes.c_float), ("rep_penalty", ctypes.c_float), ("rep_window", ctypes.c_int32),
                ("rep_codebooks", ctypes.c_int32), ("seed", ctypes.c_uint32), ("greedy", ctypes.c_int32)]

    def __init__(self, temperature=1.15, top_k=106, top_p=0.0, min_p=0.18, rep_penalty=1.2, rep_window=50,
                 rep_codebooks=8, seed=0, greedy=False):
        super().__init__(temperature, top_k, top_p, min_p, rep_penalty, rep_window, rep_codebooks, seed,
                         1 if greedy else 0)


class PromptOptions(ctypes.Structure):
    """zonos2_prompt_options (src/zonos2.h:181-188)."""
    _fields_ = [("prepend_silence", ctypes.c_int32), ("speaking_rate_bucket", ctypes.c_int32),
                ("n_quality", ctypes.c_int32), ("quality_buckets", ctypes.c_int32 * 16),
                ("add_speaker_slot", ctypes.c_int32), ("clean_speaker_background", ctypes.c_int32),
                ("accurate_mode", ctypes.c_int32)]


class SlotDesc(ctypes.Structure):
    _fields_ = [("slot", ctypes.c_int32), ("n_past", ctypes.c_int32), ("n_new", ctypes.c_int32),
                ("flags", ctypes.c_int32), ("cfg_twin", ctypes.c_int32), ("cfg_scale", ctypes.c_float)]


_lib = None


def lib():
    """Load libz2b.so (built in-tree by __graft_entry__.build() / build.py)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            raise Z2BError(-1, f"{LIB} is not built; run __graft_entry__.build()")
        L = ctypes.CDLL(LIB)
        P, I, V = ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p
        sig = {
            "z2b_model_load": ([ctypes.c_char_p, I, ctypes.POINTER(P)], I),
            "z2b_model_free": ([P], I),
            "z2b_model_hparams": ([P, ctypes.POINTER(HParams)], I),
            "z2b_set_expert_mask": ([P, V, I, V, V], I),
            "z2b_ctx_create": ([P, I, I, ctypes.POINTER(P)], I),
            "z2b_ctx_destroy": ([P], I),
            "z2b_slot_reset": ([P, I, ctypes.POINTER(Sampling)], I),
            "z2b_set_slot_sampling": ([P, I, ctypes.POINTER(Sampling)], I),
            "z2b_slot_prefill": ([P, I, V, I, V], I),
            "z2b_slot_prefill_spk": ([P, I, V, I, V, I, V, V], I),
            "z2b_logits": ([P, V, I, V, V, I, V], I),
            "z2b_step": ([P, V, I, V, V, V], I),
            "z2b_step_logits": ([P, I], ctypes.POINTER(ctypes.c_float)),
            "z2b_decode_loop": ([P, V, I, V, I], I),
            "z2b_sync": ([P], I),
            "z2b_ctx_stream": ([P], P),
            "z2b_last_step_bytes": ([P, V, V, V], I),
            "z2b_last_step_launches": ([P], I),
            "z2b_last_error": ([], ctypes.c_char_p),
            "z2b_last_step_active": ([P, V, I], I),
            "z2b_last_codes": ([P, V, I], I),
            "z2b_last_step_io": ([P, V, V], I),
            "z2b_set_logits_readback": ([P, I], I),
            "z2b_run_schedule": ([P, I, I, V, V, I, V], I),
            "z2b_last_run_launches": ([P], ctypes.c_long),
            "z2b_profile": ([P, I, V, V, I], I),
            "z2b_time_expert_gemv": ([P, I, I, V, V], I),
            "z2b_expert_op": ([P, I, V, I, V, V, I, V, I, V, V, V], I),
            "z2b_test_dequant": ([ctypes.c_uint32, ctypes.c_int64, ctypes.c_int64, V, I, V], I),
            "z2b_test_gemv": ([ctypes.c_uint32, ctypes.c_int64, ctypes.c_int64, V, V, I, V], I),
            "z2b_host_tiles_bytes": ([ctypes.c_uint32, ctypes.c_int64, ctypes.c_int64], ctypes.c_int64),
            "z2b_host_repack": ([ctypes.c_uint32, ctypes.c_int64, ctypes.c_int64, V, V], I),
            "z2b_host_unpack_tiles": ([ctypes.c_uint32, ctypes.c_int64, ctypes.c_int64, V, V], I),
            "z2b_slot_after_frame": ([ctypes.POINTER(HParams), ctypes.POINTER(SlotState), V, I, I], I),
            "z2b_debug_fill_kv": ([P, I, I, ctypes.c_uint32], I),
            "z2b_set_expert_gemm_min": ([P, I], I),
            "z2b_debug_router_capture": ([P, I], I),
            "z2b_debug_router_inputs": ([P, I, V, V, ctypes.POINTER(ctypes.c_int)], I),
            "z2b_debug_last_sel": ([P, V, I], I),
            "z2b_prompt_options_default": ([V], None),
            "z2b_build_prompt": ([ctypes.POINTER(HParams), ctypes.c_char_p, ctypes.c_int64, V, V, I, V, V], I),
            "z2b_dac_load": ([ctypes.c_char_p, I, ctypes.POINTER(P)], I),
            "z2b_dac_free": ([P], I),
            "z2b_dac_get_hparams": ([P, V], I),
            "z2b_dac_decode": ([P, V, I, I, I, V, ctypes.c_int64, V], I),
            "z2b_dac_decode_window": ([P, V, I, I, I, I, I, V, ctypes.c_int64, V], I),
            "z2b_dac_decode_windows": ([P, V, I, V, ctypes.c_int64, V], I),
            "z2b_dac_last_launches": ([P], ctypes.c_long),
            "z2b_dac_stream": ([P], P),
            "z2b_dac_wav_bytes": ([V, ctypes.c_int64, I, V, ctypes.c_int64], ctypes.c_int64),
        }
        for name, (args, res) in sig.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib = L
    return _lib


def _check(rc):
    if rc != 0:
        raise Z2BError(rc, lib().z2b_last_error().decode(errors="replace"))


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


class Model:
    """A zonos2 GGUF loaded onto one GPU (zonos2_model)."""

    def __init__(self, path: str, device: int = 0):
        h = ctypes.c_void_p()
        _check(lib().z2b_model_load(path.encode(), device, ctypes.byref(h)))
        self.h = h
        self.hp = HParams()
        _check(lib().z2b_model_hparams(self.h, ctypes.byref(self.hp)))

    def set_expert_mask(self, keep: dict[int, list[int]]):
        layers = np.array(sorted(keep), np.int32)
        offs, ids = [0], []
        for L in layers:
            ids += list(keep[int(L)])
            offs.append(len(ids))
        offs = np.array(offs, np.int32)
        ids = np.array(ids or [0], np.int32)
        _check(lib().z2b_set_expert_mask(self.h, _ptr(layers), len(layers), _ptr(offs), _ptr(ids)))

    def logits(self, ids, spk=None, spk_pos: int = 0, spk_emotion_delta=None) -> np.ndarray:
        """zonos2_logits: teacher-forced logits [n, ncb, av] of every row of one sequence."""
        ids = np.ascontiguousarray(ids, np.int32).reshape(-1, NCOL)
        n = ids.shape[0]
        out = np.empty((n, self.hp.n_codebooks, self.hp.audio_vocab), np.float32)
        sp = None if spk is None else np.ascontiguousarray(spk, np.float32)
        dl = None if spk_emotion_delta is None else np.ascontiguousarray(spk_emotion_delta, np.float32)
        _check(lib().z2b_logits(self.h, _ptr(ids), n, _ptr(out), _ptr(sp), int(spk_pos), _ptr(dl)))
        return out

    def close(self):
        if self.h:
            lib().z2b_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


@dataclass
class Slot:
    """zonos2_slot: graph-facing per-stream state owned by the caller."""
    index: int
    n_past: int = 0
    step: int = 0
    eos_frame: int = -1
    countdown: int = -1
    done: bool = False
    next_ids: list = field(default_factory=list)


class BatchCtx:
    """Continuous-batching context (zonos2_batch_ctx) on one GPU."""

    def __init__(self, model: Model, n_slots: int, slot_cap_frames: int):
        self.model = model
        h = ctypes.c_void_p()
        _check(lib().z2b_ctx_create(model.h, n_slots, slot_cap_frames, ctypes.byref(h)))
        self.h = h
        hp = model.hp
        self.ncb, self.av = hp.n_codebooks, hp.audio_vocab
        self.n_slots = n_slots

    def close(self):
        if self.h:
            lib().z2b_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def slot_reset(self, slot: int, sampling: Sampling | None = None):
        _check(lib().z2b_slot_reset(self.h, slot, ctypes.byref(sampling) if sampling else None))

    def set_sampling(self, slot: int, sampling: Sampling | None = None):
        """The stream's sampler (parameters, seed, empty history), keeping its KV."""
        _check(lib().z2b_set_slot_sampling(self.h, slot, ctypes.byref(sampling) if sampling else None))

    def slot_prefill(self, slot: int, ids, spk=None, spk_pos: int = 0, spk_emotion_delta=None) -> np.ndarray:
        """zonos2_batch_slot_prefill: returns the last prompt row's logits [ncb, av]. With
        spk ([spk_dim] f32), row spk_pos's embedding is replaced by the projected speaker
        (+ spk_emotion_delta, [n_embd] f32, when given)."""
        ids = np.ascontiguousarray(ids, np.int32).reshape(-1, NCOL)
        out = np.empty((self.ncb, self.av), np.float32)
        if spk is None:
            _check(lib().z2b_slot_prefill(self.h, slot, _ptr(ids), ids.shape[0], _ptr(out)))
        else:
            spk = np.ascontiguousarray(spk, np.float32)
            delta = None if spk_emotion_delta is None else np.ascontiguousarray(spk_emotion_delta, np.float32)
            _check(lib().z2b_slot_prefill_spk(self.h, slot, _ptr(ids), ids.shape[0], _ptr(spk), int(spk_pos),
                                              _ptr(out), _ptr(delta) if delta is not None else None))
        return out

    def step(self, descs, ids, want_logits=True):
        """One batched step. descs: list of (slot, n_past, n_new, flags[, cfg_twin, cfg_scale]).
        Returns (codes [n, ncb] int32, logits [n, ncb, av] or None)."""
        n = len(descs)
        arr = (SlotDesc * n)()
        for i, d in enumerate(descs):
            d = tuple(d) + (-1, 1.0)[len(d) - 4:] if len(d) < 6 else tuple(d)
            arr[i] = SlotDesc(int(d[0]), int(d[1]), int(d[2]), int(d[3]), int(d[4]), float(d[5]))
        ids = np.ascontiguousarray(ids, np.int32).reshape(-1, NCOL)
        codes = np.full((n, self.ncb), -1, np.int32)
        logits = np.empty((n, self.ncb, self.av), np.float32) if want_logits else None
        _check(lib().z2b_step(self.h, ctypes.cast(arr, ctypes.c_void_p), n, _ptr(ids), _ptr(codes), _ptr(logits)))
        return codes, logits

    def fill_kv(self, slot: int, n: int, seed: int):
        """Test support: KV of positions [0, n) from the hash the oracle's hash_fill uses."""
        _check(lib().z2b_debug_fill_kv(self.h, slot, n, seed))

    def router_capture(self, enable: bool):
        """Test support: record every MoE router's inputs of the following steps."""
        _check(lib().z2b_debug_router_capture(self.h, 1 if enable else 0))

    def router_inputs(self, layer: int):
        """(residual rows [T, d], incoming router state [T, rd]) of `layer` in the last step."""
        T = ctypes.c_int(0)
        _check(lib().z2b_debug_router_inputs(self.h, layer, None, None, ctypes.byref(T)))
        hp = self.model.hp
        res = np.empty((T.value, hp.n_embd), np.float32)
        st = np.empty((T.value, hp.router_dim), np.float32)
        _check(lib().z2b_debug_router_inputs(self.h, layer, _ptr(res), _ptr(st), ctypes.byref(T)))
        return res, st

    def last_sel(self) -> np.ndarray:
        """Router ids of every layer of the last step: [n_layer, T, kmax]."""
        need = lib().z2b_debug_last_sel(self.h, None, 0)
        buf = np.empty(need, np.int32)
        lib().z2b_debug_last_sel(self.h, _ptr(buf), need)
        return buf

    def step_logits(self, index: int):
        """zonos2_batch_slot_logits: logits [ncb, av] of desc `index` of the last step (a copy of
        the context's host view), or None when that desc has none."""
        p = lib().z2b_step_logits(self.h, int(index))
        if not p:
            return None
        return np.ctypeslib.as_array(p, shape=(self.ncb * self.av,)).reshape(self.ncb, self.av).copy()

    def decode_loop(self, descs, first_ids, n_steps: int):
        n = len(descs)
        arr = (SlotDesc * n)()
        for i, d in enumerate(descs):
            arr[i] = SlotDesc(int(d[0]), int(d[1]), 1, WANT_SAMPLE, -1, 1.0)
        first_ids = np.ascontiguousarray(first_ids, np.int32).reshape(-1, NCOL)
        _check(lib().z2b_decode_loop(self.h, ctypes.cast(arr, ctypes.c_void_p), n, _ptr(first_ids), n_steps))

    def sync(self):
        _check(lib().z2b_sync(self.h))

    def stream(self) -> int:
        return lib().z2b_ctx_stream(self.h) or 0

    def time_expert_gemv(self, which: int, reps: int):
        """(ms per launch, algorithmic bytes per launch) of the expert gate/up (0) or down (1)
        GEMV, timed over `reps` back-to-back launches on the last step's routing."""
        ms, nb = ctypes.c_double(), ctypes.c_uint64()
        _check(lib().z2b_time_expert_gemv(self.h, int(which), int(reps), ctypes.byref(ms), ctypes.byref(nb)))
        return ms.value, nb.value

    def set_expert_gemm_min(self, routes: int):
        """Routes from which an expert of the isolated expert op takes the tensor-core GEMM."""
        _check(lib().z2b_set_expert_gemm_min(self.h, int(routes)))

    def expert_op(self, layer: int, x, sel, selw, reps: int = 0, want_out: bool = True):
        """The isolated expert op of a MoE layer: returns (out [T][d] or None, ms per
        repetition or None, routed weight bytes, experts on the tensor-core GEMM)."""
        x = np.ascontiguousarray(x, np.float32)
        sel = np.ascontiguousarray(sel, np.int32)
        selw = np.ascontiguousarray(selw, np.float32)
        T, k = sel.shape
        out = np.empty((T, x.shape[1]), np.float32) if want_out else None
        ms, nb, ng = ctypes.c_double(0.0), ctypes.c_uint64(0), ctypes.c_int32(0)
        _check(lib().z2b_expert_op(self.h, int(layer), _ptr(x), T, _ptr(sel), _ptr(selw), k, _ptr(out), int(reps),
                                   ctypes.byref(ms), ctypes.byref(nb), ctypes.byref(ng)))
        return out, (ms.value if reps > 0 else None), nb.value, ng.value

    def last_step_bytes(self):
        w, k, o = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
        _check(lib().z2b_last_step_bytes(self.h, ctypes.byref(w), ctypes.byref(k), ctypes.byref(o)))
        return w.value, k.value, o.value

    def last_step_launches(self) -> int:
        return lib().z2b_last_step_launches(self.h)

    def last_step_active(self) -> np.ndarray:
        out = np.zeros(self.model.hp.n_layer, np.int32)
        lib().z2b_last_step_active(self.h, _ptr(out), len(out))
        return out

    def run_schedule(self, descs: np.ndarray, rows: np.ndarray, row_src: np.ndarray):
        """descs: int32/float [n_steps, n, 6] (slot, n_past, n_new, flags, cfg_twin, cfg_scale)."""
        n_steps, n = descs.shape[:2]
        arr = (SlotDesc * (n_steps * n))()
        flat = descs.reshape(-1, 6)
        for j in range(n_steps * n):
            d = flat[j]
            arr[j] = SlotDesc(int(d[0]), int(d[1]), int(d[2]), int(d[3]), int(d[4]), float(d[5]))
        rows = np.ascontiguousarray(rows, np.int32).reshape(-1, NCOL)
        row_src = np.ascontiguousarray(row_src, np.int32)
        self._keep = (arr, rows, row_src)          # host copies stay alive while the run is queued
        _check(lib().z2b_run_schedule(self.h, n_steps, n, ctypes.cast(arr, ctypes.c_void_p), _ptr(rows),
                                      rows.shape[0], _ptr(row_src)))

    def last_step_io(self):
        h, d = ctypes.c_uint64(), ctypes.c_uint64()
        _check(lib().z2b_last_step_io(self.h, ctypes.byref(h), ctypes.byref(d)))
        return h.value, d.value

    def set_logits_readback(self, enable: bool):
        _check(lib().z2b_set_logits_readback(self.h, 1 if enable else 0))

    def last_codes(self, n: int) -> np.ndarray:
        out = np.zeros((n, self.ncb), np.int32)
        _check(lib().z2b_last_codes(self.h, _ptr(out), n))
        return out

    def last_run_launches(self) -> int:
        return int(lib().z2b_last_run_launches(self.h))

    PROF_CLASSES = ["pack", "embed", "qkv_gemv", "rope_append", "attention", "attn_combine", "wo_gemv", "router",
                    "expert_gateup_gemv", "expert_down_gemv", "moe_combine", "head_gemv", "sampler", "feed"]

    def profile(self, enable: bool):
        n = len(self.PROF_CLASSES)
        ms = np.zeros(n, np.float64)
        cnt = np.zeros(n, np.int64)
        _check(lib().z2b_profile(self.h, 1 if enable else 0, _ptr(ms), _ptr(cnt), n))
        if not enable:
            return {k: (float(ms[i]), int(cnt[i])) for i, k in enumerate(self.PROF_CLASSES)}


class SlotState(ctypes.Structure):
    """z2b_slot_state (include/z2b.h): zonos2_slot's per-stream fields."""
    _fields_ = [("index", ctypes.c_int32), ("done", ctypes.c_int32), ("n_past", ctypes.c_int32),
                ("step", ctypes.c_int32), ("eos_frame", ctypes.c_int32), ("countdown", ctypes.c_int32),
                ("next_ids", ctypes.c_int32 * 32)]


def slot_after_sample(hp: HParams, s: Slot, codes, max_frames: int, keep: bool = True) -> bool:
    """EOS / countdown / next_ids bookkeeping of zonos2_slot_sample (src/zonos2-graph.cpp:852-868),
    through z2b_slot_after_frame; updates `s` in place and returns keep."""
    ncb = hp.n_codebooks
    st = SlotState(s.index, 1 if s.done else 0, s.n_past, s.step, s.eos_frame, s.countdown)
    c = np.ascontiguousarray(np.asarray(codes[:ncb], np.int32))
    rc = lib().z2b_slot_after_frame(ctypes.byref(hp), ctypes.byref(st), _ptr(c), int(max_frames), 1 if keep else 0)
    if rc < 0:
        raise Z2BError(1, lib().z2b_last_error().decode())
    s.done, s.step, s.eos_frame, s.countdown = bool(st.done), st.step, st.eos_frame, st.countdown
    s.next_ids = [int(x) for x in st.next_ids[:ncb + 1]]
    return bool(rc)


def build_prompt(hp: HParams, text, prepend_silence=True, speaking_rate_bucket=-1, quality_buckets=None,
                 add_speaker_slot=False, clean_speaker_background=True, accurate_mode=True):
    """zonos2_build_prompt: TTS prompt rows [n][n_codebooks + 1] (int32) and the speaker slot's row
    (-1 without one) for text (str, encoded as UTF-8, or bytes)."""
    b = text.encode("utf-8") if isinstance(text, str) else bytes(text)
    o = PromptOptions()
    lib().z2b_prompt_options_default(ctypes.byref(o))
    o.prepend_silence = 1 if prepend_silence else 0
    o.speaking_rate_bucket = speaking_rate_bucket
    if quality_buckets:
        o.n_quality = len(quality_buckets)
        for i, q in enumerate(quality_buckets):
            o.quality_buckets[i] = q
    o.add_speaker_slot = 1 if add_speaker_slot else 0
    o.clean_speaker_background = 1 if clean_speaker_background else 0
    o.accurate_mode = 1 if accurate_mode else 0
    n, sp = ctypes.c_int(), ctypes.c_int()
    _check(lib().z2b_build_prompt(ctypes.byref(hp), b, len(b), ctypes.byref(o), None, 0, ctypes.byref(n),
                                  ctypes.byref(sp)))
    out = np.empty((n.value, hp.n_codebooks + 1), np.int32)
    _check(lib().z2b_build_prompt(ctypes.byref(hp), b, len(b), ctypes.byref(o), _ptr(out), n.value,
                                  ctypes.byref(n), ctypes.byref(sp)))
    return out, sp.value


def test_dequant(qtype: int, rows: int, k: int, raw: np.ndarray, from_tiles: bool) -> np.ndarray:
    out = np.empty((rows, k), np.float32)
    raw = np.ascontiguousarray(raw)
    rc = lib().z2b_test_dequant(qtype, rows, k, _ptr(raw), 1 if from_tiles else 0, _ptr(out))
    if rc != 0:
        raise Z2BError(rc, "z2b_test_dequant")
    return out


def test_gemv(qtype: int, rows: int, k: int, raw: np.ndarray, x: np.ndarray) -> np.ndarray:
    x16 = np.ascontiguousarray(x, np.float16)
    out = np.empty((x16.shape[0], rows), np.float32)
    raw = np.ascontiguousarray(raw)
    rc = lib().z2b_test_gemv(qtype, rows, k, _ptr(raw), x16.ctypes.data_as(ctypes.c_void_p), x16.shape[0], _ptr(out))
    if rc != 0:
        raise Z2BError(rc, "z2b_test_gemv")
    return out
