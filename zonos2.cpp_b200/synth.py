"""Synthetic ZONOS2-family GGUF files for tests and benchmarks (wraps libz2b_synth.so).

Presets follow the workload configs this library is measured on:
  tiny        d 256, 4 MoE layers (E 8, top-2, ff 512), 8x32 heads / 2 KV, theta 1e4,
              Q8_0 bulk with the converter's F16 tier for embeddings/head/router
              (models/convert-zonos2-to-gguf.py pick_qtype, outtype q8_0).
  zonos2      d 2048, 28 MoE layers (E 32, top-4, ff 1408), 16x128 heads / 4 KV,
              theta 1e6: Q4_K attention and expert gate/up, Q6_K embeddings, Q8_0
              head/router (the quantizer's one-tier-up set, src/quantize.cpp:48-70),
              expert down F16 because 1408 is not a multiple of 256 (src/quantize.cpp:129).
  zonos2_q8   same shapes, Q8_0 everywhere the quantizer would put the bulk type.
  zonos2_q6k  same shapes, Q6_K bulk (down again falls back to F16).
The audio vocabulary is codebook_size + 2 = 1026 (eoa 1024, pad 1025) as in the reference.
"""
from __future__ import annotations

import ctypes
import os

F32, F16, Q8_0, Q4_K, Q6_K = 0, 1, 8, 12, 14
MAX_LAYERS = 128


class SynthConfig(ctypes.Structure):
    _fields_ = [
        ("n_layer", ctypes.c_uint32), ("n_embd", ctypes.c_uint32), ("head_dim", ctypes.c_uint32),
        ("n_head", ctypes.c_uint32), ("n_head_kv", ctypes.c_uint32), ("n_ff", ctypes.c_uint32),
        ("n_expert", ctypes.c_uint32), ("router_dim", ctypes.c_uint32), ("n_ctx", ctypes.c_uint32),
        ("expert_used", ctypes.c_int32 * MAX_LAYERS),
        ("rope_base", ctypes.c_float), ("rms_eps", ctypes.c_float), ("qk_eps", ctypes.c_float),
        ("softcap", ctypes.c_float),
        ("n_codebooks", ctypes.c_uint32), ("codebook_size", ctypes.c_uint32),
        ("text_vocab", ctypes.c_uint32), ("spk_dim", ctypes.c_uint32), ("lda_dim", ctypes.c_uint32),
        ("t_attn", ctypes.c_uint32), ("t_gateup", ctypes.c_uint32), ("t_down", ctypes.c_uint32),
        ("t_dense", ctypes.c_uint32), ("t_head", ctypes.c_uint32), ("t_embd", ctypes.c_uint32),
        ("t_router", ctypes.c_uint32), ("t_spk", ctypes.c_uint32),
        ("init_mode", ctypes.c_uint32), ("std", ctypes.c_float), ("seed", ctypes.c_uint64),
    ]


def _base(**kw):
    d = dict(n_codebooks=9, codebook_size=1024, text_vocab=519, spk_dim=128, lda_dim=64,
             rms_eps=1e-5, qk_eps=1e-6, softcap=15.0, init_mode=1, std=0.02, seed=0,
             n_ctx=8192)
    d.update(kw)
    return d


PRESETS = {
    "tiny": _base(n_layer=4, n_embd=256, head_dim=32, n_head=8, n_head_kv=2, n_ff=512,
                  n_expert=8, router_dim=128, expert_used=[2] * 4, rope_base=1e4,
                  t_attn=Q8_0, t_gateup=Q8_0, t_down=Q8_0, t_dense=Q8_0, t_head=F16,
                  t_embd=F16, t_router=F16, t_spk=F16, n_ctx=2048),
    "zonos2": _base(n_layer=28, n_embd=2048, head_dim=128, n_head=16, n_head_kv=4, n_ff=1408,
                    n_expert=32, router_dim=128, expert_used=[4] * 28, rope_base=1e6,
                    t_attn=Q4_K, t_gateup=Q4_K, t_down=Q4_K, t_dense=Q4_K, t_head=Q8_0,
                    t_embd=Q6_K, t_router=Q8_0, t_spk=Q8_0),
    "zonos2_q8": _base(n_layer=28, n_embd=2048, head_dim=128, n_head=16, n_head_kv=4, n_ff=1408,
                       n_expert=32, router_dim=128, expert_used=[4] * 28, rope_base=1e6,
                       t_attn=Q8_0, t_gateup=Q8_0, t_down=Q8_0, t_dense=Q8_0, t_head=F16,
                       t_embd=F16, t_router=F16, t_spk=F16),
    "zonos2_q6k": _base(n_layer=28, n_embd=2048, head_dim=128, n_head=16, n_head_kv=4, n_ff=1408,
                        n_expert=32, router_dim=128, expert_used=[4] * 28, rope_base=1e6,
                        t_attn=Q6_K, t_gateup=Q6_K, t_down=Q6_K, t_dense=Q6_K, t_head=Q8_0,
                        t_embd=Q8_0, t_router=Q8_0, t_spk=Q8_0),
}


def make_config(preset: str = "tiny", **overrides) -> SynthConfig:
    p = dict(PRESETS[preset])
    p.update(overrides)
    c = SynthConfig()
    for k, v in p.items():
        if k == "expert_used":
            for i, x in enumerate(v):
                c.expert_used[i] = x
        else:
            setattr(c, k, v)
    if len(p["expert_used"]) != p["n_layer"]:
        raise ValueError("expert_used must have n_layer entries")
    return c


_lib = None


def _load():
    global _lib
    if _lib is None:
        from .build import SYNTH_LIB, build_synth
        if not os.path.exists(SYNTH_LIB):
            build_synth()
        _lib = ctypes.CDLL(SYNTH_LIB)
        _lib.z2b_synth_write.argtypes = [ctypes.POINTER(SynthConfig), ctypes.c_char_p,
                                         ctypes.c_char_p, ctypes.c_int]
        _lib.z2b_synth_write.restype = ctypes.c_int
    return _lib


def write(path: str, preset: str = "tiny", **overrides) -> str:
    """Write a synthetic GGUF; returns the path."""
    cfg = make_config(preset, **overrides)
    err = ctypes.create_string_buffer(512)
    rc = _load().z2b_synth_write(ctypes.byref(cfg), path.encode(), err, 512)
    if rc != 0:
        raise RuntimeError("z2b_synth_write: " + err.value.decode())
    return path


def cached(preset: str = "tiny", directory: str | None = None, **overrides) -> str:
    """Path of a synthetic GGUF for (preset, overrides), generating it once per directory."""
    directory = directory or os.environ.get("Z2B_MODEL_DIR", "/tmp/z2b_models")
    os.makedirs(directory, exist_ok=True)
    tag = preset + "".join(f"_{k}-{v}" for k, v in sorted(overrides.items()) if k != "expert_used")
    if "expert_used" in overrides:
        tag += "_eu-" + "-".join(map(str, overrides["expert_used"]))
    path = os.path.join(directory, tag + ".gguf")
    if not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        write(tmp, preset, **overrides)
        os.replace(tmp, path)
    return path


# ---------------------------------------------------------------- DAC decoder files

DAC_PRESETS = {
    # the real decoder's shapes (DAC 44 kHz: latent 1024, decoder 1536, rates 8/8/4/2, hop 512)
    "dac44k": dict(latent=1024, decoder_dim=1536, rates=(8, 8, 4, 2)),
    # small shapes for parity tests: every kernel path (channel padding, four blocks, all rates)
    "dac_small": dict(latent=64, decoder_dim=256, rates=(8, 8, 4, 2)),
    "dac_tiny": dict(latent=8, decoder_dim=16, rates=(2, 2)),
}


def write_dac(path: str, preset: str = "dac_small", seed: int = 0, n_codebooks: int = 9,
              codebook_size: int = 1024, sample_rate: int = 44100) -> str:
    """Write a synthetic DAC decoder GGUF with the tensor names, shapes and f32 storage of the
    reference's converter (models/convert-dac-to-gguf.py): folded quantizer tables, conv_in,
    the decoder blocks (snake, transposed conv, three residual units), snake_out, conv_out.
    Random weights scaled so activations stay O(1) through the residual stack and the
    pre-tanh output spans tanh's linear and saturated ranges."""
    import numpy as np
    from gguf import GGUFWriter

    p = DAC_PRESETS[preset]
    lat, dd, rates = p["latent"], p["decoder_dim"], list(p["rates"])
    rng = np.random.default_rng(seed)
    w = GGUFWriter(path, "dac")
    w.add_string("general.name", f"DAC-synthetic-{preset}")
    for k, v in (("n_codebooks", n_codebooks), ("codebook_size", codebook_size), ("latent_dim", lat),
                 ("decoder_dim", dd), ("sample_rate", sample_rate), ("hop_length", int(np.prod(rates))),
                 ("audio_pad_id", codebook_size + 1)):
        w.add_uint32(f"dac.{k}", v)
    w.add_array("dac.decoder_rates", rates)

    def put(name, a):
        w.add_tensor(name, np.ascontiguousarray(a, dtype=np.float32))

    def normal(shape, std):
        return (rng.standard_normal(shape) * std).astype(np.float32)

    def conv(name, oc, ic, k, gain=1.0):
        put(name + ".weight", normal((oc, ic, k), gain / np.sqrt(ic * k)))
        put(name + ".bias", normal((oc, 1), 0.1))

    def snake(name, c):
        a = rng.uniform(0.5, 1.5, (c, 1)).astype(np.float32)
        put(name + ".alpha", a)
        put(name + ".inv_alpha", (1.0 / (a + 1e-9)).astype(np.float32))

    for i in range(n_codebooks):
        put(f"quant.{i}.table", normal((codebook_size, lat), 1.0 / np.sqrt(n_codebooks)))
    put("quant.bias", normal((lat,), 0.1))
    conv("dec.conv_in", dd, lat, 7)
    for b, s in enumerate(rates):
        ci, co = dd >> b, dd >> (b + 1)
        snake(f"dec.b{b}.snake", ci)
        put(f"dec.b{b}.convt.weight", normal((ci, co, 2 * s), 1.0 / np.sqrt(2 * ci)))
        put(f"dec.b{b}.convt.bias", normal((co, 1), 0.1))
        for r in range(3):
            snake(f"dec.b{b}.res{r}.snake1", co)
            conv(f"dec.b{b}.res{r}.conv1", co, co, 7)
            snake(f"dec.b{b}.res{r}.snake2", co)
            conv(f"dec.b{b}.res{r}.conv2", co, co, 1, gain=0.5)
    cf = dd >> len(rates)
    snake("dec.snake_out", cf)
    conv("dec.conv_out", 1, cf, 7, gain=0.3)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file(progress=False)
    w.close()
    return path


def cached_dac(preset: str = "dac_small", seed: int = 0, directory: str | None = None) -> str:
    """Path of a synthetic DAC GGUF for (preset, seed), generating it once per directory."""
    directory = directory or os.environ.get("Z2B_MODEL_DIR", "/tmp/z2b_models")
    os.makedirs(directory, exist_ok=True)
    path = os.path.join(directory, f"{preset}_seed-{seed}.gguf")
    if not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        write_dac(tmp, preset, seed)
        os.replace(tmp, path)
    return path
