"""Synthetic GGUF contract (CPU): keys and tensor names the reference loader requires."""
from __future__ import annotations

import numpy as np
import pytest
from gguf import GGUFReader

import z2b.synth as S

# keys read by zonos2_model_load (src/zonos2.cpp:34-71)
REQUIRED_KEYS = [
    "zonos2.block_count", "zonos2.embedding_length", "zonos2.head_dim", "zonos2.attention.head_count",
    "zonos2.attention.head_count_kv", "zonos2.feed_forward_length", "zonos2.expert_count",
    "zonos2.context_length", "zonos2.rope.freq_base", "zonos2.attention.layer_norm_rms_epsilon",
    "zonos2.attention.qk_norm_epsilon", "zonos2.logit_softcap", "zonos2.n_codebooks", "zonos2.codebook_size",
    "zonos2.audio_vocab", "zonos2.eoa_id", "zonos2.audio_pad_id", "zonos2.text_vocab",
    "zonos2.speaker.embedding_dim", "zonos2.speaker.lda_dim", "zonos2.expert_used_count_per_layer",
]


def _names(n_layer, eu):
    # tensor names mapped by zonos2_model_load (src/zonos2.cpp:137-182)
    names = [f"audio_embd.{i}.weight" for i in range(9)] + ["text_embd.weight", "spk_lda.weight", "spk_lda.bias",
             "spk_proj.weight", "spk_proj.bias", "output_norm.weight", "output.weight"]
    first = True
    for L in range(n_layer):
        b = f"blk.{L}."
        names += [b + x for x in ["attn_norm.weight", "ffn_norm.weight", "attn_q.weight", "attn_k.weight",
                                  "attn_v.weight", "attn_output.weight", "attn_temp", "attn_gate.weight"]]
        if eu[L] == 0:
            names += [b + "ffn_up.weight", b + "ffn_gate.weight", b + "ffn_down.weight"]
        else:
            names += [b + x for x in ["ffn_gate_exps.weight", "ffn_up_exps.weight", "ffn_down_exps.weight",
                                      "router_down.weight", "router_down.bias", "router_mlp0.weight",
                                      "router_mlp0.bias", "router_mlp2.weight", "router_mlp2.bias",
                                      "router_mlp4.weight", "router_norm.weight", "router_bias"]]
            if not first:
                names.append(b + "router_eda_scale")
            first = False
    return names


@pytest.mark.parametrize("eu", [[2, 2, 2, 2], [0, 1, 2, 0]])
def test_keys_and_names(tmp_path, eu):
    p = S.write(str(tmp_path / "m.gguf"), "tiny", expert_used=eu)
    r = GGUFReader(p)
    for k in REQUIRED_KEYS:
        assert k in r.fields, k
    have = {t.name for t in r.tensors}
    assert set(_names(4, eu)) == have


def test_audio_vocab_and_ids(tmp_path):
    p = S.write(str(tmp_path / "m.gguf"), "tiny")
    f = GGUFReader(p).fields
    v = lambda k: int(f[k].parts[f[k].data[0]][0])
    assert v("zonos2.audio_vocab") == 1026 and v("zonos2.eoa_id") == 1024 and v("zonos2.audio_pad_id") == 1025


def test_zonos2_type_policy(tmp_path):
    """Q4_K preset: attention/gate/up Q4_K, expert down F16 (1408 % 256 != 0), head/router Q8_0,
    embeddings Q6_K, 1-D f32 — the reference quantizer's fallbacks (src/quantize.cpp:116-131)."""
    p = S.write(str(tmp_path / "z.gguf"), "zonos2", n_layer=1, expert_used=[4], n_expert=2)
    t = {x.name: x.tensor_type.name for x in GGUFReader(p).tensors}
    assert t["blk.0.attn_q.weight"] == "Q4_K" and t["blk.0.ffn_gate_exps.weight"] == "Q4_K"
    assert t["blk.0.ffn_down_exps.weight"] == "F16"
    assert t["output.weight"] == "Q8_0" and t["blk.0.router_down.weight"] == "Q8_0"
    assert t["audio_embd.0.weight"] == "Q6_K" and t["blk.0.attn_norm.weight"] == "F32"


def test_generator_deterministic(tmp_path):
    a = S.write(str(tmp_path / "a.gguf"), "tiny")
    b = S.write(str(tmp_path / "b.gguf"), "tiny")
    assert open(a, "rb").read() == open(b, "rb").read()
