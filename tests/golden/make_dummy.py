"""Regenerate the reference's CI fixture model, tests/fixtures/dummy-zonos2.gguf.

The reference commits a tiny random zonos2 GGUF for its smoke test and documents its
recipe (scripts/make-dummy-model.py): numpy default_rng(0), N(0, 0.02) draws in tensor
order, f32 for 1-D tensors and f16 for matrices, 4 layers with expert_used [0, 1, 2, 0]
(dense, first MoE without EDA scale, top-2 MoE with EDA scale, dense), d 32, head_dim 16,
2 heads / 1 KV head, ffn 128, 4 experts, router 32, speaker 32/16, real 9 x 1026 head and
520-row text table. This script rebuilds that file from the documented recipe with
gguf-py's writer so the GPU tests can use the same model on a machine without the
reference tree; tests/test_dummy_fixture.py checks that the bytes are identical to the
committed fixture wherever the reference tree is available.

    python tests/golden/make_dummy.py OUT.gguf
"""
from __future__ import annotations

import sys

import numpy as np
from gguf import GGUFWriter

ARCH = "zonos2"
D, HD, NH, NKV, FF, NE, RD, SPK, LDA = 32, 16, 2, 1, 128, 4, 32, 32, 16
EXPERT_USED = [0, 1, 2, 0]
NCB, CB = 9, 1024
AV = CB + 2
TV = 519


def write(path: str) -> str:
    g = np.random.default_rng(0)

    def draw(*shape):
        x = g.standard_normal(shape) * 0.02
        return x.astype(np.float32 if len(shape) == 1 else np.float16)

    w = GGUFWriter(path, ARCH)
    w.add_string("general.name", "ZONOS2-dummy")
    for key, val in [("block_count", len(EXPERT_USED)), ("context_length", 512), ("embedding_length", D),
                     ("head_dim", HD), ("attention.head_count", NH), ("attention.head_count_kv", NKV),
                     ("feed_forward_length", FF)]:
        w.add_uint32(f"{ARCH}.{key}", val)
    w.add_float32(f"{ARCH}.rope.freq_base", 10000.0)
    w.add_float32(f"{ARCH}.attention.layer_norm_rms_epsilon", 1e-5)
    w.add_float32(f"{ARCH}.attention.qk_norm_epsilon", 1e-6)
    w.add_float32(f"{ARCH}.logit_softcap", 15.0)
    w.add_uint32(f"{ARCH}.expert_count", NE)
    w.add_array(f"{ARCH}.expert_used_count_per_layer", EXPERT_USED)
    for key, val in [("n_codebooks", NCB), ("codebook_size", CB), ("audio_vocab", AV), ("eoa_id", CB),
                     ("audio_pad_id", CB + 1), ("text_vocab", TV), ("speaker.embedding_dim", SPK),
                     ("speaker.lda_dim", LDA)]:
        w.add_uint32(f"{ARCH}.{key}", val)
    w.add_file_type(1)

    for i in range(NCB):
        w.add_tensor(f"audio_embd.{i}.weight", draw(AV, D))
    w.add_tensor("text_embd.weight", draw(TV + 1, D))
    w.add_tensor("spk_lda.weight", draw(LDA, SPK))
    w.add_tensor("spk_lda.bias", draw(LDA))
    w.add_tensor("spk_proj.weight", draw(D, LDA))
    w.add_tensor("spk_proj.bias", draw(D))
    w.add_tensor("output_norm.weight", draw(D))
    w.add_tensor("output.weight", draw(NCB * AV, D))
    moe_seen = False
    for L, k in enumerate(EXPERT_USED):
        b = f"blk.{L}."
        w.add_tensor(b + "attn_norm.weight", draw(D))
        w.add_tensor(b + "ffn_norm.weight", draw(D))
        w.add_tensor(b + "attn_q.weight", draw(NH * HD, D))
        w.add_tensor(b + "attn_k.weight", draw(NKV * HD, D))
        w.add_tensor(b + "attn_v.weight", draw(NKV * HD, D))
        w.add_tensor(b + "attn_output.weight", draw(D, NH * HD))
        w.add_tensor(b + "attn_temp", draw(NH))
        w.add_tensor(b + "attn_gate.weight", draw(NH, D))
        if k == 0:
            for nm, shape in [("ffn_up", (FF, D)), ("ffn_gate", (FF, D)), ("ffn_down", (D, FF))]:
                w.add_tensor(b + nm + ".weight", draw(*shape))
            continue
        for nm, shape in [("ffn_gate_exps", (NE, FF, D)), ("ffn_up_exps", (NE, FF, D)), ("ffn_down_exps", (NE, D, FF))]:
            w.add_tensor(b + nm + ".weight", draw(*shape))
        w.add_tensor(b + "router_down.weight", draw(RD, D))
        w.add_tensor(b + "router_down.bias", draw(RD))
        for nm in ("router_mlp0", "router_mlp2"):
            w.add_tensor(b + nm + ".weight", draw(RD, RD))
            w.add_tensor(b + nm + ".bias", draw(RD))
        w.add_tensor(b + "router_mlp4.weight", draw(NE, RD))
        w.add_tensor(b + "router_norm.weight", draw(RD))
        w.add_tensor(b + "router_bias", draw(NE))
        if moe_seen:
            w.add_tensor(b + "router_eda_scale", draw(RD))
        moe_seen = True
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return path


if __name__ == "__main__":
    print(write(sys.argv[1]))
