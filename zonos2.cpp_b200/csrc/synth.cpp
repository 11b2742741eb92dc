// synth.cpp — synthetic ZONOS2-family GGUF writer (host, OpenMP).
//
// Emits the same keys (src/zonos2.cpp:34-71) and tensor names/shapes
// (src/zonos2.cpp:137-182; scripts/make-dummy-model.py:95-136) the reference
// loader requires, with random weights from a counter-based generator so the
// bytes are identical for any thread count and the 7.6B-parameter file is
// produced in seconds on the benchmark host. Storage types follow the
// reference quantizer policy (src/quantize.cpp:116-131): 1-D tensors stay F32,
// a matrix whose row length is not a multiple of its block falls back to F16.
#include "gguf.h"
#include "quant.h"
#include "../../include/z2b_tools.h"

#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

using namespace z2b;

namespace {

inline uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

// Standard normals for elements (2p, 2p+1) of tensor `tid` (Box-Muller over a hashed counter).
inline void normal_pair(uint64_t seed, uint64_t tid, uint64_t p, float* z0, float* z1) {
    const uint64_t base = splitmix64(seed * 0x100000001B3ull ^ (tid << 40)) ^ p;
    const uint64_t h1 = splitmix64(base * 2 + 0), h2 = splitmix64(base * 2 + 1);
    const double u1 = ((double)(h1 >> 11) + 0.5) * (1.0 / 9007199254740992.0);
    const double u2 = (double)(h2 >> 11) * (1.0 / 9007199254740992.0);
    const double r = std::sqrt(-2.0 * std::log(u1));
    const double a = 6.283185307179586 * u2;
    *z0 = (float)(r * std::cos(a));
    *z1 = (float)(r * std::sin(a));
}

enum Init { I_NORMAL, I_ONE_PLUS, I_ABS_ONE_PLUS };

struct TSpec {
    std::string name;
    uint32_t type;
    int n_dims;
    int64_t ne[4];
    Init init;
    float std;
};

uint32_t pick_type(uint32_t want, int n_dims, int64_t ne0) {
    if (n_dims == 1) return GT_F32;
    int be = 0, bb = 0;
    if (!gtype_info(want, &be, &bb)) return GT_F16;
    return (ne0 % be == 0) ? want : GT_F16;
}

}  // namespace

extern "C" int z2b_synth_write(const z2b_synth_config* c, const char* path, char* err, int errlen) {
    auto fail = [&](const std::string& m) {
        if (err && errlen > 0) { std::snprintf(err, (size_t)errlen, "%s", m.c_str()); }
        return 1;
    };
    if (!c || !path) return fail("null argument");
    if (c->n_layer < 1 || c->n_layer > Z2B_MAX_LAYERS) return fail("n_layer out of range");
    if (c->n_head * c->head_dim == 0 || c->n_head_kv == 0 || c->n_head % c->n_head_kv) return fail("bad head configuration");
    if (c->n_embd % 2 || c->n_ff % 2 || c->router_dim % 2 || c->spk_dim % 2 || c->lda_dim % 2) return fail("dimensions must be even");
    const int64_t d = c->n_embd, hd = c->head_dim, nh = c->n_head, nkv = c->n_head_kv;
    const int64_t ff = c->n_ff, E = c->n_expert, rd = c->router_dim;
    const int64_t av = c->codebook_size + 2, ncb = c->n_codebooks;
    const float sd = c->std;
    const bool scaled = c->init_mode == 1;

    std::vector<TSpec> ts;
    auto add = [&](const std::string& n, uint32_t want, std::vector<int64_t> np_shape, Init init, float stdv) {
        TSpec t; t.name = n; t.n_dims = (int)np_shape.size(); t.init = init; t.std = stdv;
        for (int i = 0; i < 4; ++i) t.ne[i] = 1;
        for (int i = 0; i < t.n_dims; ++i) t.ne[i] = np_shape[t.n_dims - 1 - i];   // numpy -> ggml ne
        t.type = pick_type(want, t.n_dims, t.ne[0]);
        ts.push_back(t);
    };
    const Init norm_init = scaled ? I_ONE_PLUS : I_NORMAL;
    const float r_std0 = scaled ? 1.0f / std::sqrt((float)rd) : sd;
    const float r_std4 = scaled ? 1.5f / std::sqrt((float)rd) : sd;

    for (int i = 0; i < ncb; ++i) add("audio_embd." + std::to_string(i) + ".weight", c->t_embd, {av, d}, I_NORMAL, sd);
    add("text_embd.weight", c->t_embd, {(int64_t)c->text_vocab + 1, d}, I_NORMAL, sd);
    add("spk_lda.weight", c->t_spk, {(int64_t)c->lda_dim, (int64_t)c->spk_dim}, I_NORMAL, sd);
    add("spk_lda.bias", GT_F32, {(int64_t)c->lda_dim}, I_NORMAL, sd);
    add("spk_proj.weight", c->t_spk, {d, (int64_t)c->lda_dim}, I_NORMAL, sd);
    add("spk_proj.bias", GT_F32, {d}, I_NORMAL, sd);
    add("output_norm.weight", GT_F32, {d}, norm_init, sd);
    add("output.weight", c->t_head, {ncb * av, d}, I_NORMAL, sd);
    bool seen_moe = false;
    for (uint32_t L = 0; L < c->n_layer; ++L) {
        const std::string b = "blk." + std::to_string(L) + ".";
        add(b + "attn_norm.weight", GT_F32, {d}, norm_init, sd);
        add(b + "ffn_norm.weight", GT_F32, {d}, norm_init, sd);
        add(b + "attn_q.weight", c->t_attn, {nh * hd, d}, I_NORMAL, sd);
        add(b + "attn_k.weight", c->t_attn, {nkv * hd, d}, I_NORMAL, sd);
        add(b + "attn_v.weight", c->t_attn, {nkv * hd, d}, I_NORMAL, sd);
        add(b + "attn_output.weight", c->t_attn, {d, nh * hd}, I_NORMAL, sd);
        add(b + "attn_temp", GT_F32, {nh}, scaled ? I_ABS_ONE_PLUS : I_NORMAL, sd);
        add(b + "attn_gate.weight", c->t_attn, {nh, d}, I_NORMAL, sd);
        if (c->expert_used[L] == 0) {
            add(b + "ffn_up.weight", c->t_dense, {ff, d}, I_NORMAL, sd);
            add(b + "ffn_gate.weight", c->t_dense, {ff, d}, I_NORMAL, sd);
            add(b + "ffn_down.weight", c->t_dense, {d, ff}, I_NORMAL, sd);
        } else {
            add(b + "ffn_gate_exps.weight", c->t_gateup, {E, ff, d}, I_NORMAL, sd);
            add(b + "ffn_up_exps.weight", c->t_gateup, {E, ff, d}, I_NORMAL, sd);
            add(b + "ffn_down_exps.weight", c->t_down, {E, d, ff}, I_NORMAL, sd);
            add(b + "router_down.weight", c->t_router, {rd, d}, I_NORMAL, sd);
            add(b + "router_down.bias", GT_F32, {rd}, I_NORMAL, sd);
            add(b + "router_mlp0.weight", c->t_router, {rd, rd}, I_NORMAL, r_std0);
            add(b + "router_mlp0.bias", GT_F32, {rd}, I_NORMAL, sd);
            add(b + "router_mlp2.weight", c->t_router, {rd, rd}, I_NORMAL, r_std0);
            add(b + "router_mlp2.bias", GT_F32, {rd}, I_NORMAL, sd);
            add(b + "router_mlp4.weight", c->t_router, {E, rd}, I_NORMAL, r_std4);
            add(b + "router_norm.weight", GT_F32, {rd}, norm_init, sd);
            add(b + "router_bias", GT_F32, {E}, I_NORMAL, sd);
            if (seen_moe) add(b + "router_eda_scale", GT_F32, {rd}, I_NORMAL, sd);
            seen_moe = true;
        }
    }

    GGUFWriter w;
    w.add_str("general.architecture", "zonos2");
    w.add_str("general.name", "ZONOS2-synthetic");
    w.add_u32("zonos2.block_count", c->n_layer);
    w.add_u32("zonos2.context_length", c->n_ctx);
    w.add_u32("zonos2.embedding_length", c->n_embd);
    w.add_u32("zonos2.head_dim", c->head_dim);
    w.add_u32("zonos2.attention.head_count", c->n_head);
    w.add_u32("zonos2.attention.head_count_kv", c->n_head_kv);
    w.add_u32("zonos2.feed_forward_length", c->n_ff);
    w.add_f32("zonos2.rope.freq_base", c->rope_base);
    w.add_f32("zonos2.attention.layer_norm_rms_epsilon", c->rms_eps);
    w.add_f32("zonos2.attention.qk_norm_epsilon", c->qk_eps);
    w.add_f32("zonos2.logit_softcap", c->softcap);
    w.add_u32("zonos2.expert_count", c->n_expert);
    w.add_arr_i32("zonos2.expert_used_count_per_layer",
                  std::vector<int32_t>(c->expert_used, c->expert_used + c->n_layer));
    w.add_u32("zonos2.n_codebooks", c->n_codebooks);
    w.add_u32("zonos2.codebook_size", c->codebook_size);
    w.add_u32("zonos2.audio_vocab", (uint32_t)av);
    w.add_u32("zonos2.eoa_id", c->codebook_size);
    w.add_u32("zonos2.audio_pad_id", c->codebook_size + 1);
    w.add_u32("zonos2.text_vocab", c->text_vocab);
    w.add_u32("zonos2.speaker.embedding_dim", c->spk_dim);
    w.add_u32("zonos2.speaker.lda_dim", c->lda_dim);
    w.add_u32("general.file_type", 1);
    for (auto& t : ts) w.add_tensor(t.name, t.type, t.n_dims, t.ne);
    std::string e;
    if (!w.begin(path, e)) return fail(e);

    std::vector<uint8_t> buf;
    for (size_t ti = 0; ti < ts.size(); ++ti) {
        const TSpec& t = ts[ti];
        const int64_t ne0 = t.ne[0], rows = t.ne[1] * t.ne[2] * t.ne[3];
        const size_t rb = gtype_row_bytes(t.type, ne0);
        buf.resize(rb * (size_t)rows);
        int bad = 0;
#pragma omp parallel
        {
            std::vector<float> row((size_t)ne0);
#pragma omp for schedule(static)
            for (int64_t r = 0; r < rows; ++r) {
                for (int64_t i = 0; i < ne0; i += 2) {      // ne0 is even for every tensor
                    float z[2];
                    normal_pair(c->seed, ti, (uint64_t)(r * ne0 + i) >> 1, &z[0], &z[1]);
                    for (int j = 0; j < 2; ++j) {
                        float v = z[j] * t.std;
                        if (t.init == I_ONE_PLUS) v = 1.0f + v;
                        else if (t.init == I_ABS_ONE_PLUS) v = std::fabs(1.0f + v);
                        row[i + j] = v;
                    }
                }
                if (!quantize_row(t.type, row.data(), buf.data() + (size_t)r * rb, ne0)) {
#pragma omp atomic write
                    bad = 1;
                }
            }
        }
        if (bad) return fail("unsupported type for " + t.name);
        if (!w.write_tensor((int)ti, buf.data(), buf.size(), 0, e)) return fail(e);
    }
    if (!w.finish(e)) return fail(e);
    return 0;
}
