// model.cpp — ggml-free zonos2 GGUF loader: hyper-parameters, tensor mapping, tile
// repack and device upload. Follows zonos2_model_load (src/zonos2.cpp:15-186): the same
// required keys (:34-71), the same tensor names (:137-182), router_eda_scale optional.
#include "model.h"
#include "quant.h"
#include "repack.h"
#include "tile_layout.h"

#include <cstring>
#include <cuda_runtime.h>

namespace z2b {

Model::~Model() {
    for (void* p : allocs) cudaFree(p);
}

namespace {

struct Loader {
    GGUFFile f;
    Model* m;
    std::string err;
    int rc = Z2B_OK;

    bool fail(int code, const std::string& e) { if (rc == Z2B_OK) { rc = code; err = e; } return false; }

    bool u32(const char* key, uint32_t& dst) {
        const GKV* kv = f.kv(key);
        if (!kv) return fail(Z2B_ERR_FORMAT, std::string("missing kv '") + key + "'");
        dst = (uint32_t)kv->u;
        return true;
    }
    bool f32(const char* key, float& dst) {
        const GKV* kv = f.kv(key);
        if (!kv) return fail(Z2B_ERR_FORMAT, std::string("missing kv '") + key + "'");
        dst = (float)kv->f;
        return true;
    }
    const GTensor* req(const std::string& n) {
        const GTensor* t = f.tensor(n);
        if (!t) fail(Z2B_ERR_FORMAT, "required tensor '" + n + "' not found");
        else if (!t->data) fail(Z2B_ERR_UNSUPPORTED, "tensor '" + n + "' has unsupported type " + std::to_string(t->type));
        return t && t->data ? t : nullptr;
    }
    void* dalloc(size_t n) {
        void* p = nullptr;
        if (cudaMalloc(&p, n ? n : 16) != cudaSuccess) { fail(Z2B_ERR_OOM, "cudaMalloc failed"); return nullptr; }
        m->allocs.push_back(p);
        return p;
    }
    bool h2d(void* dst, const void* src, size_t n) {
        if (cudaMemcpy(dst, src, n, cudaMemcpyHostToDevice) != cudaSuccess) return fail(Z2B_ERR_CUDA, "cudaMemcpy failed");
        return true;
    }
    // f32 copy of any tensor (dequantised), expected element count n
    const float* small(const GTensor* t, int64_t n) {
        if (!t) return nullptr;
        if (t->nelements() != n) { fail(Z2B_ERR_FORMAT, "tensor '" + t->name + "' has unexpected size"); return nullptr; }
        std::vector<float> v((size_t)n);
        dequant_row(t->type, t->data, v.data(), n);
        float* d = (float*)dalloc((size_t)n * 4);
        if (!d || !h2d(d, v.data(), (size_t)n * 4)) return nullptr;
        return d;
    }
    // weight matrix [experts][rows][K] -> tile image
    bool mat(const GTensor* t, int64_t K, int64_t rows, int experts, DevMat& out) {
        if (!t) return false;
        if (t->ne[0] != K || t->ne[1] != rows || t->ne[2] != experts || t->ne[3] != 1)
            return fail(Z2B_ERR_FORMAT, "tensor '" + t->name + "' has unexpected shape");
        uint32_t type = t->type;
        const size_t rb = gtype_row_bytes(type, K);
        std::vector<uint8_t> conv;
        const uint8_t* src = t->data;
        TileGeom g;
        if (!tile_geom(type, K, &g)) {
            // no tile format for this type/K (F32, BF16, or a K the block tiles do not
            // divide): store as F16
            if (!tile_geom(GT_F16, K, &g)) return fail(Z2B_ERR_UNSUPPORTED, "tensor '" + t->name + "': K not a multiple of 16");
            const int64_t n = K * rows * experts;
            std::vector<float> tmp((size_t)K);
            conv.resize((size_t)n * 2);
            for (int64_t r = 0; r < rows * experts; ++r) {
                dequant_row(type, t->data + (size_t)r * rb, tmp.data(), K);
                quantize_row_f16(tmp.data(), conv.data() + (size_t)r * K * 2, K);
            }
            src = conv.data();
            type = GT_F16;
        }
        const size_t srb = gtype_row_bytes(type, K);
        const int64_t per = tiles_bytes(type, rows, K);
        std::vector<uint8_t> img((size_t)per * experts);
        for (int e = 0; e < experts; ++e)
            if (!repack_rows(type, rows, K, src + (size_t)e * rows * srb, img.data() + (size_t)e * per))
                return fail(Z2B_ERR_UNSUPPORTED, "repack failed for '" + t->name + "'");
        uint8_t* d = (uint8_t*)dalloc(img.size());
        if (!d || !h2d(d, img.data(), img.size())) return false;
        out.tiles = d;
        out.type = type;
        out.rows = (int)rows;
        out.K = (int)K;
        out.n_row_tiles = (int)((rows + TILE_ROWS - 1) / TILE_ROWS);
        out.chunks = (int)g.chunks;
        out.tile_bytes = g.tile_bytes;
        out.steps = g.steps;
        out.expert_stride = per;
        out.n_expert = experts;
        out.gguf_bytes = t->nbytes;
        return true;
    }

    bool load(const char* path, int device) {
        std::string e;
        if (!f.open(path, e)) return fail(Z2B_ERR_IO, e);
        z2b_hparams& hp = m->hp;
        bool ok = u32("zonos2.block_count", hp.n_layer) & u32("zonos2.embedding_length", hp.n_embd) &
                  u32("zonos2.head_dim", hp.head_dim) & u32("zonos2.attention.head_count", hp.n_head) &
                  u32("zonos2.attention.head_count_kv", hp.n_head_kv) & u32("zonos2.feed_forward_length", hp.n_ff) &
                  u32("zonos2.expert_count", hp.n_expert) & u32("zonos2.context_length", hp.n_ctx_train) &
                  f32("zonos2.rope.freq_base", hp.rope_freq_base) &
                  f32("zonos2.attention.layer_norm_rms_epsilon", hp.rms_eps) &
                  f32("zonos2.attention.qk_norm_epsilon", hp.qk_norm_eps) & f32("zonos2.logit_softcap", hp.logit_softcap) &
                  u32("zonos2.n_codebooks", hp.n_codebooks) & u32("zonos2.codebook_size", hp.codebook_size) &
                  u32("zonos2.audio_vocab", hp.audio_vocab) & u32("zonos2.eoa_id", hp.eoa_id) &
                  u32("zonos2.audio_pad_id", hp.audio_pad_id) & u32("zonos2.text_vocab", hp.text_vocab) &
                  u32("zonos2.speaker.embedding_dim", hp.spk_dim) & u32("zonos2.speaker.lda_dim", hp.spk_lda_dim);
        if (!ok) return false;
        const GKV* eu = f.kv("zonos2.expert_used_count_per_layer");
        if (!eu || eu->type != GV_ARR || eu->arr_type != GV_I32)
            return fail(Z2B_ERR_FORMAT, "missing/!int32 expert_used_count_per_layer");
        if (eu->ai.size() != hp.n_layer) return fail(Z2B_ERR_FORMAT, "expert_used length != n_layer");
        if (hp.n_layer > 128) return fail(Z2B_ERR_UNSUPPORTED, "more than 128 layers");
        for (uint32_t L = 0; L < hp.n_layer; ++L) hp.expert_used[L] = (int32_t)eu->ai[L];
        const int hd = (int)hp.head_dim, nh = (int)hp.n_head, nkv = (int)hp.n_head_kv, d = (int)hp.n_embd;
        if (hd != 16 && hd != 32 && hd != 64 && hd != 128) return fail(Z2B_ERR_UNSUPPORTED, "head_dim must be 16/32/64/128");
        if (nkv == 0 || nh % nkv || nh / nkv > 8) return fail(Z2B_ERR_UNSUPPORTED, "GQA group size must divide and be <= 8");
        if (hp.n_codebooks > 15) return fail(Z2B_ERR_UNSUPPORTED, "more than 15 codebooks");
        if (d % 16) return fail(Z2B_ERR_UNSUPPORTED, "n_embd must be a multiple of 16");

        if (cudaSetDevice(device) != cudaSuccess) return fail(Z2B_ERR_CUDA, "cudaSetDevice failed");
        m->device = device;
        cudaDeviceGetAttribute(&m->n_sm, cudaDevAttrMultiProcessorCount, device);

        // embeddings: raw GGUF rows
        const GTensor* te = req("text_embd.weight");
        if (!te) return false;
        m->emb.type = te->type;
        m->emb.row_bytes = gtype_row_bytes(te->type, d);
        auto up_raw = [&](const GTensor* t) -> const uint8_t* {
            if (!t) return nullptr;
            if (t->type != m->emb.type || t->ne[0] != d) { fail(Z2B_ERR_UNSUPPORTED, "embedding tables must share type and width"); return nullptr; }
            uint8_t* p = (uint8_t*)dalloc(t->nbytes);
            if (!p || !h2d(p, t->data, t->nbytes)) return nullptr;
            return p;
        };
        for (uint32_t i = 0; i < hp.n_codebooks; ++i) {
            const GTensor* t = req("audio_embd." + std::to_string(i) + ".weight");
            if (!t) return false;
            if (t->ne[1] != hp.audio_vocab) return fail(Z2B_ERR_FORMAT, "audio_embd rows != audio_vocab");
            m->emb.audio[i] = up_raw(t);
            if (!m->emb.audio[i]) return false;
        }
        if (te->ne[1] != (int64_t)hp.text_vocab + 1) return fail(Z2B_ERR_FORMAT, "text_embd rows != text_vocab+1");
        m->emb.text = up_raw(te);
        if (!m->emb.text) return false;
        m->emb_row_bytes = m->emb.row_bytes;
        {
            const int64_t sd = hp.spk_dim, ld = hp.spk_lda_dim;
            if (sd < 1 || ld < 1 || sd > 8192 || ld > 1024) return fail(Z2B_ERR_UNSUPPORTED, "speaker dims out of range");
            const GTensor* lw = req("spk_lda.weight");
            const GTensor* pw = req("spk_proj.weight");
            if (!lw || !pw) return false;
            if (lw->ne[0] != sd || lw->ne[1] != ld || pw->ne[0] != ld || pw->ne[1] != d)
                return fail(Z2B_ERR_FORMAT, "speaker projection shapes");
            m->spk_lda_w = small(req("spk_lda.weight"), sd * ld);
            m->spk_lda_b = small(req("spk_lda.bias"), ld);
            m->spk_proj_w = small(req("spk_proj.weight"), ld * d);
            m->spk_proj_b = small(req("spk_proj.bias"), d);
            if (!m->spk_lda_w || !m->spk_lda_b || !m->spk_proj_w || !m->spk_proj_b) return false;
        }
        m->out_norm = small(req("output_norm.weight"), d);
        if (!m->out_norm) return false;
        const int64_t nout = (int64_t)hp.n_codebooks * hp.audio_vocab;
        if (!mat(req("output.weight"), d, nout, 1, m->head)) return false;
        m->head_bytes = m->head.gguf_bytes;

        m->layers.resize(hp.n_layer);
        int rd = 0;
        bool first = true;
        for (uint32_t L = 0; L < hp.n_layer; ++L) {
            LayerDev& ly = m->layers[L];
            const std::string b = "blk." + std::to_string(L) + ".";
            LayerSmall& s = ly.small;
            s.attn_norm = small(req(b + "attn_norm.weight"), d);
            s.ffn_norm = small(req(b + "ffn_norm.weight"), d);
            s.attn_temp = small(req(b + "attn_temp"), nh);
            if (!s.attn_norm || !s.ffn_norm || !s.attn_temp) return false;
            if (!mat(req(b + "attn_q.weight"), d, (int64_t)nh * hd, 1, ly.wq)) return false;
            if (!mat(req(b + "attn_k.weight"), d, (int64_t)nkv * hd, 1, ly.wk)) return false;
            if (!mat(req(b + "attn_v.weight"), d, (int64_t)nkv * hd, 1, ly.wv)) return false;
            if (!mat(req(b + "attn_output.weight"), (int64_t)nh * hd, d, 1, ly.wo)) return false;
            if (!mat(req(b + "attn_gate.weight"), d, nh, 1, ly.wgate)) return false;
            ly.qkvg_fused = ly.wq.type == ly.wk.type && ly.wq.type == ly.wv.type && ly.wq.type == ly.wgate.type;
            if (L == 0) m->attn_bytes_per_layer = ly.wq.gguf_bytes + ly.wk.gguf_bytes + ly.wv.gguf_bytes +
                                                  ly.wo.gguf_bytes + ly.wgate.gguf_bytes;
            const int k = hp.expert_used[L];
            ly.top_k = k;
            ly.is_moe = k > 0;
            s.is_moe = ly.is_moe ? 1 : 0;
            s.top_k = k;
            if (!ly.is_moe) {
                ly.n_expert = 1;
                s.n_expert = 1;
                if (!mat(req(b + "ffn_gate.weight"), d, hp.n_ff, 1, ly.gate_exps)) return false;
                if (!mat(req(b + "ffn_up.weight"), d, hp.n_ff, 1, ly.up_exps)) return false;
                if (!mat(req(b + "ffn_down.weight"), hp.n_ff, d, 1, ly.down_exps)) return false;
            } else {
                const GTensor* gu = req(b + "ffn_up_exps.weight");
                if (!gu) return false;
                const int E = (int)gu->ne[2];     // per-layer expert count (pruned files differ)
                if (E > MAX_EXPERTS) return fail(Z2B_ERR_UNSUPPORTED, "more than 256 experts");
                if (k > 8 || k > E) return fail(Z2B_ERR_UNSUPPORTED, "top-k must be <= 8 and <= experts");
                ly.n_expert = E;
                s.n_expert = E;
                if (!mat(req(b + "ffn_gate_exps.weight"), d, hp.n_ff, E, ly.gate_exps)) return false;
                if (!mat(gu, d, hp.n_ff, E, ly.up_exps)) return false;
                if (!mat(req(b + "ffn_down_exps.weight"), hp.n_ff, d, E, ly.down_exps)) return false;
                const GTensor* rdw = req(b + "router_down.weight");
                if (!rdw) return false;
                if (rd == 0) rd = (int)rdw->ne[1];
                if (rdw->ne[1] != rd || rdw->ne[0] != d) return fail(Z2B_ERR_FORMAT, "router_down shape");
                if (rdw->type == GT_Q8_0) {
                    // split Q8_0 blocks into int8 rows and f32 scales: w = q * d exactly
                    const int64_t nb = (int64_t)rd * d / 32;
                    std::vector<int8_t> qs((size_t)rd * d);
                    std::vector<float> ds((size_t)nb);
                    for (int64_t blk = 0; blk < nb; ++blk) {
                        uint16_t dh; std::memcpy(&dh, rdw->data + blk * 34, 2);
                        ds[blk] = f16_to_f32(dh);
                        std::memcpy(&qs[blk * 32], rdw->data + blk * 34 + 2, 32);
                    }
                    int8_t* dq = (int8_t*)dalloc(qs.size());
                    float* dd = (float*)dalloc(ds.size() * 4);
                    if (!dq || !dd || !h2d(dq, qs.data(), qs.size()) || !h2d(dd, ds.data(), ds.size() * 4)) return false;
                    s.rdown_q = dq;
                    s.rdown_qd = dd;
                    s.rdown_w = nullptr;
                } else {
                    s.rdown_w = small(rdw, (int64_t)rd * d);
                    s.rdown_q = nullptr;
                    s.rdown_qd = nullptr;
                }
                s.rdown_b = small(req(b + "router_down.bias"), rd);
                s.m0_w = small(req(b + "router_mlp0.weight"), (int64_t)rd * rd);
                s.m0_b = small(req(b + "router_mlp0.bias"), rd);
                s.m2_w = small(req(b + "router_mlp2.weight"), (int64_t)rd * rd);
                s.m2_b = small(req(b + "router_mlp2.bias"), rd);
                s.m4_w = small(req(b + "router_mlp4.weight"), (int64_t)E * rd);
                s.rnorm = small(req(b + "router_norm.weight"), rd);
                s.rbias = small(req(b + "router_bias"), E);
                const GTensor* eda = f.tensor(b + "router_eda_scale");
                s.eda = eda ? small(eda, rd) : nullptr;
                if ((!s.rdown_w && !s.rdown_q) || !s.rdown_b || !s.m0_w || !s.m0_b || !s.m2_w || !s.m2_b || !s.m4_w || !s.rnorm || !s.rbias)
                    return false;
                if (eda && !s.eda) return false;
                // prompt-row routes run on the tcgen05 GEMM when every expert matrix type has
                // its dequantiser there and the gate/up type matches
                s.gemm_ok = moe_gemm_supported(ly.gate_exps) && moe_gemm_supported(ly.up_exps) &&
                            moe_gemm_supported(ly.down_exps) && ly.gate_exps.type == ly.up_exps.type ? 1 : 0;
                if (first) {
                    m->router_bytes_per_layer = rdw->nbytes + f.tensor(b + "router_mlp0.weight")->nbytes +
                                                f.tensor(b + "router_mlp2.weight")->nbytes +
                                                f.tensor(b + "router_mlp4.weight")->nbytes;
                    m->expert_bytes = (ly.gate_exps.gguf_bytes + ly.up_exps.gguf_bytes + ly.down_exps.gguf_bytes) / E;
                }
                first = false;
            }
        }
        hp.router_dim = (uint32_t)rd;
        uint64_t total = 0;
        for (const GTensor& t : f.tensors()) total += t.nbytes;
        hp.weight_bytes = total;
        Dims& D = m->dims;
        D.n_embd = d; D.head_dim = hd; D.n_head = nh; D.n_head_kv = nkv; D.n_ff = (int)hp.n_ff;
        D.rd = rd; D.n_layer = (int)hp.n_layer; D.n_codebooks = (int)hp.n_codebooks;
        D.audio_vocab = (int)hp.audio_vocab; D.text_vocab = (int)hp.text_vocab;
        D.rms_eps = hp.rms_eps; D.qk_eps = hp.qk_norm_eps; D.rope_base = hp.rope_freq_base; D.softcap = hp.logit_softcap;
        if (rd > 512 || rd % 8) return fail(Z2B_ERR_UNSUPPORTED, "router_dim must be a multiple of 8, at most 512");
        if (d % 16) return fail(Z2B_ERR_UNSUPPORTED, "n_embd must be a multiple of 16 (router K slices)");
        return true;
    }
};

}  // namespace

int model_load(const char* path, int device, Model** out, std::string& err) {
    Model* m = new Model();
    Loader ld;
    ld.m = m;
    if (!ld.load(path, device)) {
        err = ld.err;
        const int rc = ld.rc == Z2B_OK ? Z2B_ERR_FORMAT : ld.rc;
        delete m;
        return rc;
    }
    *out = m;
    return Z2B_OK;
}

}  // namespace z2b
