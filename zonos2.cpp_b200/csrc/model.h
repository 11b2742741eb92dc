// model.h — device-resident zonos2 backbone (weights in tile layout).
#pragma once

#include "gguf.h"
#include "kernels.h"
#include "../../include/z2b.h"

#include <string>
#include <vector>

namespace z2b {

struct LayerDev {
    DevMat wq, wk, wv, wo, wgate;
    bool qkvg_fused = false;             // q, k, v, gate share type and K: one launch
    bool is_moe = false;
    int top_k = 0, n_expert = 0;
    DevMat gate_exps, up_exps, down_exps;   // stacks (dense layers: one "expert")
    LayerSmall small{};
    // device f32 copies owned by the model
    std::vector<float*> owned;
};

struct Model {
    z2b_hparams hp{};
    Dims dims{};
    int device = 0;
    int n_sm = 148;
    EmbedDev emb{};
    std::vector<void*> allocs;            // every cudaMalloc of the model
    DevMat head;
    const float* out_norm = nullptr;
    // speaker injection (src/zonos2-graph.cpp:262-292): lda [lda_dim][spk_dim], proj [n_embd][lda_dim], f32
    const float* spk_lda_w = nullptr;
    const float* spk_lda_b = nullptr;
    const float* spk_proj_w = nullptr;
    const float* spk_proj_b = nullptr;
    std::vector<LayerDev> layers;
    uint64_t attn_bytes_per_layer = 0;    // GGUF bytes of the attention matrices (all layers equal)
    uint64_t head_bytes = 0, router_bytes_per_layer = 0;
    uint64_t expert_bytes = 0;            // GGUF bytes of one expert (gate + up + down)
    size_t emb_row_bytes = 0;
    ~Model();
};

// Loads and uploads; on failure returns an error code and sets err.
int model_load(const char* path, int device, Model** out, std::string& err);

}  // namespace z2b
