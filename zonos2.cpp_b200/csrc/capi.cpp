// capi.cpp — extern "C" entry points declared in include/z2b.h.
#include "runtime.h"

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <new>

using namespace z2b;

struct z2b_model { Model* m; };
struct z2b_ctx { Ctx* c; };

extern "C" {

int z2b_model_load(const char* path, int device, z2b_model** out) {
    if (!path || !out) { set_error("null argument"); return Z2B_ERR_ARG; }
    int n_dev = 0;
    if (cudaGetDeviceCount(&n_dev) != cudaSuccess || n_dev == 0) { set_error("no CUDA device"); return Z2B_ERR_CUDA; }
    if (device < 0 || device >= n_dev) { set_error("device index out of range"); return Z2B_ERR_ARG; }
    Model* m = nullptr;
    std::string err;
    const int rc = model_load(path, device, &m, err);
    if (rc) { set_error(err); return rc; }
    *out = new (std::nothrow) z2b_model{m};
    if (!*out) { delete m; set_error("out of host memory"); return Z2B_ERR_OOM; }
    return Z2B_OK;
}

int z2b_model_free(z2b_model* model) {
    if (!model) return Z2B_OK;
    cudaSetDevice(model->m->device);
    delete model->m;
    delete model;
    return Z2B_OK;
}

int z2b_model_hparams(const z2b_model* model, z2b_hparams* out) {
    if (!model || !out) { set_error("null argument"); return Z2B_ERR_ARG; }
    *out = model->m->hp;
    return Z2B_OK;
}

int z2b_set_expert_mask(z2b_model* model, const int32_t* layers, int n_layers, const int32_t* keep_offsets,
                        const int32_t* keep_ids) {
    if (!model) { set_error("null argument"); return Z2B_ERR_ARG; }
    Model* m = model->m;
    cudaSetDevice(m->device);
    for (auto& ly : m->layers) ly.small.rmask = nullptr;     // clear (buffers stay owned by the model)
    for (int i = 0; i < n_layers; ++i) {
        const int L = layers[i];
        if (L < 0 || L >= (int)m->layers.size() || !m->layers[L].is_moe) continue;
        const int E = m->layers[L].n_expert;
        std::vector<float> h(E, -INFINITY);
        for (int j = keep_offsets[i]; j < keep_offsets[i + 1]; ++j)
            if (keep_ids[j] >= 0 && keep_ids[j] < E) h[keep_ids[j]] = 0.0f;
        float* d = nullptr;
        if (cudaMalloc(&d, E * 4) != cudaSuccess) { set_error("cudaMalloc failed"); return Z2B_ERR_OOM; }
        m->allocs.push_back(d);
        cudaMemcpy(d, h.data(), E * 4, cudaMemcpyHostToDevice);
        m->layers[L].small.rmask = d;
    }
    return Z2B_OK;
}

int z2b_ctx_create(z2b_model* model, int n_slots, int slot_cap_frames, z2b_ctx** out) {
    if (!model || !out) { set_error("null argument"); return Z2B_ERR_ARG; }
    Ctx* c = nullptr;
    const int rc = ctx_create(model->m, n_slots, slot_cap_frames, &c);
    if (rc) return rc;
    const char* ng = std::getenv("Z2B_NO_GRAPH");
    c->graphs_enabled = !(ng && ng[0] == '1');
    *out = new z2b_ctx{c};
    return Z2B_OK;
}

int z2b_ctx_destroy(z2b_ctx* ctx) {
    if (!ctx) return Z2B_OK;
    cudaSetDevice(ctx->c->m->device);
    delete ctx->c;
    delete ctx;
    return Z2B_OK;
}

int z2b_slot_reset(z2b_ctx* ctx, int slot, const z2b_sampling* sp) {
    if (!ctx) { set_error("null argument"); return Z2B_ERR_ARG; }
    cudaSetDevice(ctx->c->m->device);
    return ctx_slot_reset(ctx->c, slot, sp);
}

int z2b_set_slot_sampling(z2b_ctx* ctx, int slot, const z2b_sampling* sp) {
    if (!ctx) { set_error("null argument"); return Z2B_ERR_ARG; }
    cudaSetDevice(ctx->c->m->device);
    return ctx_set_sampling(ctx->c, slot, sp);
}

int z2b_slot_prefill(z2b_ctx* ctx, int slot, const int32_t* ids, int n0, float* out_logits) {
    if (!ctx || !ids) { set_error("null argument"); return Z2B_ERR_ARG; }
    cudaSetDevice(ctx->c->m->device);
    return ctx_prefill(ctx->c, slot, ids, n0, out_logits);
}

int z2b_slot_prefill_spk(z2b_ctx* ctx, int slot, const int32_t* ids, int n0, const float* spk, int spk_pos,
                         float* out_logits, const float* spk_emotion_delta) {
    if (!ctx || !ids) { set_error("null argument"); return Z2B_ERR_ARG; }
    cudaSetDevice(ctx->c->m->device);
    return ctx_prefill_spk(ctx->c, slot, ids, n0, spk, spk_pos, spk_emotion_delta, out_logits);
}

int z2b_logits(z2b_model* model, const int32_t* ids, int n_tokens, float* out_logits, const float* spk, int spk_pos,
               const float* spk_emotion_delta) {
    if (!model || !ids || !out_logits) { set_error("null argument"); return Z2B_ERR_ARG; }
    cudaSetDevice(model->m->device);
    return model_logits(model->m, ids, n_tokens, spk, spk_pos, spk_emotion_delta, out_logits);
}

int z2b_step(z2b_ctx* ctx, const z2b_slot_desc* descs, int n, const int32_t* ids, int32_t* out_codes,
             float* out_logits) {
    if (!ctx) { set_error("null argument"); return Z2B_ERR_ARG; }
    cudaSetDevice(ctx->c->m->device);
    return ctx_step(ctx->c, descs, n, ids, out_codes, out_logits);
}

const float* z2b_step_logits(const z2b_ctx* ctx, int index) {
    if (!ctx || index < 0 || index >= (int)ctx->c->step_has_logits.size() || !ctx->c->step_has_logits[index]) return nullptr;
    const Dims& D = ctx->c->m->dims;
    return ctx->c->step_logits.data() + (size_t)index * D.n_codebooks * D.audio_vocab;
}

int z2b_decode_loop(z2b_ctx* ctx, const z2b_slot_desc* descs, int n, const int32_t* first_ids, int n_steps) {
    if (!ctx) { set_error("null argument"); return Z2B_ERR_ARG; }
    cudaSetDevice(ctx->c->m->device);
    return ctx_decode_loop(ctx->c, descs, n, first_ids, n_steps);
}

int z2b_run_schedule(z2b_ctx* ctx, int n_steps, int n, const z2b_slot_desc* descs, const int32_t* rows, int n_rows,
                     const int32_t* row_src) {
    if (!ctx) { set_error("null argument"); return Z2B_ERR_ARG; }
    cudaSetDevice(ctx->c->m->device);
    return ctx_run_schedule(ctx->c, n_steps, n, descs, rows, n_rows, row_src);
}

long z2b_last_run_launches(const z2b_ctx* ctx) { return ctx ? ctx->c->sched_launches : -1; }

int z2b_profile(z2b_ctx* ctx, int enable, double* ms_per_class, long* count_per_class, int n_classes) {
    if (!ctx) { set_error("null argument"); return Z2B_ERR_ARG; }
    Ctx* c = ctx->c;
    cudaSetDevice(c->m->device);
    if (enable) {
        c->profiling = true;
        c->prof_used = 0;
        c->prof_class.clear();
        c->prof_ms.assign(PC_N, 0.0);
        c->prof_count.assign(PC_N, 0);
        return Z2B_OK;
    }
    if (cudaStreamSynchronize(c->stream) != cudaSuccess) { set_error("sync failed"); return Z2B_ERR_CUDA; }
    for (size_t i = 0; i < c->prof_class.size(); ++i) {
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, c->prof_ev[2 * i], c->prof_ev[2 * i + 1]);
        c->prof_ms[c->prof_class[i]] += ms;
        c->prof_count[c->prof_class[i]] += 1;
    }
    c->profiling = false;
    for (int i = 0; i < n_classes && i < PC_N; ++i) {
        if (ms_per_class) ms_per_class[i] = c->prof_ms.empty() ? 0.0 : c->prof_ms[i];
        if (count_per_class) count_per_class[i] = c->prof_count.empty() ? 0 : c->prof_count[i];
    }
    return Z2B_OK;
}

int z2b_sync(z2b_ctx* ctx) {
    if (!ctx) { set_error("null argument"); return Z2B_ERR_ARG; }
    cudaSetDevice(ctx->c->m->device);
    return ctx_sync(ctx->c);
}

void* z2b_ctx_stream(z2b_ctx* ctx) { return ctx ? (void*)ctx->c->stream : nullptr; }

int z2b_last_step_bytes(const z2b_ctx* ctx, uint64_t* weight_bytes, uint64_t* kv_bytes, uint64_t* other_bytes) {
    if (!ctx) { set_error("null argument"); return Z2B_ERR_ARG; }
    if (weight_bytes) *weight_bytes = ctx->c->last_wbytes;
    if (kv_bytes) *kv_bytes = ctx->c->last_kvbytes;
    if (other_bytes) *other_bytes = ctx->c->last_other;
    return Z2B_OK;
}

int z2b_last_step_launches(const z2b_ctx* ctx) { return ctx ? ctx->c->launches : -1; }

int z2b_last_step_io(const z2b_ctx* ctx, uint64_t* h2d_bytes, uint64_t* d2h_bytes) {
    if (!ctx) { set_error("null argument"); return Z2B_ERR_ARG; }
    if (h2d_bytes) *h2d_bytes = ctx->c->last_h2d;
    if (d2h_bytes) *d2h_bytes = ctx->c->last_d2h;
    return Z2B_OK;
}

int z2b_set_logits_readback(z2b_ctx* ctx, int enable) {
    if (!ctx) { set_error("null argument"); return Z2B_ERR_ARG; }
    ctx->c->keep_logits = enable != 0;
    return Z2B_OK;
}

int z2b_last_codes(z2b_ctx* ctx, int32_t* out, int n) {
    if (!ctx || !out) { set_error("null argument"); return Z2B_ERR_ARG; }
    Ctx* c = ctx->c;
    if (n < 0 || n > c->O_max) { set_error("row count out of range"); return Z2B_ERR_ARG; }
    cudaSetDevice(c->m->device);
    const size_t bytes = (size_t)n * c->m->dims.n_codebooks * 4;
    if (cudaMemcpyAsync(out, c->B.codes, bytes, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess ||
        cudaStreamSynchronize(c->stream) != cudaSuccess) { set_error("cudaMemcpy failed"); return Z2B_ERR_CUDA; }
    return Z2B_OK;
}

int z2b_last_step_active(const z2b_ctx* ctx, int32_t* out, int cap) {
    if (!ctx) return -1;
    const int L = ctx->c->m->dims.n_layer;
    for (int i = 0; i < L && i < cap; ++i) out[i] = (int32_t)ctx->c->h_misc[1 + i];
    return L;
}

int z2b_time_expert_gemv(z2b_ctx* ctx, int which, int reps, double* ms_per_launch, uint64_t* bytes_per_launch) {
    if (!ctx || !ms_per_launch || !bytes_per_launch || which < 0 || which > 1) { set_error("bad argument"); return Z2B_ERR_ARG; }
    cudaSetDevice(ctx->c->m->device);
    return ctx_time_expert_gemv(ctx->c, which, reps, ms_per_launch, bytes_per_launch);
}

int z2b_expert_op(z2b_ctx* ctx, int layer, const float* x, int T, const int32_t* sel, const float* selw, int k,
                  float* out, int reps, double* ms, uint64_t* weight_bytes, int32_t* n_gemm_experts) {
    if (!ctx) { set_error("null argument"); return Z2B_ERR_ARG; }
    cudaSetDevice(ctx->c->m->device);
    int ng = 0;
    const int rc = ctx_expert_op(ctx->c, layer, x, T, sel, selw, k, out, reps, ms, weight_bytes, &ng);
    if (n_gemm_experts) *n_gemm_experts = ng;
    return rc;
}

int z2b_set_expert_gemm_min(z2b_ctx* ctx, int routes) {
    if (!ctx) { set_error("null argument"); return Z2B_ERR_ARG; }
    return ctx_set_expert_gemm_min(ctx->c, routes);
}

int z2b_debug_fill_kv(z2b_ctx* ctx, int slot, int n, uint32_t seed) {
    if (!ctx) { set_error("null argument"); return Z2B_ERR_ARG; }
    cudaSetDevice(ctx->c->m->device);
    return ctx_debug_fill_kv(ctx->c, slot, n, seed);
}

int z2b_debug_router_capture(z2b_ctx* ctx, int enable) {
    if (!ctx) { set_error("null argument"); return Z2B_ERR_ARG; }
    cudaSetDevice(ctx->c->m->device);
    return ctx_debug_router_capture(ctx->c, enable);
}

int z2b_debug_router_inputs(z2b_ctx* ctx, int layer, float* res, float* state, int* T) {
    if (!ctx) { set_error("null argument"); return Z2B_ERR_ARG; }
    cudaSetDevice(ctx->c->m->device);
    return ctx_debug_router_inputs(ctx->c, layer, res, state, T);
}

int z2b_slot_after_frame(const z2b_hparams* hp, z2b_slot_state* s, const int32_t* codes, int max_frames, int keep) {
    if (!hp || !s || !codes || hp->n_codebooks < 1 || hp->n_codebooks + 1 > Z2B_MAX_ROW) {
        set_error("slot_after_frame: bad argument");
        return -1;
    }
    const int ncb = (int)hp->n_codebooks;
    const int frame_idx = s->step;
    int max_eoa = -1;                                   // last codebook holding end-of-audio
    for (int cb = 0; cb < ncb; ++cb)
        if (codes[cb] == (int32_t)hp->eoa_id) max_eoa = cb;
    if (s->eos_frame < 0 && max_eoa >= 0) {
        s->eos_frame = std::max(0, frame_idx - max_eoa);
        s->countdown = ncb + 1;
    }
    bool finished = false;
    if (s->countdown > 0) finished = --s->countdown == 0;
    for (int cb = 0; cb < ncb; ++cb) s->next_ids[cb] = codes[cb];
    s->next_ids[ncb] = (int32_t)hp->text_vocab;
    s->step += 1;
    if (!keep || finished || s->step >= max_frames) s->done = 1;
    return keep ? 1 : 0;
}

const char* z2b_last_error(void) { return last_error(); }

int z2b_debug_last_sel(z2b_ctx* ctx, int32_t* out, int cap) {
    if (!ctx) return -1;
    Ctx* c = ctx->c;
    const int L = c->m->dims.n_layer, T = c->last_T, k = c->kmax;
    const int need = L * T * k;
    if (out && cap >= need) {
        cudaSetDevice(c->m->device);
        for (int l = 0; l < L; ++l)
            if (cudaMemcpy(out + (size_t)l * T * k, c->B.sel_log + (size_t)l * c->T_max * k, (size_t)T * k * 4,
                           cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    }
    return need;
}

}  // extern "C"
