// runtime.cpp — batch context and the decode step (host side).
//
// Replaces the continuous-batching runtime of src/zonos2-graph.cpp:606-870. Differences
// by design: the KV cache is a pool of 256-token pages allocated to slots on demand
// (the reference reserves a fixed band per slot); a step carries only active streams
// (no ladder of fixed-width graphs, no idle columns, no dense mask); prompt rows and
// decode rows can share a step; sampling runs on the device after the head.
#include "runtime.h"

#include <algorithm>
#include <memory>
#include <cstring>
#include <random>

namespace z2b {

namespace {

thread_local std::string g_err;

#define CK(x) do { cudaError_t e_ = (x); if (e_ != cudaSuccess) { set_error(std::string(#x) + ": " + cudaGetErrorString(e_)); return Z2B_ERR_CUDA; } } while (0)

template <class T> T* carve(uint8_t*& p, size_t n) {
    T* r = reinterpret_cast<T*>(p);
    p += (n * sizeof(T) + 255) / 256 * 256;
    return r;
}

}  // namespace

void set_error(const std::string& e) { g_err = e; }
const char* last_error() { return g_err.c_str(); }

Ctx::~Ctx() {
    if (stream) cudaStreamSynchronize(stream);
    for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
    if (d_canon_all) cudaFree(d_canon_all);
    if (h_canon_all) cudaFreeHost(h_canon_all);
    if (d_spk) cudaFree(d_spk);
    if (d_rcap) cudaFree(d_rcap);
    if (d_sched_descs) cudaFree(d_sched_descs);
    if (d_sched_src) cudaFree(d_sched_src);
    if (d_sched_rows) cudaFree(d_sched_rows);
    for (cudaEvent_t e : prof_ev) cudaEventDestroy(e);
    for (void* p : dallocs) cudaFree(p);
    for (void* p : hallocs) cudaFreeHost(p);
    if (stream) cudaStreamDestroy(stream);
}

int ctx_create(Model* m, int n_slots, int slot_cap_frames, Ctx** out, int out_rows) {
    if (n_slots < 1 || n_slots > 1024 || slot_cap_frames < 1) { set_error("bad n_slots / slot_cap"); return Z2B_ERR_ARG; }
    std::unique_ptr<Ctx> c(new Ctx());
    c->m = m;
    if (cudaSetDevice(m->device) != cudaSuccess) { set_error("cudaSetDevice failed"); return Z2B_ERR_CUDA; }
    CK(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
    const Dims& D = m->dims;
    c->n_slots = n_slots;
    c->slot_cap = (slot_cap_frames + PAGE - 1) / PAGE * PAGE;
    c->pages_per_slot = c->slot_cap / PAGE;
    // rows per step: every slot decoding plus 4096 prompt rows admitted in the same step
    // (eight 512-row prompts, or one 4096-token expert-op batch), at most 8192
    c->T_max = std::min(8192, std::max(512, n_slots + 4096));
    c->O_max = std::max(n_slots, std::min(out_rows, c->T_max));
    c->D_max = std::min(1024, c->T_max);
    c->kmax = 1;
    for (auto& ly : m->layers) c->kmax = std::max(c->kmax, ly.top_k);
    c->R_max = c->T_max * c->kmax;
    // keys per attention split: 256 (one KV page), doubled until the split combine's
    // per-head weights fit the kernel's merge area (2 G max_split + G <= 32 (hd + 2))
    c->split_keys = 256;
    {
        const int G = m->dims.n_head / m->dims.n_head_kv, hd = m->dims.head_dim;
        while (2 * G * ((c->slot_cap + c->split_keys - 1) / c->split_keys) + G > 32 * (hd + 2)) c->split_keys *= 2;
    }
    c->max_split = (c->slot_cap + c->split_keys - 1) / c->split_keys;
    const int d = D.n_embd, hd = D.head_dim, nh = D.n_head, nkv = D.n_head_kv, ncb = D.n_codebooks, av = D.audio_vocab;

    // KV pool: every slot can reach its full capacity
    c->n_pages = n_slots * c->pages_per_slot;
    c->head_elems = (size_t)PAGE * hd;
    c->layer_elems = 2 * (size_t)nkv * c->head_elems;
    c->page_elems = (size_t)D.n_layer * c->layer_elems;
    auto dal = [&](size_t n) -> void* {
        void* p = nullptr;
        if (cudaMalloc(&p, n ? n : 16) != cudaSuccess) return nullptr;
        c->dallocs.push_back(p);
        return p;
    };
    c->kv_pool = (__half*)dal((size_t)c->n_pages * c->page_elems * sizeof(__half));
    if (!c->kv_pool) { set_error("KV pool allocation failed (" + std::to_string(c->n_pages) + " pages)"); return Z2B_ERR_OOM; }
    CK(cudaMemset(c->kv_pool, 0, (size_t)c->n_pages * c->page_elems * sizeof(__half)));
    c->free_pages.resize(c->n_pages);
    for (int i = 0; i < c->n_pages; ++i) c->free_pages[i] = c->n_pages - 1 - i;
    c->slot_pages.assign(n_slots, {});
    c->h_pt.assign((size_t)n_slots * c->pages_per_slot, -1);

    // staging (host pinned + device mirror): page table | descs | ids | canon
    c->st_pt = 0;
    c->st_descs = (size_t)n_slots * c->pages_per_slot * 4;
    c->st_descs = (c->st_descs + 255) / 256 * 256;
    c->st_ids = c->st_descs + (size_t)c->D_max * sizeof(SlotDesc);
    c->st_ids = (c->st_ids + 255) / 256 * 256;
    c->st_canon = c->st_ids + (size_t)c->T_max * NCOL * 4;
    c->st_canon = (c->st_canon + 255) / 256 * 256;
    c->st_bytes = c->st_canon + (size_t)c->O_max * ncb * 8;
    CK(cudaMallocHost(&c->h_stage, c->st_bytes));
    c->hallocs.push_back(c->h_stage);
    c->d_stage = (uint8_t*)dal(c->st_bytes);
    if (!c->d_stage) { set_error("staging allocation failed"); return Z2B_ERR_OOM; }
    std::memset(c->h_stage, 0, c->st_bytes);

    // per-step device buffers
    const size_t ldq = (size_t)nh * hd + 2 * (size_t)nkv * hd + nh;
    size_t need = 0;
    auto acc = [&](size_t bytes) { need += (bytes + 255) / 256 * 256; };
    const int T = c->T_max, R = c->R_max + 8 * MAX_EXPERTS, O = c->O_max;
    acc(T * 4); acc(T * 4); acc(T * 4); acc(T * NCOL * 4); acc(O * 4); acc(O * 4); acc(T * 4); acc(c->D_max * 4);
    acc((size_t)T * d * 4); acc((size_t)T * d * 2); acc((size_t)T * ldq * 4); acc((size_t)T * nh * hd * 2);
    acc((size_t)T * nh * c->max_split * (hd + 2) * 4); acc((size_t)T * nh * hd * 2); acc((size_t)T * std::max(D.rd, 1) * 4);
    acc((size_t)T * c->kmax * 4); acc((size_t)T * c->kmax * 4);
    acc(4); acc(MAX_EXPERTS * 4); acc((MAX_EXPERTS + 1) * 4); acc((size_t)R * 4); acc((size_t)R * 4); acc((size_t)T * c->kmax * 4);
    acc(4); acc((size_t)R * D.n_ff * 2); acc((size_t)R * d * 4); acc((size_t)O * d * 2);
    acc((size_t)O * ncb * av * 4); acc((size_t)O * ncb * 4); acc(D.n_layer * 4); acc(4);
    acc((size_t)D.n_layer * T * c->kmax * 4);
    acc((size_t)4 * T * std::max(D.rd, 1) * 4);
    acc((size_t)T * nkv * 4);
    // tensor-core GEMM activations in stage order: projection rows, or one row per route
    const size_t gx = std::max((size_t)T * std::max((size_t)d, (size_t)nh * hd), (size_t)R * std::max(D.n_ff, d));
    acc(gx * 2);
    acc((MAX_EXPERTS + 1) * 4);
    acc(4);
    acc(MAX_EXPERTS * 4);
    acc((size_t)T * c->max_split * 8); acc(4);
    uint8_t* base = (uint8_t*)dal(need);
    if (!base) { set_error("step buffer allocation failed"); return Z2B_ERR_OOM; }
    CK(cudaMemset(base, 0, need));
    uint8_t* p = base;
    StepBufs& B = c->B;
    B.descs = (const SlotDesc*)(c->d_stage + c->st_descs);
    B.ids_in = (const int*)(c->d_stage + c->st_ids);
    B.canon = (const double*)(c->d_stage + c->st_canon);
    B.tok_slot = carve<int>(p, T); B.tok_pos = carve<int>(p, T); B.tok_desc = carve<int>(p, T);
    B.ids = carve<int>(p, (size_t)T * NCOL); B.out_tok = carve<int>(p, O); B.out_desc = carve<int>(p, O);
    B.tok_out = carve<int>(p, T); B.desc_out = carve<int>(p, c->D_max);
    B.res = carve<float>(p, (size_t)T * d); B.cur = carve<__half>(p, (size_t)T * d);
    B.qkvg = carve<float>(p, (size_t)T * ldq); B.ldq = (int)ldq;
    B.qh = carve<__half>(p, (size_t)T * nh * hd);
    B.apart = carve<float>(p, (size_t)T * nh * c->max_split * (hd + 2)); B.max_split = c->max_split;
    B.o = carve<__half>(p, (size_t)T * nh * hd);
    B.rstate = carve<float>(p, (size_t)T * std::max(D.rd, 1));
    B.rpart = carve<float>(p, (size_t)4 * T * std::max(D.rd, 1)); B.rpart_T = T;
    B.sel = carve<int>(p, (size_t)T * c->kmax); B.selw = carve<float>(p, (size_t)T * c->kmax); B.kmax = c->kmax;
    B.n_active = carve<int>(p, 1); B.active = carve<int>(p, MAX_EXPERTS); B.seg_off = carve<int>(p, MAX_EXPERTS + 1);
    B.route_tok = carve<int>(p, R); B.route_w = carve<float>(p, R); B.route_pos = carve<int>(p, (size_t)T * c->kmax);
    B.ticket = carve<int>(p, 1);
    B.y = carve<__half>(p, (size_t)R * D.n_ff); B.out_route = carve<float>(p, (size_t)R * d);
    B.hout = carve<__half>(p, (size_t)O * d); B.logits = carve<float>(p, (size_t)O * ncb * av);
    B.codes = carve<int>(p, (size_t)O * ncb); B.layer_active = carve<int>(p, D.n_layer);
    B.err = carve<uint32_t>(p, 1);
    B.sel_log = carve<int>(p, (size_t)D.n_layer * T * c->kmax); B.sel_log_T = T;
    B.attn_ticket = carve<int>(p, (size_t)T * nkv);
    B.gemm_x = carve<__half>(p, gx);
    B.tile_off = carve<int>(p, MAX_EXPERTS + 1);
    B.n_small = carve<int>(p, 1);
    B.seg_mid = carve<int>(p, MAX_EXPERTS);
    B.attn_items = carve<int2>(p, (size_t)T * c->max_split);
    B.attn_n_items = carve<int>(p, 1);
    B.split_keys = c->split_keys;

    c->kv.pool = c->kv_pool;
    c->kv.page_table = (const int*)(c->d_stage + c->st_pt);
    c->kv.max_pages = c->pages_per_slot;
    c->kv.page_elems = c->page_elems;
    c->kv.layer_elems = c->layer_elems;
    c->kv.head_elems = c->head_elems;

    // sampler state
    c->d_samp = (SampDev*)dal((size_t)n_slots * sizeof(SampDev));
    c->hist_cap = Z2B_MAX_REP_WINDOW;
    c->d_hist = (int*)dal((size_t)n_slots * ncb * c->hist_cap * 4);
    c->d_hist_len = (int*)dal((size_t)n_slots * ncb * 4);
    if (!c->d_samp || !c->d_hist || !c->d_hist_len) { set_error("sampler state allocation failed"); return Z2B_ERR_OOM; }
    CK(cudaMemset(c->d_hist_len, 0, (size_t)n_slots * ncb * 4));
    c->h_samp.resize(n_slots);
    c->greedy.assign(n_slots, 1);
    c->rng.resize(n_slots);
    for (int i = 0; i < n_slots; ++i) {
        SampDev& s = c->h_samp[i];
        s.temperature = 1.15f; s.top_k = 106; s.top_p = 0.0f; s.min_p = 0.18f; s.rep_penalty = 1.2f;
        s.rep_window = 50; s.rep_codebooks = 8; s.greedy = 1;
        c->rng[i].seed(0);
    }
    CK(cudaMemcpy(c->d_samp, c->h_samp.data(), (size_t)n_slots * sizeof(SampDev), cudaMemcpyHostToDevice));

    // pinned outputs
    CK(cudaMallocHost(&c->h_codes, (size_t)O * ncb * 4)); c->hallocs.push_back(c->h_codes);
    CK(cudaMallocHost(&c->h_logits, (size_t)O * ncb * av * 4)); c->hallocs.push_back(c->h_logits);
    CK(cudaMallocHost(&c->h_misc, 4096)); c->hallocs.push_back(c->h_misc);
    c->step_logits.assign((size_t)c->D_max * ncb * av, 0.0f);
    c->step_has_logits.assign(c->D_max, 0);
    *out = c.release();
    return Z2B_OK;
}

int ctx_slot_reset(Ctx* c, int slot, const z2b_sampling* sp) {
    if (slot < 0 || slot >= c->n_slots) { set_error("slot out of range"); return Z2B_ERR_ARG; }
    for (int pg : c->slot_pages[slot]) c->free_pages.push_back(pg);
    c->slot_pages[slot].clear();
    for (int i = 0; i < c->pages_per_slot; ++i) c->h_pt[(size_t)slot * c->pages_per_slot + i] = -1;
    return ctx_set_sampling(c, slot, sp);
}

int ctx_set_sampling(Ctx* c, int slot, const z2b_sampling* sp) {
    if (slot < 0 || slot >= c->n_slots) { set_error("slot out of range"); return Z2B_ERR_ARG; }
    SampDev& s = c->h_samp[slot];
    if (sp) {
        if (sp->rep_window < 0 || sp->rep_window > Z2B_MAX_REP_WINDOW) { set_error("rep_window out of range"); return Z2B_ERR_ARG; }
        s.temperature = sp->temperature; s.top_k = sp->top_k; s.top_p = sp->top_p; s.min_p = sp->min_p;
        s.rep_penalty = sp->rep_penalty; s.rep_window = sp->rep_window; s.rep_codebooks = sp->rep_codebooks;
        s.greedy = sp->greedy ? 1 : 0;
        c->rng[slot].seed(sp->seed);
    } else {
        s.greedy = 1;
        c->rng[slot].seed(0);
    }
    c->greedy[slot] = s.greedy;
    const int ncb = c->m->dims.n_codebooks;
    CK(cudaMemcpyAsync(c->d_samp + slot, &s, sizeof(SampDev), cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemsetAsync(c->d_hist_len + (size_t)slot * ncb, 0, (size_t)ncb * 4, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    return Z2B_OK;
}

// ---------------------------------------------------------------- launch sequence

namespace {

// Event pair around each launch when profiling (eager steps only).
struct ProfScope {
    Ctx* c; int cls; cudaEvent_t e1 = nullptr;
    ProfScope(Ctx* c_, int cls_) : c(c_), cls(cls_) {
        if (!c->profiling) return;
        if (c->prof_used + 2 > c->prof_ev.size()) {
            for (int i = 0; i < 256; ++i) { cudaEvent_t e; cudaEventCreate(&e); c->prof_ev.push_back(e); }
        }
        cudaEventRecord(c->prof_ev[c->prof_used], c->stream);
        e1 = c->prof_ev[c->prof_used + 1];
        c->prof_class.push_back(cls);
        c->prof_used += 2;
    }
    ~ProfScope() { if (c->profiling) cudaEventRecord(e1, c->stream); }
};

// The tensor-core GEMM could not be set up (its activation TMA view was rejected): the
// step's results would be incomplete, so the call that enqueued it fails.
void gemm_setup_failed(Ctx* c) {
    set_error("tensor-core GEMM: activation tensor map could not be encoded");
    c->enq_failed = true;
}

// Tensor-core GEMM token tile (routes or rows per tile, a multiple of 8 up to 248) for a
// launch over `rows` token rows (for the expert passes, routes / 4): 248 from 1024 rows,
// where each dequantised weight block then serves the most tokens and the tiles still
// outnumber the blocks; else 120, whose smaller, more numerous tiles keep the 148 blocks
// evenly loaded.
int gemm_token_tile(int rows) { return rows >= 1024 ? 248 : 120; }

int ctas_per_sm(int smem) { return std::max(1, std::min(4, 233472 / (smem + 1024))); }

// Projection of T rows (tokens or output rows). With t_dec >= 0 the rows are a step's
// tokens, decode rows [0, t_dec) first: when the prompt rows [t_dec, T) are many, they run
// on the tensor-core GEMM and the tile GEMV keeps the decode rows, so a decode row's result
// never depends on what else the step carries.
void gemv_proj(Ctx* c, const DevMat* const* mats, const int* offs, int nmat, int T, const __half* X, int ldx,
               float* out, int ldo, int epi, float cap, int cls, int t_dec = -1) {
    ProfScope ps(c, cls);
    bool gemm_ok = t_dec >= 0 && T - t_dec >= PROJ_GEMM_MIN_ROWS;
    for (int i = 0; i < nmat; ++i) gemm_ok = gemm_ok && moe_gemm_supported(*mats[i]);
    const int T_gemv = gemm_ok ? t_dec : T;
    GemvParams p{};
    p.mode = GM_PROJ; p.epi = epi;
    p.type = mats[0]->type; p.K = mats[0]->K; p.chunks = mats[0]->chunks;
    p.tile_bytes = mats[0]->tile_bytes; p.steps = mats[0]->steps;
    p.n_seg = nmat;
    int items = 0;
    for (int i = 0; i < nmat; ++i) {
        p.seg[i] = ProjSeg{mats[i]->tiles, mats[i]->n_row_tiles, mats[i]->rows, offs[i]};
        items += mats[i]->n_row_tiles;
    }
    p.total_items = items;
    p.X = X; p.ldx = ldx; p.T = T_gemv; p.out = out; p.ldo = ldo; p.cap = cap; p.err = c->B.err;
    if (T_gemv > 0) {
        int nw, smem;
        gemv_geometry(*mats[0], 1, 2, &nw, &p.n_stages, &p.stage_bytes, &smem, &p.cps, &p.x_rs);
        const int grid = std::min(items, c->m->n_sm * ctas_per_sm(smem));
        launch_gemv(p, nw, grid, smem, c->stream);
        c->launches++;
    }
    if (gemm_ok) {
        p.tok0 = t_dec;
        p.T = T - t_dec;
        p.x_rows = T;
        p.x_row0 = t_dec;
        p.gm_nt = gemm_token_tile(T - t_dec);
        p.xperm = c->B.gemm_x;
        if (!launch_moe_gemm(p, c->m->n_sm, c->stream)) gemm_setup_failed(c);
        c->launches++;
    }
}

// Expert pass (gate/up + SwiGLU, or down x route weight) over the routes of the step:
// the tile GEMV takes each expert's routes [seg_off, seg_mid); when the step can have
// routes for the tcgen05 GEMM (bulk: prompt rows, or a large expert-op batch) the GEMM
// takes [seg_mid, seg_off + 1).
// Expert segment arrays a pass reads (the step buffers' own, or a saved copy).
struct SegSet {
    const int *n_active, *n_small, *active, *seg_off, *seg_mid, *tile_off, *route_tok;
    const float* route_w;
};

SegSet step_segs(const StepBufs& B) {
    return SegSet{B.n_active, B.n_small, B.active, B.seg_off, B.seg_mid, B.tile_off, B.route_tok, B.route_w};
}

void gemv_moe(Ctx* c, const LayerDev& ly, int mode, bool bulk, const SegSet* segs = nullptr) {
    ProfScope ps(c, mode == GM_GATEUP ? PC_GATEUP : PC_DOWN);
    const SegSet sg = segs ? *segs : step_segs(c->B);
    const Dims& D = c->m->dims;
    GemvParams p{};
    const DevMat& w0 = mode == GM_GATEUP ? ly.gate_exps : ly.down_exps;
    p.mode = mode; p.epi = EPI_STORE;
    p.type = w0.type; p.K = w0.K; p.chunks = w0.chunks; p.tile_bytes = w0.tile_bytes; p.steps = w0.steps;
    p.n_row_tiles = w0.n_row_tiles;
    p.w0 = w0.tiles;
    p.w1 = mode == GM_GATEUP ? ly.up_exps.tiles : nullptr;
    p.expert_stride = w0.expert_stride;
    const bool split = bulk && ly.small.gemm_ok;
    p.n_active = sg.n_small;
    p.n_small = sg.n_small;
    p.active = sg.active; p.seg_off = sg.seg_off; p.seg_mid = sg.seg_mid; p.tile_off = sg.tile_off;
    p.route_tok = sg.route_tok; p.route_w = sg.route_w;
    if (mode == GM_GATEUP) {
        p.X = c->B.cur; p.ldx = D.n_embd; p.yout = c->B.y; p.ldy = D.n_ff; p.out_rows = D.n_ff;
    } else {
        p.X = c->B.y; p.ldx = D.n_ff; p.out = c->B.out_route; p.ldo = D.n_embd; p.out_rows = D.n_embd;
    }
    p.err = c->B.err;
    int nw, smem;
    gemv_geometry(w0, mode == GM_GATEUP ? 2 : 1, mode == GM_GATEUP ? 2 : 1, &nw, &p.n_stages, &p.stage_bytes, &smem,
                  &p.cps);
    // blocks per SM the kernel is built for: two for gate/up, three for down
    const int grid = c->m->n_sm * std::min(mode == GM_GATEUP ? 2 : 3, ctas_per_sm(smem));
    launch_gemv(p, nw, grid, smem, c->stream);
    c->launches++;
    if (split) {
        p.n_active = sg.n_active;
        p.x_rows = c->cur_T * c->kmax;                 // one row per route
        p.x_row0 = 0;
        p.gm_nt = gemm_token_tile(c->cur_T * c->kmax / 4);
        p.n_routes = sg.seg_off + ly.n_expert;
        p.xperm = c->B.gemm_x;
        if (!launch_moe_gemm(p, c->m->n_sm, c->stream)) gemm_setup_failed(c);
        c->launches++;
    }
}

}  // namespace


void enqueue_step(Ctx* c, int T, int n_out) {
    c->cur_T = T;
    Model* m = c->m;
    const Dims& D = m->dims;
    StepBufs B = c->B;
    B.n_desc = c->cur_n_desc;
    c->launches = 0;
    { ProfScope ps(c, PC_PACK); launch_pack(B, T, n_out, c->stream); c->launches++; }
    {
        ProfScope ps(c, PC_EMBED);
        const float* spk_row = c->d_spk ? c->d_spk + m->hp.spk_dim + D.n_embd : nullptr;
        launch_embed(B, m->emb, m->layers[0].small.attn_norm, D, T, c->spk_t, spk_row, c->stream);
        c->launches++;
    }
    const int hd = D.head_dim, nh = D.n_head, nkv = D.n_head_kv;
    bool first_moe = true;
    for (int L = 0; L < D.n_layer; ++L) {
        const LayerDev& ly = m->layers[L];
        if (ly.qkvg_fused) {
            const DevMat* mats[4] = {&ly.wq, &ly.wk, &ly.wv, &ly.wgate};
            const int offs[4] = {0, nh * hd, nh * hd + nkv * hd, nh * hd + 2 * nkv * hd};
            gemv_proj(c, mats, offs, 4, T, B.cur, D.n_embd, B.qkvg, B.ldq, EPI_STORE, 0.0f, PC_QKV, c->cur_t_dec);
        } else {
            const DevMat* mats[4] = {&ly.wq, &ly.wk, &ly.wv, &ly.wgate};
            const int offs[4] = {0, nh * hd, nh * hd + nkv * hd, nh * hd + 2 * nkv * hd};
            for (int i = 0; i < 4; ++i)
                gemv_proj(c, &mats[i], &offs[i], 1, T, B.cur, D.n_embd, B.qkvg, B.ldq, EPI_STORE, 0.0f, PC_QKV,
                          c->cur_t_dec);
        }
        { ProfScope ps(c, PC_ROPE); launch_rope_append(B, c->kv, ly.small.attn_temp, D, L, T, c->stream); c->launches++; }
        { ProfScope ps(c, PC_ATTN); launch_attention(B, c->kv, D, L, T, c->split_keys, c->max_split, c->stream); c->launches++; }
        {
            const DevMat* mats[1] = {&ly.wo};
            const int offs[1] = {0};
            gemv_proj(c, mats, offs, 1, T, B.o, nh * hd, B.res, D.n_embd, EPI_ADD, 0.0f, PC_WO, c->cur_t_dec);
        }
        if (c->rcap_on && c->d_rcap && ly.is_moe) {
            const size_t per = (size_t)D.n_embd + D.rd;
            float* rec = c->d_rcap + (size_t)L * c->T_max * per;
            cudaMemcpyAsync(rec, B.res, (size_t)T * D.n_embd * 4, cudaMemcpyDeviceToDevice, c->stream);
            cudaMemcpyAsync(rec + (size_t)c->T_max * D.n_embd, B.rstate, (size_t)T * D.rd * 4, cudaMemcpyDeviceToDevice,
                            c->stream);
        }
        { ProfScope ps(c, PC_ROUTER); launch_router(B, ly.small, D, T, (ly.is_moe && first_moe) ? 1 : 0, L, c->stream); c->launches += router_launches(ly.small); }
        if (ly.is_moe) first_moe = false;
        const bool bulk = T > c->cur_n_desc;                 // the step carries prompt rows
        gemv_moe(c, ly, GM_GATEUP, bulk);
        gemv_moe(c, ly, GM_DOWN, bulk);
        const bool last = L == D.n_layer - 1;
        {
            ProfScope ps(c, PC_COMBINE);
            launch_moe_combine(B, ly.small, last ? nullptr : m->layers[L + 1].small.attn_norm, m->out_norm, D, T,
                               last ? 1 : 0, c->stream);
            c->launches++;
        }
    }
    if (n_out > 0) {
        const DevMat* mats[1] = {&m->head};
        const int offs[1] = {0};
        gemv_proj(c, mats, offs, 1, n_out, B.hout, D.n_embd, B.logits, D.n_codebooks * D.audio_vocab, EPI_SOFTCAP,
                  D.softcap, PC_HEAD);
        ProfScope ps(c, PC_SAMPLER);
        launch_sampler(B, c->d_samp, c->d_hist, c->d_hist_len, c->hist_cap, D, n_out, c->stream);
        c->launches++;
    }
}

int run_step(Ctx* c, int T, int n_out) {
    // Every launch of a step is fixed by (rows, output rows, descriptors, decode rows): steps
    // replay a CUDA graph per such shape. Decode-only shapes are captured at once; a shape
    // carrying prompt rows on its second occurrence (repeated refill shapes replay, one-off
    // prompt lengths run eagerly), up to kMaxPromptGraphs of them.
    constexpr int kMaxPromptGraphs = 32;
    bool use_graph = c->graphs_enabled && !c->profiling && !c->rcap_on && c->spk_t < 0;
    const uint64_t key = ((uint64_t)T << 32) | (uint32_t)n_out | ((uint64_t)c->cur_n_desc << 48) |
                         ((uint64_t)c->cur_t_dec << 16);
    auto it = c->graphs.find(key);
    if (use_graph && T != c->cur_n_desc && it == c->graphs.end())
        use_graph = ++c->shape_seen[key] >= 2 && c->prompt_graphs < kMaxPromptGraphs;
    c->enq_failed = false;
    if (!use_graph) {
        enqueue_step(c, T, n_out);
        return c->enq_failed ? Z2B_ERR_CUDA : Z2B_OK;
    }
    if (it == c->graphs.end()) {
        if (T != c->cur_n_desc) c->prompt_graphs++;
        cudaGraph_t g;
        CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeRelaxed));
        enqueue_step(c, T, n_out);
        CK(cudaStreamEndCapture(c->stream, &g));
        if (c->enq_failed) { cudaGraphDestroy(g); return Z2B_ERR_CUDA; }
        cudaGraphExec_t ge;
        const cudaError_t e = cudaGraphInstantiate(&ge, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) { set_error(std::string("cudaGraphInstantiate: ") + cudaGetErrorString(e)); return Z2B_ERR_CUDA; }
        it = c->graphs.emplace(key, ge).first;
        c->graph_launches[key] = c->launches;
    }
    c->launches = c->graph_launches[key];
    CK(cudaGraphLaunch(it->second, c->stream));
    return Z2B_OK;
}

// ---------------------------------------------------------------- step API

int ctx_prepare(Ctx* c, const z2b_slot_desc* descs, int n, int extra_rows_per_desc, int* T_out, int* n_out_out) {
    const Dims& D = c->m->dims;
    if (n < 1 || n > c->D_max) { set_error("number of descs out of range"); return Z2B_ERR_ARG; }
    int T = 0, n_out = 0, t_dec = 0;
    std::vector<char> seen(c->n_slots, 0);
    for (int i = 0; i < n; ++i) {
        const z2b_slot_desc& d = descs[i];
        if (d.slot < 0 || d.slot >= c->n_slots) { set_error("desc slot out of range"); return Z2B_ERR_ARG; }
        if (seen[d.slot]) { set_error("slot listed twice in one step"); return Z2B_ERR_ARG; }
        seen[d.slot] = 1;
        if (d.n_new < 1 || d.n_past < 0) { set_error("desc n_new/n_past out of range"); return Z2B_ERR_ARG; }
        if (d.n_past + d.n_new + extra_rows_per_desc > c->slot_cap) { set_error("stream exceeds slot capacity"); return Z2B_ERR_ARG; }
        if (d.cfg_twin >= n || d.cfg_twin == i) { set_error("bad cfg_twin"); return Z2B_ERR_ARG; }
        T += d.n_new;
        t_dec += d.n_new == 1 ? 1 : 0;
        if (d.flags & Z2B_WANT_LOGITS) n_out += c->all_rows ? d.n_new : 1;
    }
    if (T > c->T_max) { set_error("rows per step exceed capacity (" + std::to_string(c->T_max) + ")"); return Z2B_ERR_ARG; }
    if (n_out > c->O_max) { set_error("too many output rows"); return Z2B_ERR_ARG; }
    // KV pages for every position this call can write
    for (int i = 0; i < n; ++i) {
        const z2b_slot_desc& d = descs[i];
        const int need = (d.n_past + d.n_new + extra_rows_per_desc - 1) / PAGE + 1;
        auto& pages = c->slot_pages[d.slot];
        while ((int)pages.size() < need) {
            if (c->free_pages.empty()) { set_error("KV page pool exhausted"); return Z2B_ERR_OOM; }
            const int pg = c->free_pages.back();
            c->free_pages.pop_back();
            c->h_pt[(size_t)d.slot * c->pages_per_slot + pages.size()] = pg;
            pages.push_back(pg);
        }
    }
    std::memcpy(c->h_stage + c->st_pt, c->h_pt.data(), c->h_pt.size() * 4);
    SlotDesc* sd = (SlotDesc*)(c->h_stage + c->st_descs);
    int o = 0;
    for (int i = 0; i < n; ++i) {
        const z2b_slot_desc& d = descs[i];
        SlotDesc s{};
        s.slot = d.slot; s.n_past = d.n_past; s.n_new = d.n_new;
        s.flags = ((d.flags & Z2B_WANT_LOGITS) ? SD_OUTPUT : 0) | (((d.flags & Z2B_WANT_SAMPLE) == Z2B_WANT_SAMPLE) ? SD_SAMPLE : 0);
        if (c->all_rows && (s.flags & SD_OUTPUT)) s.flags |= SD_ALL_ROWS;
        s.twin = d.cfg_twin; s.cfg_scale = d.cfg_scale; s.samp = d.slot;
        sd[i] = s;
        const int rows = (s.flags & SD_OUTPUT) ? ((s.flags & SD_ALL_ROWS) ? d.n_new : 1) : 0;
        c->desc_out_host[i] = rows ? o + rows - 1 : -1;                // the desc's last row
        o += rows;
    }
    (void)D;
    c->cur_n_desc = n;
    c->cur_t_dec = t_dec;
    *T_out = T;
    *n_out_out = n_out;
    return Z2B_OK;
}

// host-drawn uniforms for non-greedy sampling: one per (sampled stream, codebook) in
// codebook order, exactly as std::uniform_real_distribution<double> consumes mt19937
// in zonos2_sampler::sample (src/zonos2-sampler.cpp:73-74)
void draw_canon(Ctx* c, const z2b_slot_desc* descs, int n, double* dst) {
    const int ncb = c->m->dims.n_codebooks;
    for (int i = 0; i < n; ++i) {
        const int o = c->desc_out_host[i];
        if (o < 0) continue;
        const bool sample = (descs[i].flags & Z2B_WANT_SAMPLE) == Z2B_WANT_SAMPLE;
        for (int cb = 0; cb < ncb; ++cb)
            dst[(size_t)o * ncb + cb] = (sample && !c->greedy[descs[i].slot])
                ? std::generate_canonical<double, 53>(c->rng[descs[i].slot]) : 0.0;
    }
}

int ctx_step(Ctx* c, const z2b_slot_desc* descs, int n, const int32_t* ids, int32_t* out_codes, float* out_logits) {
    const Dims& D = c->m->dims;
    if (!descs || !ids) { set_error("null argument"); return Z2B_ERR_ARG; }
    int T, n_out;
    c->desc_out_host.assign(std::max(n, 1), -1);
    int rc = ctx_prepare(c, descs, n, 0, &T, &n_out);
    if (rc) return rc;
    std::memcpy(c->h_stage + c->st_ids, ids, (size_t)T * NCOL * 4);
    draw_canon(c, descs, n, (double*)(c->h_stage + c->st_canon));
    const int ncb = D.n_codebooks, av = D.audio_vocab;
    // inputs: only the used part of each staging section
    const size_t b_pt = c->h_pt.size() * 4, b_desc = (size_t)n * sizeof(SlotDesc), b_ids = (size_t)T * NCOL * 4,
                 b_canon = (size_t)n_out * ncb * 8;
    CK(cudaMemcpyAsync(c->d_stage + c->st_pt, c->h_stage + c->st_pt, b_pt, cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(c->d_stage + c->st_descs, c->h_stage + c->st_descs, b_desc, cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(c->d_stage + c->st_ids, c->h_stage + c->st_ids, b_ids, cudaMemcpyHostToDevice, c->stream));
    if (b_canon) CK(cudaMemcpyAsync(c->d_stage + c->st_canon, c->h_stage + c->st_canon, b_canon, cudaMemcpyHostToDevice, c->stream));
    c->last_h2d = b_pt + b_desc + b_ids + b_canon;
    rc = run_step(c, T, n_out);
    if (rc) return rc;
    c->last_d2h = 4 + (size_t)D.n_layer * 4;
    if (n_out > 0) {
        CK(cudaMemcpyAsync(c->h_codes, c->B.codes, (size_t)n_out * ncb * 4, cudaMemcpyDeviceToHost, c->stream));
        c->last_d2h += (size_t)n_out * ncb * 4;
        if (out_logits || c->keep_logits) {
            CK(cudaMemcpyAsync(c->h_logits, c->B.logits, (size_t)n_out * ncb * av * 4, cudaMemcpyDeviceToHost, c->stream));
            c->last_d2h += (size_t)n_out * ncb * av * 4;
        }
    }
    CK(cudaMemcpyAsync(c->h_misc, c->B.err, 4, cudaMemcpyDeviceToHost, c->stream));
    CK(cudaMemcpyAsync(c->h_misc + 1, c->B.layer_active, (size_t)D.n_layer * 4, cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    const bool have_logits = out_logits || c->keep_logits;
    const uint32_t derr = c->h_misc[0];
    if (derr) { set_error("device error flags 0x" + std::to_string(derr)); return Z2B_ERR_DEVICE; }
    for (int i = 0; i < n; ++i) {
        const int o = c->desc_out_host[i];
        c->step_has_logits[i] = o >= 0 && have_logits;
        if (o < 0) continue;
        if (have_logits)
            std::memcpy(&c->step_logits[(size_t)i * ncb * av], c->h_logits + (size_t)o * ncb * av, (size_t)ncb * av * 4);
        if (out_codes) std::memcpy(out_codes + (size_t)i * ncb, c->h_codes + (size_t)o * ncb, (size_t)ncb * 4);
        if (out_logits) std::memcpy(out_logits + (size_t)i * ncb * av, c->h_logits + (size_t)o * ncb * av, (size_t)ncb * av * 4);
    }
    account(c, descs, n, T);
    c->last_T = T;
    return Z2B_OK;
}

void account(Ctx* c, const z2b_slot_desc* descs, int n, int T) {
    const Model* m = c->m;
    const Dims& D = m->dims;
    uint64_t w = m->head_bytes, kvb = 0, other = 0;
    for (int L = 0; L < D.n_layer; ++L) {
        const LayerDev& ly = m->layers[L];
        w += m->attn_bytes_per_layer;
        const int na = (int)c->h_misc[1 + L];
        if (ly.is_moe) {
            w += m->router_bytes_per_layer;
            w += (uint64_t)na * ((ly.gate_exps.gguf_bytes + ly.up_exps.gguf_bytes + ly.down_exps.gguf_bytes) / ly.n_expert);
        } else {
            w += ly.gate_exps.gguf_bytes + ly.up_exps.gguf_bytes + ly.down_exps.gguf_bytes;
        }
    }
    const uint64_t kv_tok = (uint64_t)D.n_layer * 2 * D.n_head_kv * D.head_dim * 2;
    for (int i = 0; i < n; ++i)
        for (int r = 0; r < descs[i].n_new; ++r) kvb += (uint64_t)(descs[i].n_past + r + 1) * kv_tok;
    kvb += (uint64_t)T * kv_tok;                       // writes
    other = (uint64_t)T * NCOL * m->emb_row_bytes;
    c->last_wbytes = w; c->last_kvbytes = kvb; c->last_other = other;
}

int ctx_prefill(Ctx* c, int slot, const int32_t* ids, int n0, float* out_logits) {
    if (n0 < 1 || n0 > c->slot_cap) { set_error("prefill n0 out of range"); return Z2B_ERR_ARG; }
    const int chunk = c->T_max;
    for (int off = 0; off < n0; off += chunk) {
        const int nn = std::min(chunk, n0 - off);
        const bool last = off + nn == n0;
        z2b_slot_desc d{slot, off, nn, last ? Z2B_WANT_LOGITS : 0, -1, 1.0f};
        const int rc = ctx_step(c, &d, 1, ids + (size_t)off * NCOL, nullptr, last ? out_logits : nullptr);
        if (rc) return rc;
    }
    return Z2B_OK;
}

namespace {

// The projected speaker row (+ delta) into the context's speaker buffer, on its stream.
int spk_prepare(Ctx* c, const float* spk, const float* delta) {
    const Model* m = c->m;
    const int sd = (int)m->hp.spk_dim, ld = (int)m->hp.spk_lda_dim, d = m->dims.n_embd;
    if (!c->d_spk) CK(cudaMalloc(&c->d_spk, ((size_t)sd + 2 * (size_t)d) * sizeof(float)));
    float* d_in = c->d_spk;
    float* d_delta = c->d_spk + sd;
    float* d_row = c->d_spk + sd + d;
    CK(cudaMemcpyAsync(d_in, spk, (size_t)sd * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    if (delta) CK(cudaMemcpyAsync(d_delta, delta, (size_t)d * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    launch_spk_proj(m->spk_lda_w, m->spk_lda_b, m->spk_proj_w, m->spk_proj_b, d_in, delta ? d_delta : nullptr, sd, ld,
                    d, d_row, c->stream);
    return Z2B_OK;
}

}  // namespace

int ctx_prefill_spk(Ctx* c, int slot, const int32_t* ids, int n0, const float* spk, int spk_pos, const float* delta,
                    float* out_logits) {
    // as the reference (src/zonos2-graph.cpp:36-37, 716): a negative spk_pos means no speaker
    if (!spk || spk_pos < 0) return ctx_prefill(c, slot, ids, n0, out_logits);
    if (n0 < 1 || n0 > c->slot_cap) { set_error("prefill n0 out of range"); return Z2B_ERR_ARG; }
    if (spk_pos >= n0) { set_error("spk_pos outside the prompt rows"); return Z2B_ERR_ARG; }
    const int src = spk_prepare(c, spk, delta);
    if (src) return src;
    const int chunk = c->T_max;
    for (int off = 0; off < n0; off += chunk) {
        const int nn = std::min(chunk, n0 - off);
        const bool last = off + nn == n0;
        z2b_slot_desc dsc{slot, off, nn, last ? Z2B_WANT_LOGITS : 0, -1, 1.0f};
        c->spk_t = (spk_pos >= off && spk_pos < off + nn) ? spk_pos - off : -1;
        const int rc = ctx_step(c, &dsc, 1, ids + (size_t)off * NCOL, nullptr, last ? out_logits : nullptr);
        c->spk_t = -1;
        if (rc) return rc;
    }
    return Z2B_OK;
}

int model_logits(Model* m, const int32_t* ids, int n, const float* spk, int spk_pos, const float* delta, float* out) {
    if (!ids || !out || n < 1) { set_error("logits: bad arguments"); return Z2B_ERR_ARG; }
    if (spk_pos < 0) spk = nullptr;                  // no speaker, as the reference
    if (spk && spk_pos >= n) { set_error("spk_pos outside the rows"); return Z2B_ERR_ARG; }
    constexpr int kRowsPerStep = 512;
    Ctx* c = nullptr;
    int rc = ctx_create(m, 1, n, &c, std::min(n, kRowsPerStep));
    if (rc) return rc;
    std::unique_ptr<Ctx> own(c);
    rc = ctx_slot_reset(c, 0, nullptr);
    if (rc) return rc;
    if (spk && (rc = spk_prepare(c, spk, delta))) return rc;
    c->all_rows = true;
    c->keep_logits = true;
    const size_t per = (size_t)m->dims.n_codebooks * m->dims.audio_vocab;
    const int step = std::min(c->T_max, c->O_max);
    for (int off = 0; off < n; off += step) {
        const int nn = std::min(step, n - off);
        z2b_slot_desc dsc{0, off, nn, Z2B_WANT_LOGITS, -1, 1.0f};
        c->spk_t = (spk && spk_pos >= off && spk_pos < off + nn) ? spk_pos - off : -1;
        rc = ctx_step(c, &dsc, 1, ids + (size_t)off * NCOL, nullptr, nullptr);
        c->spk_t = -1;
        if (rc) return rc;
        std::memcpy(out + (size_t)off * per, c->h_logits, (size_t)nn * per * sizeof(float));
    }
    return Z2B_OK;
}

int ctx_decode_loop(Ctx* c, const z2b_slot_desc* descs, int n, const int32_t* first_ids, int n_steps) {
    const Dims& D = c->m->dims;
    if (!descs || !first_ids || n_steps < 1) { set_error("bad decode-loop arguments"); return Z2B_ERR_ARG; }
    for (int i = 0; i < n; ++i)
        if (descs[i].n_new != 1 || (descs[i].flags & Z2B_WANT_SAMPLE) != Z2B_WANT_SAMPLE) {
            set_error("decode loop needs n_new == 1 and Z2B_WANT_SAMPLE for every stream");
            return Z2B_ERR_ARG;
        }
    int T, n_out;
    c->desc_out_host.assign(n, -1);
    int rc = ctx_prepare(c, descs, n, n_steps - 1, &T, &n_out);
    if (rc) return rc;
    const int ncb = D.n_codebooks;
    std::memcpy(c->h_stage + c->st_ids, first_ids, (size_t)T * NCOL * 4);
    // uniforms for every step, drawn in step order
    const size_t per = (size_t)n_out * ncb;
    if (c->canon_all_cap < per * n_steps) {
        if (c->d_canon_all) cudaFree(c->d_canon_all);
        if (c->h_canon_all) cudaFreeHost(c->h_canon_all);
        CK(cudaMalloc(&c->d_canon_all, per * n_steps * 8));
        CK(cudaMallocHost(&c->h_canon_all, per * n_steps * 8));
        c->canon_all_cap = per * n_steps;
    }
    for (int s = 0; s < n_steps; ++s) draw_canon(c, descs, n, c->h_canon_all + per * s);
    CK(cudaMemcpyAsync(c->d_stage, c->h_stage, c->st_bytes, cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(c->d_canon_all, c->h_canon_all, per * n_steps * 8, cudaMemcpyHostToDevice, c->stream));
    // desc_out on the device is written by the pack kernel of the first step
    SlotDesc* d_descs = (SlotDesc*)(c->d_stage + c->st_descs);
    int* d_ids = (int*)(c->d_stage + c->st_ids);
    double* d_canon = (double*)(c->d_stage + c->st_canon);
    for (int s = 0; s < n_steps; ++s) {
        launch_feed(d_descs, n, d_ids, c->B.codes, c->B.desc_out, d_canon, c->d_canon_all + per * s, ncb,
                    D.text_vocab, s > 0 ? 1 : 0, c->stream);
        rc = run_step(c, T, n_out);
        if (rc) return rc;
    }
    c->loop_launches = c->launches + 1;
    return Z2B_OK;
}

int ctx_run_schedule(Ctx* c, int n_steps, int n, const z2b_slot_desc* descs, const int32_t* rows, int n_rows,
                     const int32_t* row_src) {
    const Dims& D = c->m->dims;
    const int ncb = D.n_codebooks;
    if (n_steps < 1 || n < 1 || n > c->D_max || n > c->O_max || !descs || !row_src) { set_error("bad schedule arguments"); return Z2B_ERR_ARG; }
    std::vector<int> need(c->n_slots, 0);
    std::vector<int> T(n_steps, 0), T_dec(n_steps, 0);
    for (int s = 0; s < n_steps; ++s) {
        std::vector<char> seen(c->n_slots, 0);
        for (int i = 0; i < n; ++i) {
            const z2b_slot_desc& d = descs[(size_t)s * n + i];
            const int src = row_src[(size_t)s * n + i];
            if (d.slot < 0 || d.slot >= c->n_slots || seen[d.slot] || d.n_new < 1 || d.n_past < 0 ||
                d.n_past + d.n_new > c->slot_cap || (d.flags & Z2B_WANT_LOGITS) == 0 || d.cfg_twin >= n) {
                set_error("schedule step " + std::to_string(s) + ": invalid desc " + std::to_string(i)); return Z2B_ERR_ARG;
            }
            if (s > 0 && descs[(size_t)(s - 1) * n + i].slot != d.slot) { set_error("schedule must keep desc i on one slot"); return Z2B_ERR_ARG; }
            // at s == 0 a fed-back row continues from the previous step on this context
            if (src < 0 && d.n_new != 1) { set_error("fed-back rows need n_new == 1"); return Z2B_ERR_ARG; }
            if (src >= 0 && (rows == nullptr || src + d.n_new > n_rows)) { set_error("schedule row index out of range"); return Z2B_ERR_ARG; }
            seen[d.slot] = 1;
            need[d.slot] = std::max(need[d.slot], d.n_past + d.n_new);
            T[s] += d.n_new;
            T_dec[s] += d.n_new == 1 ? 1 : 0;
        }
        if (T[s] > c->T_max) { set_error("schedule step exceeds rows per step"); return Z2B_ERR_ARG; }
    }
    for (int sl = 0; sl < c->n_slots; ++sl) {
        auto& pages = c->slot_pages[sl];
        const int np = need[sl] ? (need[sl] - 1) / PAGE + 1 : 0;
        while ((int)pages.size() < np) {
            if (c->free_pages.empty()) { set_error("KV page pool exhausted"); return Z2B_ERR_OOM; }
            const int pg = c->free_pages.back();
            c->free_pages.pop_back();
            c->h_pt[(size_t)sl * c->pages_per_slot + pages.size()] = pg;
            pages.push_back(pg);
        }
    }
    // upload schedule
    const size_t nd = (size_t)n_steps * n;
    auto grow = [&](void** p, size_t* cap, size_t bytes) -> bool {
        if (*cap >= bytes) return true;
        if (*p) cudaFree(*p);
        *p = nullptr;
        if (cudaMalloc(p, bytes) != cudaSuccess) { *cap = 0; return false; }
        *cap = bytes;
        return true;
    };
    if (!grow((void**)&c->d_sched_descs, &c->sched_descs_cap, nd * sizeof(SlotDesc)) ||
        !grow((void**)&c->d_sched_src, &c->sched_src_cap, nd * 4) ||
        !grow((void**)&c->d_sched_rows, &c->sched_rows_cap, (size_t)std::max(n_rows, 1) * NCOL * 4)) {
        set_error("schedule buffers: cudaMalloc failed"); return Z2B_ERR_OOM;
    }
    std::vector<SlotDesc> sd(nd);
    c->desc_out_host.assign(n, 0);
    for (int i = 0; i < n; ++i) c->desc_out_host[i] = i;
    for (size_t j = 0; j < nd; ++j) {
        const z2b_slot_desc& d = descs[j];
        sd[j] = SlotDesc{d.slot, d.n_past, d.n_new,
                         SD_OUTPUT | (((d.flags & Z2B_WANT_SAMPLE) == Z2B_WANT_SAMPLE) ? SD_SAMPLE : 0),
                         d.cfg_twin, d.cfg_scale, d.slot, 0};
    }
    const size_t per = (size_t)n * ncb;
    if (c->canon_all_cap < per * n_steps) {
        if (c->d_canon_all) cudaFree(c->d_canon_all);
        if (c->h_canon_all) cudaFreeHost(c->h_canon_all);
        CK(cudaMalloc(&c->d_canon_all, per * n_steps * 8));
        CK(cudaMallocHost(&c->h_canon_all, per * n_steps * 8));
        c->canon_all_cap = per * n_steps;
    }
    for (int s = 0; s < n_steps; ++s) draw_canon(c, descs + (size_t)s * n, n, c->h_canon_all + per * s);
    std::memcpy(c->h_stage + c->st_pt, c->h_pt.data(), c->h_pt.size() * 4);
    CK(cudaMemcpyAsync(c->d_stage, c->h_stage, c->st_bytes, cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(c->d_sched_descs, sd.data(), nd * sizeof(SlotDesc), cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(c->d_sched_src, row_src, nd * 4, cudaMemcpyHostToDevice, c->stream));
    if (n_rows > 0) CK(cudaMemcpyAsync(c->d_sched_rows, rows, (size_t)n_rows * NCOL * 4, cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(c->d_canon_all, c->h_canon_all, per * n_steps * 8, cudaMemcpyHostToDevice, c->stream));
    CK(cudaStreamSynchronize(c->stream));          // host staging stays valid across the loop
    c->cur_n_desc = n;
    SlotDesc* d_descs = (SlotDesc*)(c->d_stage + c->st_descs);
    int* d_ids = (int*)(c->d_stage + c->st_ids);
    double* d_canon = (double*)(c->d_stage + c->st_canon);
    long total_launches = 0;
    for (int s = 0; s < n_steps; ++s) {
        {
            ProfScope ps(c, PC_FEED);
            launch_sched_feed(c->d_sched_descs + (size_t)s * n, c->d_sched_src + (size_t)s * n, n, d_descs, d_ids,
                              c->B.codes, c->d_sched_rows, c->d_canon_all + per * s, d_canon, ncb, D.text_vocab,
                              c->stream);
        }
        c->cur_t_dec = T_dec[s];
        const int rc = run_step(c, T[s], n);
        if (rc) return rc;
        total_launches += c->launches + 1;
    }
    c->sched_launches = total_launches;
    return Z2B_OK;
}

// Test support: KV of positions [0, n) of `slot` from the integer hash the CPU oracle's
// hash fill uses (pages allocated from the pool as a step would).
int ctx_debug_fill_kv(Ctx* c, int slot, int n, uint32_t seed) {
    const Dims& D = c->m->dims;
    if (slot < 0 || slot >= c->n_slots || n < 1 || n > c->slot_cap) { set_error("fill_kv: bad slot or length"); return Z2B_ERR_ARG; }
    auto& pages = c->slot_pages[slot];
    const int need = (n - 1) / PAGE + 1;
    while ((int)pages.size() < need) {
        if (c->free_pages.empty()) { set_error("KV page pool exhausted"); return Z2B_ERR_OOM; }
        const int pg = c->free_pages.back();
        c->free_pages.pop_back();
        c->h_pt[(size_t)slot * c->pages_per_slot + pages.size()] = pg;
        pages.push_back(pg);
    }
    int* d_pages = nullptr;
    CK(cudaMalloc(&d_pages, (size_t)need * 4));
    cudaMemcpy(d_pages, pages.data(), (size_t)need * 4, cudaMemcpyHostToDevice);
    launch_kv_hash_fill(c->kv, d_pages, n, D.n_layer, D.n_head_kv, D.head_dim, seed, c->stream);
    const cudaError_t e = cudaStreamSynchronize(c->stream);
    cudaFree(d_pages);
    if (e != cudaSuccess) { set_error(std::string("fill_kv: ") + cudaGetErrorString(e)); return Z2B_ERR_CUDA; }
    return Z2B_OK;
}

int ctx_debug_router_capture(Ctx* c, int enable) {
    const Dims& D = c->m->dims;
    if (enable && !c->d_rcap) {
        const size_t bytes = (size_t)D.n_layer * c->T_max * ((size_t)D.n_embd + D.rd) * 4;
        CK(cudaMalloc(&c->d_rcap, bytes));
    }
    c->rcap_on = enable != 0;
    return Z2B_OK;
}

int ctx_debug_router_inputs(Ctx* c, int layer, float* res, float* state, int* T) {
    const Dims& D = c->m->dims;
    if (!c->d_rcap || layer < 0 || layer >= D.n_layer || !c->m->layers[layer].is_moe || c->last_T < 1) {
        set_error("router_inputs: no capture for that layer");
        return Z2B_ERR_ARG;
    }
    const size_t per = (size_t)D.n_embd + D.rd;
    const float* rec = c->d_rcap + (size_t)layer * c->T_max * per;
    CK(cudaStreamSynchronize(c->stream));
    if (res) CK(cudaMemcpy(res, rec, (size_t)c->last_T * D.n_embd * 4, cudaMemcpyDeviceToHost));
    if (state) CK(cudaMemcpy(state, rec + (size_t)c->T_max * D.n_embd, (size_t)c->last_T * D.rd * 4, cudaMemcpyDeviceToHost));
    if (T) *T = c->last_T;
    return Z2B_OK;
}

int ctx_sync(Ctx* c) {
    CK(cudaMemcpyAsync(c->h_misc, c->B.err, 4, cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    if (c->h_misc[0]) { set_error("device error flags 0x" + std::to_string(c->h_misc[0])); return Z2B_ERR_DEVICE; }
    return Z2B_OK;
}

}  // namespace z2b

namespace z2b {

// Times one expert GEMV class (0 = gate/up, 1 = down) over the MoE layers, each on its own
// weights and its own routing of the last step: the router ids every layer chose (the
// step's router log) are turned into that layer's expert segments and kept, then `reps`
// launches cycle over the layers back to back between CUDA events on the context's
// stream. Returns the average duration per launch and the average algorithmic bytes per
// launch (routed experts' weights + activations in + results out).
int ctx_time_expert_gemv(Ctx* c, int which, int reps, double* ms_per_launch, uint64_t* bytes_per_launch) {
    Model* m = c->m;
    const Dims& D = m->dims;
    std::vector<int> moe;
    for (int L = 0; L < (int)m->layers.size(); ++L)
        if (m->layers[L].is_moe) moe.push_back(L);
    if (moe.empty() || reps < 1 || c->last_T < 1) { set_error("time_expert_gemv: needs a MoE model and a previous step"); return Z2B_ERR_ARG; }
    const int T = c->last_T, km = c->kmax, R = T * km, E = MAX_EXPERTS;
    const int nl = (int)moe.size();
    // per layer: n_active, n_small | active[E] | seg_off[E+1] | seg_mid[E] | tile_off[E+1] | route_tok[R] | route_w[R]
    const size_t per = 2 + E + (E + 1) + E + (E + 1) + 2 * (size_t)R;
    int* save = nullptr;
    CK(cudaMalloc(&save, per * nl * 4));
    std::unique_ptr<int, decltype(&cudaFree)> own(save, cudaFree);
    std::vector<SegSet> sets(nl);
    std::vector<float> ones((size_t)R, 1.0f);
    StepBufs B = c->B;
    CK(cudaMemcpyAsync(B.selw, ones.data(), (size_t)R * 4, cudaMemcpyHostToDevice, c->stream));
    uint64_t bytes = 0;
    for (int i = 0; i < nl; ++i) {
        const LayerDev& ly = m->layers[moe[i]];
        CK(cudaMemcpyAsync(B.sel, B.sel_log + (size_t)moe[i] * B.sel_log_T * km, (size_t)R * 4, cudaMemcpyDeviceToDevice,
                           c->stream));
        launch_segments(B, T, ly.top_k, ly.n_expert, 0, c->stream);
        int* q = save + per * i;
        int *na = q, *ns = q + 1, *act = q + 2, *so = act + E, *sm = so + E + 1, *to = sm + E, *rt = to + E + 1;
        float* rw = reinterpret_cast<float*>(rt + R);
        auto d2d = [&](void* dst, const void* src, size_t n) {
            return cudaMemcpyAsync(dst, src, n, cudaMemcpyDeviceToDevice, c->stream);
        };
        CK(d2d(na, B.n_active, 4)); CK(d2d(ns, B.n_small, 4)); CK(d2d(act, B.active, E * 4));
        CK(d2d(so, B.seg_off, (E + 1) * 4)); CK(d2d(sm, B.seg_mid, E * 4)); CK(d2d(to, B.tile_off, (E + 1) * 4));
        CK(d2d(rt, B.route_tok, (size_t)R * 4)); CK(d2d(rw, B.route_w, (size_t)R * 4));
        sets[i] = SegSet{na, ns, act, so, sm, to, rt, rw};
        int n_active = 0, routes = 0;
        CK(cudaMemcpyAsync(&n_active, B.n_active, 4, cudaMemcpyDeviceToHost, c->stream));
        CK(cudaMemcpyAsync(&routes, B.seg_off + ly.n_expert, 4, cudaMemcpyDeviceToHost, c->stream));
        CK(cudaStreamSynchronize(c->stream));
        const DevMat& w = which == 0 ? ly.gate_exps : ly.down_exps;
        const uint64_t per_expert = (uint64_t)w.n_row_tiles * w.chunks * w.tile_bytes * (which == 0 ? 2 : 1);
        const uint64_t act_bytes = which == 0 ? (uint64_t)routes * D.n_embd * 2 + (uint64_t)routes * D.n_ff * 2
                                              : (uint64_t)routes * D.n_ff * 2 + (uint64_t)routes * D.n_embd * 4;
        bytes += (uint64_t)n_active * per_expert + act_bytes;
    }
    cudaEvent_t e0, e1;
    CK(cudaEventCreate(&e0));
    CK(cudaEventCreate(&e1));
    const bool prof = c->profiling;
    c->profiling = false;
    CK(cudaEventRecord(e0, c->stream));
    for (int r = 0; r < reps; ++r)
        gemv_moe(c, m->layers[moe[r % nl]], which == 0 ? GM_GATEUP : GM_DOWN, false, &sets[r % nl]);
    CK(cudaEventRecord(e1, c->stream));
    CK(cudaEventSynchronize(e1));
    c->profiling = prof;
    float ms = 0.0f;
    CK(cudaEventElapsedTime(&ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    *ms_per_launch = ms / reps;
    *bytes_per_launch = bytes / nl;
    return Z2B_OK;
}

}  // namespace z2b

namespace z2b {

// One MoE layer's expert FFN on given activations and routing (the isolated expert op):
// x -> f16, segments from the given ids, then the decode step's own expert passes
// (tile GEMV for experts with few routes, tcgen05 GEMM for the rest). out[t] = sum over
// the token's routes of selw * down(SwiGLU(gate, up)).
int ctx_set_expert_gemm_min(Ctx* c, int routes) {
    if (routes < 1) { set_error("expert GEMM threshold must be >= 1 route"); return Z2B_ERR_ARG; }
    c->expert_gemm_min = routes;
    c->expert_gemm_set = true;
    return Z2B_OK;
}

int ctx_expert_op(Ctx* c, int layer, const float* x, int T, const int32_t* sel, const float* selw, int k, float* out,
                  int reps, double* ms, uint64_t* weight_bytes, int* n_gemm) {
    Model* m = c->m;
    const Dims& D = m->dims;
    if (layer < 0 || layer >= (int)m->layers.size() || !m->layers[layer].is_moe) { set_error("expert_op: not a MoE layer"); return Z2B_ERR_ARG; }
    const LayerDev& ly = m->layers[layer];
    if (T < 1 || T > c->T_max || k < 1 || k > c->kmax || !x || !sel || !selw) { set_error("expert_op: bad T, k or pointers"); return Z2B_ERR_ARG; }
    for (int i = 0; i < T * k; ++i)
        if (sel[i] < 0 || sel[i] >= ly.n_expert) { set_error("expert_op: expert id out of range"); return Z2B_ERR_ARG; }
    StepBufs B = c->B;
    const size_t d = (size_t)D.n_embd;
    std::vector<int32_t> hs((size_t)T * c->kmax, -1);
    std::vector<float> hw((size_t)T * c->kmax, 0.0f);
    for (int t = 0; t < T; ++t)
        for (int j = 0; j < k; ++j) { hs[(size_t)t * c->kmax + j] = sel[t * k + j]; hw[(size_t)t * c->kmax + j] = selw[t * k + j]; }
    CK(cudaMemcpyAsync(B.res, x, (size_t)T * d * 4, cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(B.sel, hs.data(), hs.size() * 4, cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(B.selw, hw.data(), hw.size() * 4, cudaMemcpyHostToDevice, c->stream));
    launch_to_f16(B.res, B.cur, (size_t)T * d, c->stream);
    // some expert can reach the threshold, and (unless set explicitly) the op is large enough
    const bool bulk = T >= c->expert_gemm_min && ly.small.gemm_ok && (c->expert_gemm_set || T >= GEMM_OP_MIN_ROWS);
    launch_segments(B, T, k, ly.n_expert, bulk ? 1 : 0, c->stream, c->expert_gemm_min);
    const bool prof = c->profiling;
    c->profiling = false;
    c->enq_failed = false;
    c->cur_T = T;
    gemv_moe(c, ly, GM_GATEUP, bulk);
    gemv_moe(c, ly, GM_DOWN, bulk);
    CK(cudaStreamSynchronize(c->stream));
    CK(cudaGetLastError());
    if (c->enq_failed) { c->profiling = prof; return Z2B_ERR_CUDA; }
    if (reps > 0 && ms) {
        cudaEvent_t e0, e1;
        CK(cudaEventCreate(&e0));
        CK(cudaEventCreate(&e1));
        CK(cudaEventRecord(e0, c->stream));
        for (int r = 0; r < reps; ++r) {
            gemv_moe(c, ly, GM_GATEUP, bulk);
            gemv_moe(c, ly, GM_DOWN, bulk);
        }
        CK(cudaEventRecord(e1, c->stream));
        CK(cudaEventSynchronize(e1));
        float t_ms = 0.0f;
        CK(cudaEventElapsedTime(&t_ms, e0, e1));
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        *ms = t_ms / reps;
    }
    c->profiling = prof;
    int na = 0, ns = 0;
    CK(cudaMemcpy(&na, B.n_active, 4, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(&ns, B.n_small, 4, cudaMemcpyDeviceToHost));
    uint32_t err = 0;
    CK(cudaMemcpy(&err, B.err, 4, cudaMemcpyDeviceToHost));
    if (err) { set_error("expert_op: device error word " + std::to_string(err)); return Z2B_ERR_DEVICE; }
    const auto bytes = [](const DevMat& w) { return (uint64_t)w.n_row_tiles * w.chunks * w.tile_bytes; };
    if (weight_bytes) *weight_bytes = (uint64_t)na * (bytes(ly.gate_exps) + bytes(ly.up_exps) + bytes(ly.down_exps));
    if (n_gemm) *n_gemm = bulk ? na - ns : 0;
    if (out) {
        const int R = T * k;
        std::vector<float> orr((size_t)R * d);
        std::vector<int32_t> pos((size_t)T * c->kmax);
        CK(cudaMemcpy(orr.data(), B.out_route, orr.size() * 4, cudaMemcpyDeviceToHost));
        CK(cudaMemcpy(pos.data(), B.route_pos, pos.size() * 4, cudaMemcpyDeviceToHost));
        for (int t = 0; t < T; ++t) {
            float* o = out + (size_t)t * d;
            std::fill(o, o + d, 0.0f);
            for (int j = 0; j < k; ++j) {
                const int pr = pos[(size_t)t * c->kmax + j];
                if (pr < 0 || pr >= R) { set_error("expert_op: route without a position"); return Z2B_ERR_DEVICE; }
                const float* src = orr.data() + (size_t)pr * d;
                for (size_t i = 0; i < d; ++i) o[i] += src[i];
            }
        }
    }
    return Z2B_OK;
}

}  // namespace z2b
