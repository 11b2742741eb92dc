// runtime.h — batch context (host side of the decode step).
#pragma once

#include "kernels.h"
#include "model.h"
#include "../../include/z2b.h"

#include <cstdint>
#include <map>
#include <memory>
#include <random>
#include <string>
#include <vector>

namespace z2b {

struct Ctx {
    Model* m = nullptr;
    cudaStream_t stream = nullptr;
    int n_slots = 0, slot_cap = 0, pages_per_slot = 0;
    int T_max = 0, O_max = 0, D_max = 0, R_max = 0, kmax = 1;
    int split_keys = 256, max_split = 1;
    // KV page pool and the host page allocator
    int n_pages = 0;
    size_t head_elems = 0, layer_elems = 0, page_elems = 0;
    __half* kv_pool = nullptr;
    std::vector<int> free_pages;
    std::vector<std::vector<int>> slot_pages;
    std::vector<int> h_pt;                   // [n_slots][pages_per_slot]
    KVDev kv{};
    // per-step staging: page table | descs | ids | canon (pinned host + device mirror)
    size_t st_pt = 0, st_descs = 0, st_ids = 0, st_canon = 0, st_bytes = 0;
    uint8_t* h_stage = nullptr;
    uint8_t* d_stage = nullptr;
    StepBufs B{};
    // sampler state
    SampDev* d_samp = nullptr;
    std::vector<SampDev> h_samp;
    std::vector<int> greedy;
    std::vector<std::mt19937> rng;
    int* d_hist = nullptr;
    int* d_hist_len = nullptr;
    int hist_cap = 0;
    // outputs
    int32_t* h_codes = nullptr;
    float* h_logits = nullptr;
    uint32_t* h_misc = nullptr;              // [0] error word, [1..] active experts per layer
    std::vector<float> step_logits;
    std::vector<char> step_has_logits;
    std::vector<int> desc_out_host;
    int cur_n_desc = 0;
    int cur_t_dec = 0;                       // single-row (decode) descriptors of the current step:
                                             // tokens [0, cur_t_dec), prompt rows after them
    int last_T = 0;                          // tokens of the last z2b_step
    size_t last_h2d = 0, last_d2h = 0;       // bytes copied by the last z2b_step
    bool keep_logits = true;                 // read logits back even without out_logits
    // speaker injection: token of the current step whose embedding is replaced (-1: none),
    // and a device buffer [spk_dim (input) | n_embd (delta) | n_embd (row)]
    int spk_t = -1;
    // every row of a Z2B_WANT_LOGITS desc is an output row (teacher-forced logits)
    bool all_rows = false;
    float* d_spk = nullptr;
    // graphs keyed by (n_desc, T, n_out)
    bool graphs_enabled = true;
    std::map<uint64_t, cudaGraphExec_t> graphs;
    std::map<uint64_t, int> graph_launches;
    std::map<uint64_t, int> shape_seen;      // occurrences of step shapes carrying prompt rows
    int prompt_graphs = 0;
    bool enq_failed = false;
    int cur_T = 0;                           // rows of the step (or expert op) being enqueued
    int expert_gemm_min = GEMM_MIN_TOKENS;   // expert op: routes from which an expert takes the GEMM
    bool expert_gemm_set = false;            // set explicitly: the op's minimum rows no longer apply                 // a launch could not be set up while enqueuing (error set)
    int launches = 0, loop_launches = 0;
    // decode-loop uniforms
    double* d_canon_all = nullptr;
    double* h_canon_all = nullptr;
    size_t canon_all_cap = 0;
    // per-launch profiling (eager steps only): class of each launch and its event pair
    bool profiling = false;
    std::vector<int> prof_class;
    std::vector<cudaEvent_t> prof_ev;
    size_t prof_used = 0;
    std::vector<double> prof_ms;             // accumulated per class
    std::vector<long> prof_count;
    // scheduled device loop
    int* d_sched_rows = nullptr;             // prompt rows uploaded for a schedule
    size_t sched_rows_cap = 0;
    SlotDesc* d_sched_descs = nullptr;
    size_t sched_descs_cap = 0;
    int* d_sched_src = nullptr;              // [steps][n] row offset or -1 (feed from codes)
    size_t sched_src_cap = 0;
    long sched_launches = 0;                 // kernel launches of the last schedule
    // test support: router inputs recorded before every MoE router of a step
    bool rcap_on = false;
    float* d_rcap = nullptr;                 // [n_layer][T_max][n_embd + rd]
    // accounting of the last step
    uint64_t last_wbytes = 0, last_kvbytes = 0, last_other = 0;
    std::vector<void*> dallocs, hallocs;
    ~Ctx();
};

void set_error(const std::string& e);
const char* last_error();
// out_rows: output (logits) rows per step, at least n_slots.
int ctx_create(Model* m, int n_slots, int slot_cap_frames, Ctx** out, int out_rows = 0);
// Teacher-forced logits of every row of one sequence (zonos2_logits): out [n][ncb][av].
int model_logits(Model* m, const int32_t* ids, int n, const float* spk, int spk_pos, const float* delta, float* out);
int ctx_slot_reset(Ctx* c, int slot, const z2b_sampling* sp);
int ctx_set_sampling(Ctx* c, int slot, const z2b_sampling* sp);
int ctx_step(Ctx* c, const z2b_slot_desc* descs, int n, const int32_t* ids, int32_t* out_codes, float* out_logits);
int ctx_prefill(Ctx* c, int slot, const int32_t* ids, int n0, float* out_logits);
// Prefill with an optional speaker embedding replacing the embedding of prompt row spk_pos
// (and an optional emotion delta added to the projected speaker row).
int ctx_prefill_spk(Ctx* c, int slot, const int32_t* ids, int n0, const float* spk, int spk_pos, const float* delta,
                    float* out_logits);
int ctx_decode_loop(Ctx* c, const z2b_slot_desc* descs, int n, const int32_t* first_ids, int n_steps);
int ctx_sync(Ctx* c);
void enqueue_step(Ctx* c, int T, int n_out);
int ctx_run_schedule(Ctx* c, int n_steps, int n, const z2b_slot_desc* descs, const int32_t* rows, int n_rows,
                     const int32_t* row_src);
enum ProfClass { PC_PACK, PC_EMBED, PC_QKV, PC_ROPE, PC_ATTN, PC_ATTN_COMB, PC_WO, PC_ROUTER, PC_GATEUP, PC_DOWN,
                 PC_COMBINE, PC_HEAD, PC_SAMPLER, PC_FEED, PC_N };
void account(Ctx* c, const z2b_slot_desc* descs, int n, int T);
int ctx_time_expert_gemv(Ctx* c, int which, int reps, double* ms_per_launch, uint64_t* bytes_per_launch);
int ctx_debug_fill_kv(Ctx* c, int slot, int n, uint32_t seed);
int ctx_debug_router_capture(Ctx* c, int enable);
int ctx_debug_router_inputs(Ctx* c, int layer, float* res, float* state, int* T);
int ctx_set_expert_gemm_min(Ctx* c, int routes);
int ctx_expert_op(Ctx* c, int layer, const float* x, int T, const int32_t* sel, const float* selw, int k, float* out,
                  int reps, double* ms, uint64_t* weight_bytes, int* n_gemm);

}  // namespace z2b
