// kernels.h — host-side launch interface of the sm_100a kernels.
// Plain structs of device pointers and sizes; no torch / ggml types.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace z2b {

constexpr int MAX_EXPERTS = 256;
// Routes from which an expert takes the tensor-core GEMM rather than the tile GEMV. With
// every expert on one path the crossover is 48 routes (bench.py --crossover), but the two
// passes run back to back and, once the GEMM launches, its tiles fill one wave of the SMs:
// an expert added to it costs little, while one moved to the GEMV adds a pass per 16
// routes, and every expert the GEMV keeps costs it a full weight stream. Measured on the
// skewed config-4 op (ms at T = 64 / 256): threshold 1: 0.184 / 0.280, 5: 0.140 / 0.222,
// 9: 0.127 / 0.205, 17: 0.148 / 0.215, 48: 0.266 / 0.372.
constexpr int GEMM_MIN_TOKENS = 9;   // isolated expert op
// ... and only from 64 rows: a GEMM launch costs a wave of decode-bound tiles (~70 us),
// which the GEMV's passes undercut when the op carries few routes (T = 16: 0.045 ms on the
// GEMV alone, 0.112 ms when the experts with >= 9 routes launch the GEMM).
constexpr int GEMM_OP_MIN_ROWS = 64;
constexpr int PROJ_GEMM_MIN_ROWS = 17;      // prompt rows from which a step's projections run them
                                            // on the tensor-core GEMM (the GEMV holds 16 per pass)
// Decode step: prompt-row routes from which an expert's prompt routes take the GEMM (fewer
// join its GEMV pass). Config-2 bench (refill steps carry one 96-row prompt), frames/s:
// 4411 / 4540 / 4532 / 4453 / 4375 with 1 / 9 / 17 / 24 / 33.
constexpr int GEMM_MIN_PROMPT_ROUTES = 17;
constexpr int NCOL = 10;            // input columns per row: 9 audio codebooks + text
constexpr int PAGE = 256;           // KV page length (tokens)

// A weight matrix in tile layout (tile_layout.h).
struct DevMat {
    const uint8_t* tiles = nullptr;
    uint32_t type = 0;
    int rows = 0, K = 0;
    int n_row_tiles = 0;            // per expert for expert stacks
    int chunks = 0, tile_bytes = 0, steps = 0;
    int64_t expert_stride = 0;      // bytes between experts (stacks only)
    int n_expert = 1;
    size_t gguf_bytes = 0;          // bytes of the same weights in the GGUF file
};

// ---- tile GEMV ---------------------------------------------------------------------
enum GemvMode { GM_PROJ = 0, GM_GATEUP = 1, GM_DOWN = 2 };
enum GemvEpi { EPI_STORE = 0, EPI_ADD = 1, EPI_SOFTCAP = 2 };

struct ProjSeg { const uint8_t* tiles; int n_row_tiles; int rows; int out_off; };

struct GemvParams {
    int mode, epi;
    uint32_t type;
    int K, chunks, tile_bytes, steps, n_row_tiles;
    // projection mode: up to 4 matrices of the same type / K, all tokens
    ProjSeg seg[4];
    int n_seg, total_items;
    // expert mode: stacked experts, routed tokens
    const uint8_t* w0;              // gate (GM_GATEUP) or down (GM_DOWN)
    const uint8_t* w1;              // up   (GM_GATEUP)
    int64_t expert_stride;
    const int* n_active;            // device: number of experts with routes
    const int* active;              // device: active expert ids (ascending)
    const int* seg_off;             // device: [E+1] route offsets in expert order
    const int* tile_off;            // device: [n_active+1] prefix of 8-token tiles per active expert
    const int* n_small;             // device: GEMV experts active[0, n_small); GEMM experts after them
    const int* seg_mid;             // device: [E] GEMV routes [seg_off, seg_mid), GEMM routes [seg_mid, seg_off+1)
    const int* route_tok;           // device: token of each route (expert order)
    const float* route_w;           // device: route probability (GM_DOWN)
    // activations
    const __half* X; int ldx;       // GM_PROJ / GM_GATEUP: [T][ldx]; GM_DOWN: y [routes][ldx]
    int T;                          // GM_PROJ token count
    int tok0;                       // GM_PROJ on the tensor-core GEMM: first token of the range
    float* out; int ldo;            // GM_PROJ / GM_DOWN output (f32)
    __half* yout; int ldy;          // GM_GATEUP output y (f16)
    int out_rows;                   // valid rows per expert (GM_GATEUP / GM_DOWN)
    float cap;                      // EPI_SOFTCAP
    uint32_t* err;
    // launch geometry (host-filled)
    int n_stages, stage_bytes, cps;  // ring depth per warp, bytes per stage, chunks per stage
    int x_rs;                       // GM_PROJ: bytes per token row of a warp's shared activation slice (0: none)
    int gm_nt;                      // tensor-core GEMM: routed tokens per tile (multiple of 16, <= 256);
                                    // 0 lets launch_moe_gemm choose
    int x_rows;                     // tensor-core GEMM: rows [x_row0, x_rows) of X that it reads
    int x_row0;
    __half* xperm;                  // tensor-core GEMM: scratch [x_rows][K] for X in stage order
    const int* n_routes;            // device: routes of the step (gate/up gathers one row per route)
};

// Chooses warps/stages for a weight matrix and fills the launch geometry.
void gemv_geometry(const DevMat& m, int nmat, int ntg, int* nwarps, int* n_stages, int* stage_bytes, int* smem,
                   int* cps, int* x_rs = nullptr);
void launch_gemv(const GemvParams& p, int nwarps, int grid, int smem, cudaStream_t s);
// tcgen05 grouped GEMM over the experts active[n_small, n_active) (k_gemm.cu)
bool moe_gemm_supported(const DevMat& m);
// Returns false (nothing launched) when the activation buffer's TMA view cannot be built.
bool launch_moe_gemm(const GemvParams& p, int grid, cudaStream_t s);

// ---- decode-step kernels -----------------------------------------------------------
struct Dims {
    int n_embd, head_dim, n_head, n_head_kv, n_ff, rd, n_layer;
    int n_codebooks, audio_vocab, text_vocab;
    float rms_eps, qk_eps, rope_base, softcap;
};

// One step's input descriptor per active stream (uploaded by the host each step).
struct SlotDesc {
    int slot;        // cache band / column
    int n_past;      // logical position of the first new row
    int n_new;       // rows this step
    int flags;       // SD_* bits
    int twin;        // desc index of the unconditional CFG twin, or -1
    float cfg_scale;
    int samp;        // index into the per-slot sampling table (= slot)
    int pad_;
};
enum SlotFlags { SD_OUTPUT = 1, SD_SAMPLE = 2, SD_ALL_ROWS = 4 };   // SD_ALL_ROWS: every row is an output row

// Sampling parameters per slot, device copy (mirrors zonos2_sampling).
struct SampDev {
    float temperature, top_p, min_p, rep_penalty;
    int top_k, rep_window, rep_codebooks, greedy;
};

// Paged KV cache: page p holds PAGE tokens of every layer:
//   [p][layer][kvh] K block: [PAGE][hd] f16, rows swizzled (16-byte chunk c of key j at c ^ swz(j))
//                   V block: [PAGE/64][hd][64] f16 (V transposed per 64 keys, rows swizzled by dim)
struct KVDev {
    __half* pool;
    const int* page_table;          // [n_slots][max_pages]
    int max_pages;
    size_t page_elems;              // elements per page (all layers)
    size_t layer_elems;             // elements per layer within a page
    size_t head_elems;              // elements per (K or V) block of one kv head
};

// Per-step device buffers (capacity T_max tokens, R_max routes, O_max output rows).
struct StepBufs {
    const SlotDesc* descs; int n_desc;
    const int* ids_in;              // [T][NCOL] packed host input rows
    int* tok_slot; int* tok_pos; int* tok_desc; int* ids;   // [T], [T][NCOL]
    int* out_tok;                   // [n_out] token of each output row
    int* out_desc;                  // [n_out] desc of each output row
    int* tok_out;                   // [T] output row of a token, or -1
    int* desc_out;                  // [n_desc] output row of a desc, or -1
    float* res; __half* cur;        // [T][d]
    float* qkvg; int ldq;           // [T][ldq]
    __half* qh;                     // [T][nh][hd]
    float* apart; int max_split;    // [T][nh][max_split][hd+2]
    int* attn_ticket;               // [T][nkv] split arrivals (zero between steps)
    int2* attn_items;               // [T * max_split] attention work list: (token, split), token order
    int* attn_n_items;              // [1] entries of the work list
    int split_keys;                 // keys per attention split
    __half* o;                      // [T][nh*hd]
    float* rstate;                  // [T][rd]
    float* rpart; int rpart_T;      // [4][rpart_T][rd] router down-projection partial sums
    int* sel; float* selw; int kmax;// [T][kmax]
    int* n_active; int* active; int* seg_off; int* route_tok; float* route_w; int* route_pos;
    int* tile_off;                  // [MAX_EXPERTS + 1] prefix of 8-token tiles over active experts
    int* n_small;                   // active[0, n_small): experts with GEMV routes; then GEMM experts
    __half* gemm_x;                 // tensor-core GEMM: activations in stage order (k permuted per chunk)
    int* seg_mid;                   // [MAX_EXPERTS] first GEMM route of each expert
    int* ticket;
    __half* y;                      // [R][ff]
    float* out_route;               // [R][d]
    __half* hout;                   // [O][d]
    float* logits;                  // [O][ncb*av]
    int* codes;                     // [O][ncb]
    const double* canon;            // [O][ncb] host-drawn uniform(0,1) values
    int* layer_active;              // [n_layer] experts with routes, per layer (accounting)
    int* sel_log; int sel_log_T;    // optional [n_layer][sel_log_T][kmax] record of router ids
    uint32_t* err;
};

// Per-layer small tensors kept as f32 on the device.
struct LayerSmall {
    const float *attn_norm, *ffn_norm, *attn_temp;
    const float *rdown_w, *rdown_b, *m0_w, *m0_b, *m2_w, *m2_b, *m4_w, *rnorm, *rbias, *eda, *rmask;
    const int8_t* rdown_q;          // router down projection kept as Q8_0 quants [rd][d] (or null)
    const float* rdown_qd;          // its block scales [rd][d/32] (f32 copies of the f16 d)
    int is_moe, top_k, n_expert;
    int gemm_ok;                    // gate/up and down both run on the tcgen05 GEMM (prompt routes)
};

// Embedding tables in GGUF block format (rows dequantised in the kernel).
struct EmbedDev {
    const uint8_t* audio[16]; const uint8_t* text; uint32_t type; size_t row_bytes;
};

void launch_pack(const StepBufs& b, int T, int n_out, cudaStream_t s);
// spk_t >= 0: token spk_t's embedding sum is replaced by spk_row (speaker injection).
void launch_embed(const StepBufs& b, const EmbedDev& e, const float* attn_norm0, const Dims& d, int T, int spk_t,
                  const float* spk_row, cudaStream_t s);
// row = W_proj (W_lda spk + b_lda) + b_proj (+ delta), f32 (src/zonos2-graph.cpp:262-275).
void launch_spk_proj(const float* lda_w, const float* lda_b, const float* proj_w, const float* proj_b, const float* spk,
                     const float* delta, int spk_dim, int lda_dim, int n_embd, float* row, cudaStream_t s);
void launch_rope_append(const StepBufs& b, const KVDev& kv, const float* temp, const Dims& d, int layer, int T, cudaStream_t s);
// Test fill: positions [0, n) of one slot (pages[] = the slot's page ids) in every layer
// from an integer hash of (seed, layer, K/V, position, kv head, dim); exact in f16.
void launch_kv_hash_fill(const KVDev& kv, const int* pages, int n, int n_layer, int nkv, int hd, uint32_t seed,
                         cudaStream_t s);
void launch_attention(const StepBufs& b, const KVDev& kv, const Dims& d, int layer, int T, int split_keys, int max_split, cudaStream_t s);
void launch_attn_combine(const StepBufs& b, const Dims& d, int T, int split_keys, int max_split, cudaStream_t s);
void launch_router(const StepBufs& b, const LayerSmall& ly, const Dims& d, int T, int first_moe, int layer,
                   cudaStream_t s);
int router_launches(const LayerSmall& ly);
// Expert segments from given router ids b.sel/b.selw (one block; the router's own last step).
// bulk_mode 1: experts with >= gemm_min routes take the tensor-core GEMM.
void launch_segments(const StepBufs& b, int T, int k, int E, int bulk_mode, cudaStream_t s,
                     int gemm_min = GEMM_MIN_TOKENS);
// f32 rows -> f16 rows (n values).
void launch_to_f16(const float* x, __half* y, size_t n, cudaStream_t s);
// Device-resident decode loop: feed each stream its sampled frame (+ text pad) as the
// next input row, advance n_past, and copy this step's host-drawn uniforms.
void launch_sched_feed(const SlotDesc* step_descs, const int* src, int n, SlotDesc* descs, int* ids_in,
                       const int* codes, const int* rows, const double* canon_src, double* canon_dst, int ncb,
                       int text_pad, cudaStream_t s);
void launch_feed(SlotDesc* descs, int n, int* ids_in, const int* codes, const int* desc_out, double* canon_dst,
                 const double* canon_src, int ncb, int text_pad, int advance, cudaStream_t s);
void launch_moe_combine(const StepBufs& b, const LayerSmall& ly, const float* next_norm, const float* out_norm,
                        const Dims& d, int T, int last, cudaStream_t s);
void launch_sampler(const StepBufs& b, const SampDev* samp, int* hist, int* hist_len, int hist_cap,
                    const Dims& d, int n_out, cudaStream_t s);

}  // namespace z2b
