/* z2b_tools.h — host-side tools around the decode-step boundary.
 *
 * Two shared libraries export these:
 *   libz2b_synth.so  z2b_synth_write: synthetic ZONOS2-family GGUF files (no GPU needed).
 *                    Replaces, for benchmarks, the reference's checkpoint converters and
 *                    dummy generator (models/convert-zonos2-to-gguf.py,
 *                    scripts/make-dummy-model.py): same keys, tensor names and shapes.
 *   libz2b.so        z2b_host_repack / z2b_host_unpack_tiles: the load-time weight repack
 *                    that z2b_model_load applies before upload, callable on host memory so
 *                    the tile layout can be checked without a GPU.
 * All functions return 0 on success.
 */
#ifndef Z2B_TOOLS_H
#define Z2B_TOOLS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define Z2B_MAX_LAYERS 128

/* ggml type ids accepted for matrices: 0 F32, 1 F16, 8 Q8_0, 12 Q4_K, 14 Q6_K. */
typedef struct z2b_synth_config {
    uint32_t n_layer, n_embd, head_dim, n_head, n_head_kv, n_ff, n_expert, router_dim, n_ctx;
    int32_t  expert_used[Z2B_MAX_LAYERS]; /* per layer: 0 = dense FFN, else MoE top-k */
    float    rope_base, rms_eps, qk_eps, softcap;
    uint32_t n_codebooks, codebook_size, text_vocab, spk_dim, lda_dim;
    /* storage types by tensor class */
    uint32_t t_attn, t_gateup, t_down, t_dense, t_head, t_embd, t_router, t_spk;
    /* 0: every tensor N(0, std) (the reference dummy model's recipe);
     * 1: matrices N(0, std), norm weights 1+N(0,std), |attn_temp| near 1 and router MLP
     *    gains 1/sqrt(router_dim) so routing varies per token instead of collapsing onto
     *    the balancing bias. */
    uint32_t init_mode;
    float    std;
    uint64_t seed;
} z2b_synth_config;

/* Writes a GGUF file; on failure returns nonzero and writes a message into err. */
int z2b_synth_write(const z2b_synth_config* cfg, const char* path, char* err, int errlen);

/* Repack `rows` rows of a GGUF tensor (type, ne0 = k) into the device tile layout.
 * dst must hold z2b_host_tiles_bytes(type, rows, k) bytes. */
int64_t z2b_host_tiles_bytes(uint32_t type, int64_t rows, int64_t k);
int z2b_host_repack(uint32_t type, int64_t rows, int64_t k, const void* src, void* dst);
/* Decode a tile-layout buffer back to f32 rows [rows][k] on the host (layout check). */
int z2b_host_unpack_tiles(uint32_t type, int64_t rows, int64_t k, const void* tiles, float* out);

/* Host-only: the tile GEMV's launch geometry for a weight type, K, matrices per item
 * (1, or 2 for gate/up) and token tiles per pass (ntg 2 for projections and gate/up, 1
 * for the down pass). out[0..6] = warps, ring stages, stage bytes, dynamic shared bytes,
 * chunks per stage, bytes per token row of a warp's shared activation slice (0 when the
 * activations are read into registers directly), chunks per warp. Returns 7 for an
 * unsupported type / K. */
int z2b_test_gemv_geometry(uint32_t type, int64_t k, int nmat, int ntg, int32_t* out);

/* Device checks (libz2b.so, need a GPU). z2b_test_dequant decodes `rows` GGUF rows of
 * type/k on the device to f32 [rows][k], either from the tile image the GEMV reads
 * (from_tiles = 1) or straight from GGUF rows as the embedding gather does (0), with
 * gguf-py's rounding order. z2b_test_gemv computes out[n][r] = sum_k W[r][k] x[n][k]
 * for n_tok f16 activation rows with the projection-mode tile GEMV.
 * Return 0, 4 (CUDA error), 6 (device error flag) or 7 (unsupported). */
int z2b_test_dequant(uint32_t type, int64_t rows, int64_t k, const void* gguf_rows, int from_tiles, float* out);
/* Runs the kernels' bounded mbarrier wait (at most `polls` <= 4096 polls) on a phase that
 * never completes: *outcome = 2 when the wait gave up (1 if it completed), *err_word =
 * the device error word it left (DERR_WAIT_TIMEOUT = 1), *elapsed_ns = how long the
 * wait took. No fault, no trap. */
int z2b_test_wait_timeout(uint32_t polls, uint32_t* err_word, uint32_t* outcome, uint64_t* elapsed_ns);
int z2b_test_gemv(uint32_t type, int64_t rows, int64_t k, const void* gguf_rows, const uint16_t* x_f16,
                  int n_tok, float* out);

/* Device packer on host descriptors {slot, n_past, n_new, flags(bit0 = output)}[n] with
 * T = sum(n_new): per-token slot, position, output row (-1 if none) and the token of each
 * output row. */
int z2b_test_pack(const int32_t* desc4, int n, int T, int32_t* tok_slot, int32_t* tok_pos, int32_t* tok_out,
                  int32_t* out_tok);
/* Device segment builder on given router ids sel[T][k] and weights: expert offsets
 * seg_off[E+1], token of each route in expert order, and the position of route (t, j). */
int z2b_test_route(const int32_t* sel, const float* selw, int T, int k, int E, int32_t* seg_off,
                   int32_t* route_tok, int32_t* route_pos);

/* Largest T * k that z2b_route_segments_noalloc accepts (its fixed device scratch is
 * 5 words per route plus 2 * 256 + 2 words, about 320 KB). */
#define Z2B_NOALLOC_MAX_ROUTES 16384
/* No reference counterpart. The segment builder of z2b_test_route (same arguments, same
 * results) without any device allocation: it works in a fixed scratch array compiled
 * into the library (every GPU that loads the library holds it until exit). It is for
 * callers that may not call cudaMalloc/cudaFree: a server that gave all but a fixed
 * budget of the GPU to its KV page pool, or a latency-critical thread, since allocation
 * can synchronise the whole device and stall decode steps queued by other threads.
 * Runs on the current device and the calling thread's per-thread default stream, and
 * returns when the results are in the host arrays. The first call on each device also
 * looks up the scratch address (a one-time set-up on that device). Calls
 * that overlap on the GPU share the scratch and race: serialise them. T * k >
 * Z2B_NOALLOC_MAX_ROUTES returns Z2B_ERR_ARG with z2b_last_error() naming the limit. */
int z2b_route_segments_noalloc(const int32_t* sel, const float* selw, int T, int k, int E, int32_t* seg_off,
                               int32_t* route_tok, int32_t* route_pos);

/* No reference counterpart. Tuning of z2b_expert_op (z2b.h): an expert with at least
 * `routes` routes takes the tcgen05 grouped GEMM, one with fewer the tile GEMV (default 9,
 * applied from T = 64 rows; once set, at any T: 1 sends every expert to the GEMM, a value
 * above the op's route count none). Used to
 * measure the GEMV / GEMM crossover; the decode step keeps its own rule. Z2B_ERR_ARG for
 * routes < 1. */
struct z2b_ctx;
int z2b_set_expert_gemm_min(struct z2b_ctx* ctx, int routes);

/* Router ids of every layer for the last z2b_step: writes [n_layer][T][kmax] when cap is
 * large enough; returns the number of entries (or -1). */
int z2b_debug_last_sel(struct z2b_ctx* ctx, int32_t* out, int cap);

/* Test support, no reference counterpart (need a GPU).
 * z2b_debug_fill_kv: positions [0, n) of `slot` get KV pages from the context's pool
 * holding, in every layer, k / 1024 (k in [-2048, 2048), exact in f16) from a splitmix64
 * hash of (seed, layer, K or V, position, kv head, dim): the values the CPU oracle's
 * hash fill writes, so decode over long contexts can be checked without a prefill.
 * Decode steps then continue from n_past = n.
 * z2b_debug_router_capture: with enable = 1 the following steps run without graphs and
 * record, before every MoE layer's router, the residual rows [T][n_embd] and the
 * incoming router state [T][router_dim]; z2b_debug_router_inputs copies layer `layer`'s
 * record of the last step into res / state (either may be NULL) and its T into *T. */
int z2b_debug_fill_kv(struct z2b_ctx* ctx, int slot, int n, uint32_t seed);
int z2b_debug_router_capture(struct z2b_ctx* ctx, int enable);
int z2b_debug_router_inputs(struct z2b_ctx* ctx, int layer, float* res, float* state, int* T);

#ifdef __cplusplus
}
#endif
#endif
