/* z2b.h — C ABI of the B200 batched backbone decode step (libz2b.so).
 *
 * Drop-in for the batched backbone path of zonos2.cpp: the model loader, the
 * continuous-batching context, per-slot prefill, the batched decode step, per-slot
 * logits and the multi-codebook sampler. Plain pointers and sizes only; every call
 * returns Z2B_OK (0) or an error code, and z2b_last_error() describes the last failure
 * of the calling thread. A context is owned by one thread (as the reference's worker
 * thread owns its zonos2_batch_ctx, src/server.cpp:13-14, 904-911); one context per GPU.
 */
#ifndef Z2B_H
#define Z2B_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define Z2B_OK 0
#define Z2B_ERR_ARG 1          /* invalid argument or state */
#define Z2B_ERR_IO 2           /* file cannot be read */
#define Z2B_ERR_FORMAT 3       /* not a usable zonos2 GGUF */
#define Z2B_ERR_CUDA 4         /* a CUDA runtime call failed */
#define Z2B_ERR_OOM 5          /* device or KV-page memory exhausted */
#define Z2B_ERR_DEVICE 6       /* a kernel reported an error (bad id, missing page, wait timeout) */
#define Z2B_ERR_UNSUPPORTED 7  /* tensor type or shape this build does not handle */

typedef struct z2b_model z2b_model;
typedef struct z2b_ctx z2b_ctx;

/* Hyper-parameters read from the GGUF keys zonos2.* (src/zonos2.h:14-50). */
typedef struct z2b_hparams {
    uint32_t n_layer, n_embd, head_dim, n_head, n_head_kv, n_ff, n_expert, n_ctx_train;
    float rope_freq_base, rms_eps, qk_norm_eps, logit_softcap;
    uint32_t n_codebooks, codebook_size, audio_vocab, eoa_id, audio_pad_id, text_vocab;
    uint32_t spk_dim, spk_lda_dim, router_dim;
    int32_t expert_used[128];          /* per layer: 0 dense FFN, else MoE top-k */
    uint64_t weight_bytes;             /* GGUF bytes of all tensors on the device */
} z2b_hparams;

/* Sampling parameters of one stream (zonos2_sampling, src/zonos2.h:197-208). */
typedef struct z2b_sampling {
    float temperature;                 /* 1.15 */
    int32_t top_k;                     /* 106 */
    float top_p;                       /* 0 disables */
    float min_p;                       /* 0.18 */
    float rep_penalty;                 /* 1.2 */
    int32_t rep_window;                /* 50, at most Z2B_MAX_REP_WINDOW */
    int32_t rep_codebooks;             /* 8 */
    uint32_t seed;                     /* std::mt19937 seed */
    int32_t greedy;                    /* argmax, first max wins */
} z2b_sampling;
#define Z2B_MAX_REP_WINDOW 256

/* One stream's work in a step. */
typedef struct z2b_slot_desc {
    int32_t slot;                      /* cache band / column (zonos2_slot::index) */
    int32_t n_past;                    /* logical position of the first new row (zonos2_slot::n_past) */
    int32_t n_new;                     /* rows fed this step: 1 = decode, >1 = prompt chunk */
    int32_t flags;                     /* Z2B_WANT_* */
    int32_t cfg_twin;                  /* index (in this step's desc array) of the unconditional
                                          twin for emotion CFG (src/server.cpp:1125-1142), or -1 */
    float cfg_scale;                   /* guided = u + scale * (c - u) */
} z2b_slot_desc;
#define Z2B_WANT_LOGITS 1              /* compute logits of the stream's last row */
#define Z2B_WANT_SAMPLE 3              /* logits + sample one frame with the slot's sampler */

/* Load a zonos2 GGUF onto CUDA device `device`, repacking quantised weights into the
 * kernels' tile layout. Replaces zonos2_model_load (src/zonos2.h:124, src/zonos2.cpp:15-186). */
int z2b_model_load(const char* path, int device, z2b_model** out);
/* Replaces zonos2_model_free (src/zonos2.h:125). */
int z2b_model_free(z2b_model* model);
int z2b_model_hparams(const z2b_model* model, z2b_hparams* out);
/* Runtime expert mask: for each listed layer only the listed experts stay routable.
 * keep_offsets has n_layers+1 entries into keep_ids; n_layers = 0 clears the mask.
 * Replaces zonos2_set_expert_mask (src/zonos2.h:136, src/zonos2.cpp:203-239). */
int z2b_set_expert_mask(z2b_model* model, const int32_t* layers, int n_layers,
                        const int32_t* keep_offsets, const int32_t* keep_ids);

/* Create a batch context of n_slots streams of up to slot_cap_frames rows each (rounded
 * up to whole 256-row KV pages, allocated on demand from a shared pool).
 * Replaces zonos2_batch_init (src/zonos2.h:279, src/zonos2-graph.cpp:639-690). */
int z2b_ctx_create(z2b_model* model, int n_slots, int slot_cap_frames, z2b_ctx** out);
/* Replaces zonos2_batch_free (src/zonos2.h:280). */
int z2b_ctx_destroy(z2b_ctx* ctx);

/* Admit a stream into `slot`: frees its KV pages and resets its sampler (history, RNG
 * seeded with sp->seed). sp may be NULL for greedy. */
int z2b_slot_reset(z2b_ctx* ctx, int slot, const z2b_sampling* sp);
/* Set a stream's sampler (parameters, mt19937 seeded with sp->seed, empty repetition
 * history) without touching its KV pages, e.g. after its prefill. The counterpart of
 * constructing zonos2_sampler (src/zonos2-sampler.cpp:6-7, src/zonos2-graph.cpp:528, 889). */
int z2b_set_slot_sampling(z2b_ctx* ctx, int slot, const z2b_sampling* sp);

/* Prefill prompt rows ids[n0][10] (int32, row-major) into `slot` from position 0 and
 * return the last row's logits [n_codebooks * audio_vocab] in out_logits.
 * Replaces zonos2_batch_slot_prefill (src/zonos2.h:286-288, src/zonos2-graph.cpp:703-760). */
int z2b_slot_prefill(z2b_ctx* ctx, int slot, const int32_t* ids, int n0, float* out_logits);

/* z2b_slot_prefill with the reference's speaker arguments, in its order. spk
 * (float[spk_dim], or NULL for none) is projected as spk_proj(spk_lda(spk)), plus
 * spk_emotion_delta (float[n_embd]) when not NULL, and replaces the embedding of prompt
 * row spk_pos (0 <= spk_pos < n0) before emb_norm; a negative spk_pos means no speaker,
 * as in the reference. Replaces zonos2_batch_slot_prefill's spk / spk_pos /
 * spk_emotion_delta (src/zonos2.h:286-288, 312-313; src/zonos2-graph.cpp:36-37, 262-292,
 * 703-760). Z2B_ERR_ARG if spk_pos >= n0. */
int z2b_slot_prefill_spk(z2b_ctx* ctx, int slot, const int32_t* ids, int n0, const float* spk, int spk_pos,
                         float* out_logits, const float* spk_emotion_delta);

/* Teacher-forced logits of one sequence: ids[n_tokens][10] run from position 0 through
 * the decode kernels on a private single-slot context, and out_logits[n_tokens][n_codebooks]
 * [audio_vocab] receives every row's logits (row t after rows 0..t). spk / spk_pos /
 * spk_emotion_delta as z2b_slot_prefill_spk (spk NULL: none). Replaces zonos2_logits
 * (src/zonos2.h:156-158, src/zonos2-graph.cpp:457-473), the quality evals' entry point. */
int z2b_logits(z2b_model* model, const int32_t* ids, int n_tokens, float* out_logits, const float* spk, int spk_pos,
               const float* spk_emotion_delta);

/* Options of a TTS prompt (zonos2_prompt_options, src/zonos2.h:181-188); defaults from
 * z2b_prompt_options_default reproduce the reference's offline prompt. */
typedef struct z2b_prompt_options {
    int32_t prepend_silence;           /* 1: append the 17 sheared 0.2 s silence frames */
    int32_t speaking_rate_bucket;      /* -1: no speaking-rate row */
    int32_t n_quality;                 /* entries used in quality_buckets; 0: the default
                                          (trailing_silence_s feature at bucket 3) */
    int32_t quality_buckets[16];       /* bucket per quality feature, -1 skips the feature */
    int32_t add_speaker_slot;          /* 1: prepend the speaker slot (+ marker rows) for cloning */
    int32_t clean_speaker_background;
    int32_t accurate_mode;
} z2b_prompt_options;
void z2b_prompt_options_default(z2b_prompt_options* opt);

/* Build the input rows [n_rows][n_codebooks + 1] of a TTS prompt for the UTF-8 text
 * (text_len bytes) with the model's hyper-parameters (z2b_model_hparams): optional speaker
 * slot and marker rows, speaking-rate and quality rows, BOS, one row per byte (id byte + 192),
 * EOS, then the sheared silence frames. Replaces zonos2_build_prompt (src/zonos2.h:190-195,
 * src/zonos2-prompt.cpp:54-133), row for row. *n_rows receives the row count and *spk_pos
 * the speaker slot's row (-1 without one). A call with out_ids NULL and cap_rows 0 only
 * sizes the prompt (Z2B_OK); otherwise cap_rows < *n_rows writes nothing and returns
 * Z2B_ERR_ARG. Bucket values are not range-checked, as in the reference. Host-only: no
 * device is needed. */
int z2b_build_prompt(const z2b_hparams* hp, const char* text, int64_t text_len, const z2b_prompt_options* opt,
                     int32_t* out_ids, int cap_rows, int* n_rows, int* spk_pos);

/* One batched step over n streams: rows ids[sum(n_new)][10] are fed in desc order
 * (decode streams feed one row; prompt chunks may be mixed in). For each desc with
 * Z2B_WANT_SAMPLE, out_codes[i*n_codebooks ..] receives the sampled frame; with
 * out_logits != NULL, out_logits[i*n_codebooks*audio_vocab ..] receives the logits of
 * every desc with Z2B_WANT_LOGITS. Replaces zonos2_batch_step + zonos2_slot_sample's
 * sampling (src/zonos2.h:294, 304-306; src/zonos2-graph.cpp:762-870). The caller keeps
 * the per-stream state (n_past, EOS countdown) as in zonos2_slot. */
int z2b_step(z2b_ctx* ctx, const z2b_slot_desc* descs, int n, const int32_t* ids,
             int32_t* out_codes, float* out_logits);

/* Logits of desc `index` of the last step (host copy, valid until the next step; NULL
 * when logits readback is off and the step was given no out_logits).
 * Replaces zonos2_batch_slot_logits (src/zonos2.h:298). */
const float* z2b_step_logits(const z2b_ctx* ctx, int index);
/* Logits readback to the host after every step (default on, as the reference reads all
 * logits each step). Off: only the sampled frames cross PCIe unless a step passes
 * out_logits. */
int z2b_set_logits_readback(z2b_ctx* ctx, int enable);
/* Bytes the last z2b_step copied host->device (inputs) and device->host (outputs). */
int z2b_last_step_io(const z2b_ctx* ctx, uint64_t* h2d_bytes, uint64_t* d2h_bytes);

/* Device-resident decode loop for throughput runs: n_steps decode steps over the same
 * streams, each step feeding every stream its previous sampled frame (+ text pad) and
 * advancing n_past on the device; descs[i].n_new must be 1. Returns when all steps are
 * enqueued (asynchronous on the context's stream). */
int z2b_decode_loop(z2b_ctx* ctx, const z2b_slot_desc* descs, int n, const int32_t* first_ids, int n_steps);
/* Scheduled device-resident run of n_steps steps over n streams (desc i stays on one
 * slot). descs[s*n + i] is stream i's work at step s; every desc must want logits. Rows
 * of stream i at step s come from rows[row_src[s*n+i] ..] when row_src >= 0 (prompts,
 * first rows), or, with n_new == 1 and row_src < 0, from the frame the device sampled
 * for stream i at step s-1 (+ text pad; at s = 0, the previous step run on this context
 * with the same streams), so no host round trip sits between steps.
 * Asynchronous on the context's stream. The continuous-batching benchmark uses it to
 * replay arrivals (prompt prefills packed into decode steps) and decodes. */
int z2b_run_schedule(z2b_ctx* ctx, int n_steps, int n, const z2b_slot_desc* descs, const int32_t* rows,
                     int n_rows, const int32_t* row_src);
/* Frames sampled for the first n output rows by the last step run on the context (also
 * after z2b_run_schedule / z2b_decode_loop): out[n][n_codebooks]. Synchronises. */
int z2b_last_codes(z2b_ctx* ctx, int32_t* out, int n);
/* Kernel launches issued by the last z2b_run_schedule. */
long z2b_last_run_launches(const z2b_ctx* ctx);
/* Per-kernel-class device time: enable = 1 starts recording CUDA events around every
 * launch (steps then run without graphs); enable = 0 stops, synchronises and returns
 * milliseconds and launch counts per class (pack, embed, qkv, rope, attention,
 * attention combine, wo, router, expert gate/up, expert down, combine, head, sampler,
 * feed). */
int z2b_profile(z2b_ctx* ctx, int enable, double* ms_per_class, long* count_per_class, int n_classes);

/* Wait for all work on the context's stream and report device errors. */
int z2b_sync(z2b_ctx* ctx);
/* The context's cudaStream_t (for event timing by the caller). */
void* z2b_ctx_stream(z2b_ctx* ctx);

/* Per-step accounting: algorithmic HBM bytes the last step read/wrote (weights touched
 * according to the actual routed experts, KV read and written, embedding rows). */
int z2b_last_step_bytes(const z2b_ctx* ctx, uint64_t* weight_bytes, uint64_t* kv_bytes, uint64_t* other_bytes);
/* Kernel launches issued by the last z2b_step / per decode-loop step. */
int z2b_last_step_launches(const z2b_ctx* ctx);
/* Experts that received routes in each layer during the last z2b_step (n_layer values;
 * returns n_layer). */
int z2b_last_step_active(const z2b_ctx* ctx, int32_t* out, int cap);

/* Average device time of one expert GEMV launch (which: 0 = gate/up + SwiGLU, 1 = down)
 * over `reps` plain launches that cycle through the MoE layers' weights, on the routing
 * left by the last step; also its algorithmic bytes (routed experts' weights +
 * activations). For the roofline; no reference counterpart. */
int z2b_time_expert_gemv(z2b_ctx* ctx, int which, int reps, double* ms_per_launch, uint64_t* bytes_per_launch);

/* The isolated MoE expert op of one layer (gate/up + SwiGLU + down, weighted sum over
 * each token's routes) on the decode step's own kernels: x[T][n_embd] f32, sel[T][k]
 * expert ids, selw[T][k] route weights -> out[T][n_embd] (out may be NULL). With reps > 0
 * the two expert passes run reps more times between CUDA events and *ms is the time per
 * repetition. *weight_bytes = routed experts' weight bytes; *n_gemm_experts = experts
 * that took the tensor-core GEMM (from T = 64, those with >= 9 routes; or the threshold
 * set by z2b_set_expert_gemm_min at any T). T <= the context's rows per step.
 * No reference counterpart (the reference's expert op is ggml_mul_mat_id inside its graph). */
int z2b_expert_op(z2b_ctx* ctx, int layer, const float* x, int T, const int32_t* sel, const float* selw, int k,
                  float* out, int reps, double* ms, uint64_t* weight_bytes, int32_t* n_gemm_experts);

/* A stream's graph-facing state between steps (zonos2_slot, src/zonos2.h:263-274); the
 * caller owns it, as in the reference. */
#define Z2B_MAX_ROW 32                 /* n_codebooks + 1 input columns at most */
typedef struct z2b_slot_state {
    int32_t index;                     /* cache band / column */
    int32_t done;                      /* finished: EOS countdown elapsed, max_frames, or stopped */
    int32_t n_past;                    /* position of the next row (advanced by the caller per step) */
    int32_t step;                      /* frames sampled so far (frame index of the next sample) */
    int32_t eos_frame;                 /* -1 until an end-of-audio code is seen */
    int32_t countdown;                 /* frames left after EOS, -1 before */
    int32_t next_ids[Z2B_MAX_ROW];     /* next input row: the frame's codes + the text pad */
} z2b_slot_state;

/* Per-frame bookkeeping of zonos2_slot_sample (src/zonos2-graph.cpp:843-870) after the
 * frame codes[n_codebooks] was sampled (z2b_step with Z2B_WANT_SAMPLE): the first frame
 * holding eoa_id in any codebook sets eos_frame = max(0, step - last such codebook) and a
 * countdown of n_codebooks + 1 frames; next_ids = codes + text pad (text_vocab); step + 1;
 * done when the countdown elapses, step reaches max_frames, or keep == 0 (keep: the
 * on_frame callback's verdict, 1 when there is none). Host only; returns keep, or -1 for a
 * bad argument. */
int z2b_slot_after_frame(const z2b_hparams* hp, z2b_slot_state* s, const int32_t* codes, int max_frames, int keep);

const char* z2b_last_error(void);

#ifdef __cplusplus
}
#endif
#endif
