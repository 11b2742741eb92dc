// z2o.cpp — CPU oracle for the zonos2 batched backbone decode step.
//
// TEST INFRASTRUCTURE ONLY. This is a plain C++ restatement of the reference's ggml CPU
// computation for the hot path, used by tests/, __graft_entry__.smoke() and the
// cpu_baseline leg of bench.py as the checker; no product code path links or calls it.
//
// Parity of the graph arithmetic is UNPINNED: the reference's math lives in ggml
// (git submodule @3af5f57, not vendored), so no reference output for this path can be
// produced here and the reference commits no golden vectors. What is pinned: block
// dequantisation (bit-exact with gguf-py 0.19.0, checked by the tests), the sampler's
// RNG consumption (std::mt19937 + uniform_real_distribution, as the reference uses), and
// the graph structure restated below with file:line citations.
//
// Restated from the reference (paths relative to the zonos2.cpp project):
//   build_graph            src/zonos2-graph.cpp:242-366
//   build_attention        src/zonos2-graph.cpp:101-176
//   build_dense_ffn        src/zonos2-graph.cpp:179-185
//   build_moe              src/zonos2-graph.cpp:191-239
//   zonos2_batch_slot_prefill / zonos2_batch_step  src/zonos2-graph.cpp:703-837
//   zonos2_sampler::sample / accept                src/zonos2-sampler.cpp:9-77
// Modes: Z2O_EXACT computes in f32 with dequantised weights and double accumulation;
// Z2O_GGML_EMU additionally quantises activations the way ggml-cpu's vec-dot kernels do
// (Q8_0 rows for Q8_0 weights, Q8_K super-blocks for K-quants, f16 for F16 weights) and
// accumulates decode-attention V in f16, to estimate the reference CPU path's own error.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <deque>
#include <random>
#include <vector>

namespace {

enum { T_F32 = 0, T_F16 = 1, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14, T_BF16 = 30 };
enum { Z2O_EXACT = 0, Z2O_GGML_EMU = 1 };

// ---------------------------------------------------------------- f16
uint16_t f2h(float f) {
    uint32_t x; std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u, exp = (x >> 23) & 0xffu;
    uint32_t man = x & 0x7fffffu;
    if (exp == 0xff) return (uint16_t)(sign | 0x7c00u | (man ? 0x200u : 0u));
    int e = (int)exp - 112;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        man |= 0x800000u;
        const int sh = 14 - e;
        uint32_t h = man >> sh;
        const uint32_t rem = man & ((1u << sh) - 1u), half = 1u << (sh - 1);
        if (rem > half || (rem == half && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((uint32_t)e << 10) | (man >> 13);
    const uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}
float h2f(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu, x;
    if (exp == 0) {
        if (!man) x = sign;
        else { int e = -1; do { e++; man <<= 1; } while (!(man & 0x400u)); x = sign | ((uint32_t)(112 - e) << 23) | ((man & 0x3ffu) << 13); }
    } else if (exp == 31) x = sign | 0x7f800000u | (man << 13);
    else x = sign | ((exp + 112) << 23) | (man << 13);
    float f; std::memcpy(&f, &x, 4); return f;
}
inline float rnd16(float v) { return h2f(f2h(v)); }

// ---------------------------------------------------------------- blocks (gguf-py order)
inline void q4k_sm(const uint8_t* s, int j, int* sc, int* m) {
    if (j < 4) { *sc = s[j] & 63; *m = s[j + 4] & 63; }
    else { *sc = (s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4); *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4); }
}

size_t row_bytes(uint32_t t, int64_t n) {
    switch (t) {
        case T_F32: return (size_t)n * 4;
        case T_F16: case T_BF16: return (size_t)n * 2;
        case T_Q8_0: return (size_t)(n / 32) * 34;
        case T_Q4_K: return (size_t)(n / 256) * 144;
        case T_Q6_K: return (size_t)(n / 256) * 210;
        default: return 0;
    }
}

// Dequantise one row, bit-exact with gguf.quants.dequantize (quants.py:396-401, 504-522, 554-572).
void deq(uint32_t t, const uint8_t* in, float* out, int64_t n) {
    switch (t) {
        case T_F32: std::memcpy(out, in, (size_t)n * 4); break;
        case T_F16: for (int64_t i = 0; i < n; ++i) { uint16_t h; std::memcpy(&h, in + 2 * i, 2); out[i] = h2f(h); } break;
        case T_BF16: for (int64_t i = 0; i < n; ++i) { uint16_t h; std::memcpy(&h, in + 2 * i, 2); uint32_t u = (uint32_t)h << 16; std::memcpy(out + i, &u, 4); } break;
        case T_Q8_0:
            for (int64_t b = 0; b < n / 32; ++b) {
                uint16_t dh; std::memcpy(&dh, in + b * 34, 2);
                const float d = h2f(dh);
                for (int i = 0; i < 32; ++i) out[b * 32 + i] = (float)(int8_t)in[b * 34 + 2 + i] * d;
            }
            break;
        case T_Q4_K:
            for (int64_t b = 0; b < n / 256; ++b) {
                const uint8_t* k = in + b * 144;
                uint16_t dh, mh; std::memcpy(&dh, k, 2); std::memcpy(&mh, k + 2, 2);
                const float d = h2f(dh), dmin = h2f(mh);
                for (int j = 0; j < 8; ++j) {
                    int sc, m; q4k_sm(k + 4, j, &sc, &m);
                    const float ds = d * (float)sc, dm = dmin * (float)m;
                    for (int i = 0; i < 32; ++i) {
                        const int q = (k[16 + (j / 2) * 32 + i] >> (4 * (j & 1))) & 15;
                        const float p = ds * (float)q;
                        out[b * 256 + j * 32 + i] = p - dm;
                    }
                }
            }
            break;
        case T_Q6_K:
            for (int64_t b = 0; b < n / 256; ++b) {
                const uint8_t* k = in + b * 210;
                uint16_t dh; std::memcpy(&dh, k + 208, 2);
                const float d = h2f(dh);
                for (int e = 0; e < 256; ++e) {
                    const int g = e / 32, i = e % 32;
                    const int lo = (k[(g / 4) * 64 + (g % 2) * 32 + i] >> (4 * ((g % 4) / 2))) & 15;
                    const int hi = (k[128 + (g / 4) * 32 + i] >> (2 * (g % 4))) & 3;
                    const float ds = d * (float)(int8_t)k[192 + e / 16];
                    out[b * 256 + e] = ds * (float)((lo | (hi << 4)) - 32);
                }
            }
            break;
        default: for (int64_t i = 0; i < n; ++i) out[i] = NAN;
    }
}

// ---------------------------------------------------------------- model
struct OT { const uint8_t* data; uint32_t type; int64_t ne0, ne1, ne2; };

struct OLayer {
    OT attn_norm, ffn_norm, wq, wk, wv, wo, temp, gate;
    OT up, gt, down;                      // dense (up = chunk0, gate = chunk1)
    OT gexp, uexp, dexp, rdown, rdown_b, m0, m0b, m2, m2b, m4, rnorm, rbias, eda;
    int is_moe, top_k;
    std::vector<float> mask;              // runtime expert mask (empty = none)
};

struct OHp {
    int n_layer, n_embd, head_dim, n_head, n_head_kv, n_ff, n_codebooks, audio_vocab, text_vocab, eoa_id, n_ctx_train;
    float rope_base, rms_eps, qk_eps, softcap;
};

struct OModel {
    OHp hp;
    OT audio[16], text, out_norm, output;
    OT spk_lda_w, spk_lda_b, spk_proj_w, spk_proj_b;   // speaker projection (optional)
    std::vector<OLayer> L;
    int mode = Z2O_EXACT;
};

std::vector<float> small(const OT& t) {
    std::vector<float> v((size_t)(t.ne0 * t.ne1 * std::max<int64_t>(1, t.ne2)));
    deq(t.type, t.data, v.data(), (int64_t)v.size());
    return v;
}

// ---- activation quantisation of ggml-cpu vec-dot (emu mode)
// Q8_0 row (quantize_row_q8_0_ref): d = amax/127, q = round(x/d), d kept as f16.
void quant_q8_0(const float* x, int64_t n, std::vector<int8_t>& q, std::vector<float>& d) {
    q.resize((size_t)n); d.resize((size_t)(n / 32));
    for (int64_t b = 0; b < n / 32; ++b) {
        float amax = 0.0f;
        for (int i = 0; i < 32; ++i) amax = std::max(amax, std::fabs(x[b * 32 + i]));
        const float dd = amax / 127.0f, id = dd ? 1.0f / dd : 0.0f;
        d[b] = rnd16(dd);
        for (int i = 0; i < 32; ++i) q[b * 32 + i] = (int8_t)std::lround(x[b * 32 + i] * id);
    }
}
// Q8_K super-block (quantize_row_q8_K_ref): scale from the signed max, d kept f32.
void quant_q8_k(const float* x, int64_t n, std::vector<int8_t>& q, std::vector<float>& d) {
    q.resize((size_t)n); d.resize((size_t)(n / 256));
    for (int64_t b = 0; b < n / 256; ++b) {
        float amax = 0.0f, mx = 0.0f;
        for (int i = 0; i < 256; ++i) { const float a = std::fabs(x[b * 256 + i]); if (a > amax) { amax = a; mx = x[b * 256 + i]; } }
        if (amax == 0.0f) { d[b] = 0.0f; for (int i = 0; i < 256; ++i) q[b * 256 + i] = 0; continue; }
        const float iscale = -127.0f / mx;
        for (int i = 0; i < 256; ++i) q[b * 256 + i] = (int8_t)std::min(127, (int)std::lround(iscale * x[b * 256 + i]));
        d[b] = 1.0f / iscale;
    }
}

struct ActQ { std::vector<int8_t> q; std::vector<float> d; std::vector<float> f16; };

void prep_act(int mode, uint32_t wtype, const float* x, int64_t n, ActQ& a) {
    if (mode != Z2O_GGML_EMU) return;
    if (wtype == T_Q8_0) quant_q8_0(x, n, a.q, a.d);
    else if (wtype == T_Q4_K || wtype == T_Q6_K) quant_q8_k(x, n, a.q, a.d);
    else if (wtype == T_F16) { a.f16.resize((size_t)n); for (int64_t i = 0; i < n; ++i) a.f16[i] = rnd16(x[i]); }
}

// dot of weight row (raw blocks) with activation x
float dot_row(int mode, uint32_t t, const uint8_t* w, const float* wf, const float* x, const ActQ& a, int64_t n) {
    if (mode != Z2O_GGML_EMU || t == T_F32 || t == T_BF16) {
        double s = 0.0;
        for (int64_t i = 0; i < n; ++i) s += (double)wf[i] * (double)x[i];
        return (float)s;
    }
    if (t == T_F16) {
        double s = 0.0;
        for (int64_t i = 0; i < n; ++i) s += (double)(wf[i] * a.f16[i]);
        return (float)s;
    }
    if (t == T_Q8_0) {
        float s = 0.0f;
        for (int64_t b = 0; b < n / 32; ++b) {
            uint16_t dh; std::memcpy(&dh, w + b * 34, 2);
            int isum = 0;
            for (int i = 0; i < 32; ++i) isum += (int)(int8_t)w[b * 34 + 2 + i] * (int)a.q[b * 32 + i];
            s += (float)isum * (h2f(dh) * a.d[b]);
        }
        return s;
    }
    float s = 0.0f;
    for (int64_t b = 0; b < n / 256; ++b) {
        const int8_t* q8 = a.q.data() + b * 256;
        if (t == T_Q4_K) {
            const uint8_t* k = w + b * 144;
            uint16_t dh, mh; std::memcpy(&dh, k, 2); std::memcpy(&mh, k + 2, 2);
            int64_t isum = 0, imin = 0;
            for (int j = 0; j < 8; ++j) {
                int sc, m; q4k_sm(k + 4, j, &sc, &m);
                int sub = 0, bs = 0;
                for (int i = 0; i < 32; ++i) {
                    const int q = (k[16 + (j / 2) * 32 + i] >> (4 * (j & 1))) & 15;
                    sub += q * q8[j * 32 + i];
                    bs += q8[j * 32 + i];
                }
                isum += (int64_t)sc * sub;
                imin += (int64_t)m * bs;
            }
            s += h2f(dh) * a.d[b] * (float)isum - h2f(mh) * a.d[b] * (float)imin;
        } else {
            const uint8_t* k = w + b * 210;
            uint16_t dh; std::memcpy(&dh, k + 208, 2);
            int64_t isum = 0;
            for (int j = 0; j < 16; ++j) {
                int sub = 0;
                for (int i = 0; i < 16; ++i) {
                    const int e = j * 16 + i, g = e / 32, ii = e % 32;
                    const int lo = (k[(g / 4) * 64 + (g % 2) * 32 + ii] >> (4 * ((g % 4) / 2))) & 15;
                    const int hi = (k[128 + (g / 4) * 32 + ii] >> (2 * (g % 4))) & 3;
                    sub += ((lo | (hi << 4)) - 32) * q8[e];
                }
                isum += (int64_t)(int8_t)k[192 + j] * sub;
            }
            s += h2f(dh) * a.d[b] * (float)isum;
        }
    }
    return s;
}

// Y[t][r] = W[r] . X[t] for rows [r0, r0+nr) of expert slice `ex`; X is [nt][K]
void matmul(int mode, const OT& W, int ex, const float* X, int nt, float* Y, int ldy) {
    const int64_t K = W.ne0, R = W.ne1;
    const size_t rb = row_bytes(W.type, K);
    const uint8_t* base = W.data + (size_t)ex * R * rb;
    std::vector<ActQ> acts((size_t)nt);
    for (int t = 0; t < nt; ++t) prep_act(mode, W.type, X + (size_t)t * K, K, acts[t]);
#pragma omp parallel
    {
        std::vector<float> wf((size_t)K);
#pragma omp for schedule(static)
        for (int64_t r = 0; r < R; ++r) {
            deq(W.type, base + (size_t)r * rb, wf.data(), K);
            for (int t = 0; t < nt; ++t)
                Y[(size_t)t * ldy + r] = dot_row(mode, W.type, base + (size_t)r * rb, wf.data(), X + (size_t)t * K, acts[t], K);
        }
    }
}

// ggml_rms_norm (sum in double, scale = 1/sqrt(mean + eps)), optional weight (rms_w, :92-95)
void rms_norm(const float* x, int n, float eps, const float* w, float* y) {
    double s = 0.0;
    for (int i = 0; i < n; ++i) s += (double)(x[i] * x[i]);
    const float mean = (float)(s / n);
    const float sc = 1.0f / std::sqrt(mean + eps);
    for (int i = 0; i < n; ++i) { y[i] = x[i] * sc; if (w) y[i] = y[i] * w[i]; }
}

// ---------------------------------------------------------------- context
struct OCtx {
    OModel* m;
    int n_slots, cap;
    std::vector<std::vector<uint16_t>> K, V;   // per layer [slot][cap][nkv][hd] f16
    std::vector<float> logits;                 // last call's output rows
    std::vector<int> sel_log;                  // [layer][token][k] of the last call
    std::vector<float> probs_log;              // [layer][token][E]
};

// interleaved RoPE as ggml's cache init: theta = pos, theta *= base^(-2/hd) per pair
void rope(float* x, int hd, int pos, float base) {
    const float ts = std::pow(base, -2.0f / (float)hd);
    float theta = (float)pos;
    for (int i = 0; i < hd / 2; ++i) {
        const float c = std::cos(theta), s = std::sin(theta);
        const float x0 = x[2 * i], x1 = x[2 * i + 1];
        x[2 * i] = x0 * c - x1 * s;
        x[2 * i + 1] = x0 * s + x1 * c;
        theta *= ts;
    }
}

float gelu_erf(float x) { return 0.5f * x * (1.0f + std::erf(x * 0.70710678118654752440f)); }
float silu(float x) { return x / (1.0f + std::exp(-x)); }
float sigm(float x) { return 1.0f / (1.0f + std::exp(-x)); }

// The stateful EDA router of one MoE layer (src/zonos2-graph.cpp:199-220) on the
// ffn-normed rows cur[n][d]: rh = Wd cur + b (+ state * eda_scale when a previous MoE layer
// left a state), which becomes the state; RMSNorm * router_norm, two erf-GELU layers,
// logits (+ mask), softmax (double sum), top-k of probs + bias (+ mask) with ties to the
// lower id; weight = probs[sel] (no renormalisation).
void router(const OModel& M, const OLayer& ly, const float* cur, int n, std::vector<float>& rstate, bool have_state,
            std::vector<int>& sel, std::vector<float>& w, std::vector<float>& probs) {
    const OHp& hp = M.hp;
    const int mode = M.mode;
    const int E = (int)ly.uexp.ne2, kk = ly.top_k;
    const int rd = (int)ly.rdown.ne1;
    const std::vector<float> rb = small(ly.rdown_b), b0 = small(ly.m0b), b2 = small(ly.m2b), rnw = small(ly.rnorm),
                             rbias = small(ly.rbias);
    std::vector<float> eda;
    if (ly.eda.data) eda = small(ly.eda);
    std::vector<float> rh((size_t)n * rd), h0((size_t)n * rd), h2((size_t)n * rd), lg((size_t)n * E);
    matmul(mode, ly.rdown, 0, cur, n, rh.data(), rd);
    for (int t = 0; t < n; ++t)
        for (int i = 0; i < rd; ++i) {
            float vv = rh[(size_t)t * rd + i] + rb[i];
            if (!eda.empty() && have_state) vv = vv + rstate[(size_t)t * rd + i] * eda[i];
            rh[(size_t)t * rd + i] = vv;
        }
    rstate = rh;
    std::vector<float> rn((size_t)n * rd);
    for (int t = 0; t < n; ++t) rms_norm(&rh[(size_t)t * rd], rd, hp.rms_eps, rnw.data(), &rn[(size_t)t * rd]);
    matmul(mode, ly.m0, 0, rn.data(), n, h0.data(), rd);
    for (int t = 0; t < n; ++t) for (int i = 0; i < rd; ++i) h0[(size_t)t * rd + i] = gelu_erf(h0[(size_t)t * rd + i] + b0[i]);
    matmul(mode, ly.m2, 0, h0.data(), n, h2.data(), rd);
    for (int t = 0; t < n; ++t) for (int i = 0; i < rd; ++i) h2[(size_t)t * rd + i] = gelu_erf(h2[(size_t)t * rd + i] + b2[i]);
    matmul(mode, ly.m4, 0, h2.data(), n, lg.data(), E);
    sel.assign((size_t)n * kk, 0);
    w.assign((size_t)n * kk, 0.0f);
    probs.assign((size_t)n * E, 0.0f);
    for (int t = 0; t < n; ++t) {
        float* p = &probs[(size_t)t * E];
        for (int e = 0; e < E; ++e) p[e] = lg[(size_t)t * E + e] + (ly.mask.empty() ? 0.0f : ly.mask[e]);
        float mx = -INFINITY;
        for (int e = 0; e < E; ++e) mx = std::max(mx, p[e]);
        double sum = 0.0;
        for (int e = 0; e < E; ++e) { p[e] = std::exp(p[e] - mx); sum += p[e]; }
        const float inv = (float)(1.0 / sum);
        for (int e = 0; e < E; ++e) p[e] = p[e] * inv;
        // top-k of probs + bias (+ mask); ties to the lower id
        std::vector<char> taken((size_t)E, 0);
        for (int j = 0; j < kk; ++j) {
            int best = -1; float bv = -INFINITY;
            for (int e = 0; e < E; ++e) {
                if (taken[e]) continue;
                float sv = p[e] + rbias[e];
                if (!ly.mask.empty()) sv = sv + ly.mask[e];
                if (best < 0 || sv > bv) { bv = sv; best = e; }
            }
            taken[best] = 1;
            sel[(size_t)t * kk + j] = best;
            w[(size_t)t * kk + j] = p[best];
        }
    }
}

// One forward over `n` tokens. prefill: all tokens belong to `pslot`, positions 0..n-1,
// self-attention in f32 over these tokens (manual path, :155-169) and K/V written to the
// cache as f16; decode: token t of slot slots[t] at pos[t] attends the f16 cache [0, pos]
// (flash-attn path, :139-153). Logits rows for tokens with want[t].
void forward(OCtx* c, const int32_t* ids, int n, const int* slots, const int* pos, bool prefill,
             const char* want, float* out_logits, const float* over_row = nullptr, int over_t = -1) {
    OModel& M = *c->m;
    const OHp& hp = M.hp;
    const int d = hp.n_embd, hd = hp.head_dim, nh = hp.n_head, nkv = hp.n_head_kv, G = nh / nkv;
    const int ncb = hp.n_codebooks, av = hp.audio_vocab, mode = M.mode;
    // embedding sum + emb_norm (:249-260, :300); token over_t takes the speaker row instead
    // of the sum (:262-292)
    std::vector<float> x((size_t)n * d), res((size_t)n * d), cur((size_t)n * d), row((size_t)d);
    for (int t = 0; t < n; ++t) {
        float* e = &x[(size_t)t * d];
        if (t == over_t) {
            for (int i = 0; i < d; ++i) e[i] = over_row[i];
            rms_norm(e, d, hp.rms_eps, nullptr, e);
            continue;
        }
        for (int k = 0; k <= ncb; ++k) {
            const OT& tb = k < ncb ? M.audio[k] : M.text;
            const int id = ids[t * (ncb + 1) + k];
            deq(tb.type, tb.data + (size_t)id * row_bytes(tb.type, d), row.data(), d);
            for (int i = 0; i < d; ++i) e[i] = k == 0 ? row[i] : e[i] + row[i];
        }
        rms_norm(e, d, hp.rms_eps, nullptr, e);
    }
    std::vector<float> rstate;               // EDA router state across MoE layers (:200-203)
    bool have_state = false;
    c->sel_log.clear(); c->probs_log.clear();
    for (int L = 0; L < hp.n_layer; ++L) {
        const OLayer& ly = M.L[L];
        if (L == 0) res = x; else for (size_t i = 0; i < res.size(); ++i) res[i] = x[i] + res[i];   // :332
        const std::vector<float> an = small(ly.attn_norm), fn = small(ly.ffn_norm), tmp = small(ly.temp);
        for (int t = 0; t < n; ++t) rms_norm(&res[(size_t)t * d], d, hp.rms_eps, an.data(), &cur[(size_t)t * d]);
        // ---- attention (:101-176)
        std::vector<float> q((size_t)n * nh * hd), k((size_t)n * nkv * hd), v((size_t)n * nkv * hd), g((size_t)n * nh);
        matmul(mode, ly.wq, 0, cur.data(), n, q.data(), nh * hd);
        matmul(mode, ly.wk, 0, cur.data(), n, k.data(), nkv * hd);
        matmul(mode, ly.wv, 0, cur.data(), n, v.data(), nkv * hd);
        matmul(mode, ly.gate, 0, cur.data(), n, g.data(), nh);
        for (int t = 0; t < n; ++t) {
            for (int h = 0; h < nh; ++h) {
                float* qh = &q[((size_t)t * nh + h) * hd];
                rms_norm(qh, hd, hp.qk_eps, nullptr, qh);
                for (int i = 0; i < hd; ++i) qh[i] = qh[i] * tmp[h];
                rope(qh, hd, pos[t], hp.rope_base);
            }
            for (int h = 0; h < nkv; ++h) {
                float* kh = &k[((size_t)t * nkv + h) * hd];
                rms_norm(kh, hd, hp.qk_eps, nullptr, kh);
                rope(kh, hd, pos[t], hp.rope_base);
            }
            // set_rows into the f16 cache (:131-137)
            for (int h = 0; h < nkv; ++h)
                for (int i = 0; i < hd; ++i) {
                    const size_t at = ((((size_t)slots[t] * c->cap + pos[t]) * nkv) + h) * hd + i;
                    c->K[L][at] = f2h(k[((size_t)t * nkv + h) * hd + i]);
                    c->V[L][at] = f2h(v[((size_t)t * nkv + h) * hd + i]);
                }
        }
        std::vector<float> o((size_t)n * nh * hd);
        const float scale = 1.0f / std::sqrt((float)hd);
#pragma omp parallel for schedule(dynamic) collapse(2)
        for (int t = 0; t < n; ++t)
            for (int h = 0; h < nh; ++h) {
                const int hk = h / G;
                const float* qh = &q[((size_t)t * nh + h) * hd];
                float* oh = &o[((size_t)t * nh + h) * hd];
                const int nk = pos[t] + 1;
                std::vector<float> s((size_t)nk);
                if (prefill) {
                    // manual f32 attention over this prefill's own K/V, causal mask (:155-169)
                    for (int j = 0; j < nk; ++j) {
                        double a = 0.0;
                        for (int i = 0; i < hd; ++i) a += (double)qh[i] * (double)k[((size_t)j * nkv + hk) * hd + i];
                        s[j] = (float)a * scale;
                    }
                    float mx = -INFINITY;
                    for (float z : s) mx = std::max(mx, z);
                    double sum = 0.0;
                    for (float& z : s) { z = std::exp(z - mx); sum += z; }
                    const float inv = (float)(1.0 / sum);
                    for (int i = 0; i < hd; ++i) {
                        double a = 0.0;
                        for (int j = 0; j < nk; ++j) a += (double)(s[j] * inv) * (double)v[((size_t)j * nkv + hk) * hd + i];
                        oh[i] = (float)a;
                    }
                } else {
                    // flash-attn decode over the f16 cache band [0, pos] (:139-153)
                    const size_t sb = (size_t)slots[t] * c->cap;
                    std::vector<float> qr(qh, qh + hd);
                    if (mode == Z2O_GGML_EMU) for (float& z : qr) z = rnd16(z);
                    for (int j = 0; j < nk; ++j) {
                        double a = 0.0;
                        const uint16_t* kr = &c->K[L][((sb + j) * nkv + hk) * hd];
                        for (int i = 0; i < hd; ++i) a += (double)qr[i] * (double)h2f(kr[i]);
                        s[j] = (float)a * scale;
                    }
                    if (mode == Z2O_GGML_EMU) {
                        // online softmax with f16 V accumulation (ggml-cpu VKQ16 path)
                        float M = -INFINITY, S = 0.0f;
                        std::vector<float> acc((size_t)hd, 0.0f);
                        for (int j = 0; j < nk; ++j) {
                            const float Mold = M;
                            float ms = 1.0f, vs = 1.0f;
                            if (s[j] > M) { M = s[j]; ms = std::exp(Mold - M); for (float& z : acc) z = rnd16(z * ms); }
                            else vs = std::exp(s[j] - M);
                            const uint16_t* vr = &c->V[L][((sb + j) * nkv + hk) * hd];
                            for (int i = 0; i < hd; ++i) acc[i] = rnd16(acc[i] + h2f(vr[i]) * vs);
                            S = S * ms + vs;
                        }
                        for (int i = 0; i < hd; ++i) oh[i] = acc[i] / S;
                    } else {
                        float mx = -INFINITY;
                        for (float z : s) mx = std::max(mx, z);
                        double sum = 0.0;
                        for (float& z : s) { z = std::exp(z - mx); sum += z; }
                        for (int i = 0; i < hd; ++i) {
                            double a = 0.0;
                            for (int j = 0; j < nk; ++j) a += (double)s[j] * (double)h2f(c->V[L][((sb + j) * nkv + hk) * hd + i]);
                            oh[i] = (float)(a / sum);
                        }
                    }
                }
                const float gg = sigm(g[(size_t)t * nh + h]);
                for (int i = 0; i < hd; ++i) oh[i] = oh[i] * gg;
            }
        std::vector<float> ao((size_t)n * d);
        matmul(mode, ly.wo, 0, o.data(), n, ao.data(), d);
        for (size_t i = 0; i < res.size(); ++i) res[i] = ao[i] + res[i];          // :345
        for (int t = 0; t < n; ++t) rms_norm(&res[(size_t)t * d], d, hp.rms_eps, fn.data(), &cur[(size_t)t * d]);
        // ---- FFN
        const int ff = hp.n_ff;
        std::fill(x.begin(), x.end(), 0.0f);
        if (!ly.is_moe) {                                                       // :179-185
            std::vector<float> u((size_t)n * ff), gt((size_t)n * ff), y((size_t)n * ff);
            matmul(mode, ly.up, 0, cur.data(), n, u.data(), ff);
            matmul(mode, ly.gt, 0, cur.data(), n, gt.data(), ff);
            for (size_t i = 0; i < y.size(); ++i) y[i] = u[i] * silu(gt[i]);
            matmul(mode, ly.down, 0, y.data(), n, x.data(), d);
            continue;
        }
        // router (:199-220)
        const int E = (int)ly.uexp.ne2, kk = ly.top_k;
        std::vector<int> sel;
        std::vector<float> w, probs;
        router(M, ly, cur.data(), n, rstate, have_state, sel, w, probs);
        have_state = true;
        c->sel_log.insert(c->sel_log.end(), sel.begin(), sel.end());
        c->probs_log.insert(c->probs_log.end(), probs.begin(), probs.end());
        // experts (:222-238): up/gate per route, silu(gate)*up, down, * weight, sum over j
        std::vector<float> outr((size_t)n * kk * d);
        for (int e = 0; e < E; ++e) {
            std::vector<int> rt;
            for (int r = 0; r < n * kk; ++r) if (sel[r] == e) rt.push_back(r);
            if (rt.empty()) continue;
            const int nr = (int)rt.size();
            std::vector<float> xin((size_t)nr * d), u((size_t)nr * ff), gt((size_t)nr * ff), y((size_t)nr * ff),
                dn((size_t)nr * d);
            for (int i = 0; i < nr; ++i) std::memcpy(&xin[(size_t)i * d], &cur[(size_t)(rt[i] / kk) * d], (size_t)d * 4);
            matmul(mode, ly.uexp, e, xin.data(), nr, u.data(), ff);
            matmul(mode, ly.gexp, e, xin.data(), nr, gt.data(), ff);
            for (size_t i = 0; i < y.size(); ++i) y[i] = u[i] * silu(gt[i]);
            matmul(mode, ly.dexp, e, y.data(), nr, dn.data(), d);
            for (int i = 0; i < nr; ++i)
                for (int j = 0; j < d; ++j) outr[(size_t)rt[i] * d + j] = dn[(size_t)i * d + j] * w[rt[i]];
        }
        for (int t = 0; t < n; ++t)
            for (int j = 0; j < kk; ++j)
                for (int i = 0; i < d; ++i) {
                    const float vv = outr[((size_t)t * kk + j) * d + i];
                    x[(size_t)t * d + i] = j == 0 ? vv : x[(size_t)t * d + i] + vv;
                }
    }
    // output (:352-364)
    for (size_t i = 0; i < res.size(); ++i) res[i] = x[i] + res[i];
    const std::vector<float> on = small(M.out_norm);
    std::vector<int> rows;
    for (int t = 0; t < n; ++t) if (want[t]) rows.push_back(t);
    std::vector<float> h((size_t)rows.size() * d);
    for (size_t i = 0; i < rows.size(); ++i) rms_norm(&res[(size_t)rows[i] * d], d, hp.rms_eps, on.data(), &h[i * d]);
    const int nout = ncb * av;
    matmul(mode, M.output, 0, h.data(), (int)rows.size(), out_logits, nout);
    if (hp.softcap > 0.0f)
        for (size_t i = 0; i < rows.size() * nout; ++i)
            out_logits[i] = std::tanh(out_logits[i] * (1.0f / hp.softcap)) * hp.softcap;
}

// ---------------------------------------------------------------- sampler (exact restatement)
struct OSampler {
    float temperature = 1.15f; int top_k = 106; float top_p = 0.0f, min_p = 0.18f, rep_penalty = 1.2f;
    int rep_window = 50, rep_codebooks = 8, greedy = 0;
    std::mt19937 rng;
    std::vector<std::deque<int>> hist;
};

int sample_one(OSampler& sp, const float* in, int cb, int vocab) {
    if (sp.greedy) {
        int best = 0; float bv = in[0];
        for (int i = 1; i < vocab; ++i) if (in[i] > bv) { bv = in[i]; best = i; }
        return best;
    }
    std::vector<float> logit(in, in + vocab);
    if (sp.rep_penalty != 1.0f && cb < sp.rep_codebooks)
        for (int t : sp.hist[cb]) if (t >= 0 && t < vocab) logit[t] = logit[t] > 0.0f ? logit[t] / sp.rep_penalty : logit[t] * sp.rep_penalty;
    if (sp.temperature > 0.0f) for (auto& l : logit) l /= sp.temperature;
    std::vector<int> idx(vocab);
    for (int i = 0; i < vocab; ++i) idx[i] = i;
    const int k = (sp.top_k > 0 && sp.top_k < vocab) ? sp.top_k : vocab;
    if (k < vocab) {
        // descending logit; ties by index (the reference's partial_sort leaves tie order unspecified)
        std::partial_sort(idx.begin(), idx.begin() + k, idx.end(),
                          [&](int a, int b) { return logit[a] > logit[b] || (logit[a] == logit[b] && a < b); });
        idx.resize(k);
    }
    float mx = -1e30f;
    for (int i : idx) mx = std::max(mx, logit[i]);
    std::vector<float> p(idx.size());
    double sum = 0;
    for (size_t j = 0; j < idx.size(); ++j) { p[j] = std::exp(logit[idx[j]] - mx); sum += p[j]; }
    for (auto& x : p) x = (float)(x / sum);
    std::vector<int> ord(idx.size());
    for (size_t j = 0; j < ord.size(); ++j) ord[j] = (int)j;
    std::stable_sort(ord.begin(), ord.end(), [&](int a, int b) { return p[a] > p[b]; });
    std::vector<char> keep(idx.size(), 1);
    if (sp.top_p > 0.0f && sp.top_p < 1.0f) {
        double cc = 0; bool done = false;
        for (int r : ord) { if (done) keep[r] = 0; cc += p[r]; if (cc >= sp.top_p) done = true; }
    }
    if (sp.min_p > 0.0f) {
        const float thr = sp.min_p * p[ord[0]];
        for (size_t j = 0; j < p.size(); ++j) if (p[j] < thr) keep[j] = 0;
    }
    double s2 = 0;
    for (size_t j = 0; j < p.size(); ++j) { if (!keep[j]) p[j] = 0; s2 += p[j]; }
    if (s2 <= 0) return idx[ord[0]];
    std::uniform_real_distribution<double> u(0.0, s2);
    const double r = u(sp.rng);
    double acc = 0;
    for (size_t j = 0; j < p.size(); ++j) { acc += p[j]; if (acc >= r) return idx[j]; }
    return idx[ord[0]];
}

}  // namespace

// ---------------------------------------------------------------- C ABI for the tests
extern "C" {

struct o_tensor { const void* data; uint32_t type; int64_t ne0, ne1, ne2; };
struct o_hparams {
    int n_layer, n_embd, head_dim, n_head, n_head_kv, n_ff, n_codebooks, audio_vocab, text_vocab, eoa_id, n_ctx_train;
    float rope_base, rms_eps, qk_eps, softcap;
};
// Per-layer tensor table, fixed order (missing tensors: data = NULL):
//   0 attn_norm 1 ffn_norm 2 attn_q 3 attn_k 4 attn_v 5 attn_output 6 attn_temp 7 attn_gate
//   8 ffn_up 9 ffn_gate 10 ffn_down (dense)
//   11 ffn_gate_exps 12 ffn_up_exps 13 ffn_down_exps 14 router_down.weight 15 router_down.bias
//   16 router_mlp0.weight 17 .bias 18 router_mlp2.weight 19 .bias 20 router_mlp4.weight
//   21 router_norm 22 router_bias 23 router_eda_scale
#define O_PER_LAYER 24

static OT cv(const o_tensor& t) { return OT{(const uint8_t*)t.data, t.type, t.ne0, t.ne1, t.ne2 ? t.ne2 : 1}; }

void* o_model_new(const o_hparams* hp, const o_tensor* audio, const o_tensor* text, const o_tensor* out_norm,
                  const o_tensor* output, const o_tensor* layers, const int32_t* expert_used, int mode) {
    OModel* m = new OModel();
    m->hp = OHp{hp->n_layer, hp->n_embd, hp->head_dim, hp->n_head, hp->n_head_kv, hp->n_ff, hp->n_codebooks,
                hp->audio_vocab, hp->text_vocab, hp->eoa_id, hp->n_ctx_train, hp->rope_base, hp->rms_eps,
                hp->qk_eps, hp->softcap};
    for (int i = 0; i < hp->n_codebooks; ++i) m->audio[i] = cv(audio[i]);
    m->text = cv(*text); m->out_norm = cv(*out_norm); m->output = cv(*output);
    m->mode = mode;
    m->L.resize(hp->n_layer);
    for (int L = 0; L < hp->n_layer; ++L) {
        const o_tensor* t = layers + (size_t)L * O_PER_LAYER;
        OLayer& ly = m->L[L];
        OT* f[O_PER_LAYER] = {&ly.attn_norm, &ly.ffn_norm, &ly.wq, &ly.wk, &ly.wv, &ly.wo, &ly.temp, &ly.gate,
                              &ly.up, &ly.gt, &ly.down, &ly.gexp, &ly.uexp, &ly.dexp, &ly.rdown, &ly.rdown_b,
                              &ly.m0, &ly.m0b, &ly.m2, &ly.m2b, &ly.m4, &ly.rnorm, &ly.rbias, &ly.eda};
        for (int i = 0; i < O_PER_LAYER; ++i) *f[i] = cv(t[i]);
        ly.top_k = expert_used[L];
        ly.is_moe = ly.top_k > 0;
    }
    return m;
}
void o_model_free(void* m) { delete (OModel*)m; }
void o_model_set_mode(void* m, int mode) { ((OModel*)m)->mode = mode; }
void o_model_set_mask(void* m, int layer, const float* mask, int n) {
    OModel* M = (OModel*)m;
    if (layer < 0 || layer >= (int)M->L.size()) return;
    M->L[layer].mask.assign(mask, mask + (mask ? n : 0));
}

void* o_ctx_new(void* model, int n_slots, int cap) {
    OCtx* c = new OCtx();
    c->m = (OModel*)model;
    c->n_slots = n_slots; c->cap = cap;
    const OHp& hp = c->m->hp;
    const size_t per = (size_t)n_slots * cap * hp.n_head_kv * hp.head_dim;
    c->K.assign(hp.n_layer, std::vector<uint16_t>(per, 0));
    c->V.assign(hp.n_layer, std::vector<uint16_t>(per, 0));
    return c;
}
void o_ctx_free(void* c) { delete (OCtx*)c; }

// zonos2_batch_slot_prefill: prompt ids [n0][ncb+1] -> last row logits [ncb*av]
int o_prefill(void* ctx, int slot, const int32_t* ids, int n0, float* out_logits) {
    OCtx* c = (OCtx*)ctx;
    if (slot < 0 || slot >= c->n_slots || n0 < 1 || n0 > c->cap) return 1;
    std::vector<int> slots(n0, slot), pos(n0);
    std::vector<char> want(n0, 0);
    for (int i = 0; i < n0; ++i) pos[i] = i;
    want[n0 - 1] = 1;
    forward(c, ids, n0, slots.data(), pos.data(), true, want.data(), out_logits);
    return 0;
}

// Speaker projection tensors (t[0..3] = spk_lda.weight, spk_lda.bias, spk_proj.weight,
// spk_proj.bias).
void o_model_set_spk(void* m, const o_tensor* t) {
    OModel* M = (OModel*)m;
    M->spk_lda_w = cv(t[0]); M->spk_lda_b = cv(t[1]); M->spk_proj_w = cv(t[2]); M->spk_proj_b = cv(t[3]);
}

// The projected speaker row (src/zonos2-graph.cpp:262-275): W_proj (W_lda spk + b_lda)
// + b_proj (+ delta), each product through matmul() in the model's arithmetic mode.
int o_spk_row(void* m, const float* spk, const float* delta, float* out_row) {
    OModel* M = (OModel*)m;
    if (!M->spk_lda_w.data || !M->spk_proj_w.data) return 1;
    const int ld = (int)M->spk_lda_w.ne1, d = (int)M->spk_proj_w.ne1;
    std::vector<float> sl((size_t)ld);
    matmul(M->mode, M->spk_lda_w, 0, spk, 1, sl.data(), ld);
    const std::vector<float> lb = small(M->spk_lda_b), pb = small(M->spk_proj_b);
    for (int i = 0; i < ld; ++i) sl[i] = sl[i] + lb[i];
    matmul(M->mode, M->spk_proj_w, 0, sl.data(), 1, out_row, d);
    for (int j = 0; j < d; ++j) {
        out_row[j] = out_row[j] + pb[j];
        if (delta) out_row[j] = out_row[j] + delta[j];
    }
    return 0;
}

// zonos2_batch_slot_prefill with spk / spk_pos / spk_emotion_delta (:703-760, :262-292)
int o_prefill_spk(void* ctx, int slot, const int32_t* ids, int n0, const float* spk, int spk_pos, const float* delta,
                  float* out_logits) {
    OCtx* c = (OCtx*)ctx;
    if (slot < 0 || slot >= c->n_slots || n0 < 1 || n0 > c->cap || spk_pos >= n0) return 1;
    if (!spk || spk_pos < 0) return o_prefill(ctx, slot, ids, n0, out_logits);   // no speaker (:36-37)
    std::vector<float> row((size_t)c->m->hp.n_embd);
    if (o_spk_row(c->m, spk, delta, row.data())) return 1;
    std::vector<int> slots(n0, slot), pos(n0);
    std::vector<char> want(n0, 0);
    for (int i = 0; i < n0; ++i) pos[i] = i;
    want[n0 - 1] = 1;
    forward(c, ids, n0, slots.data(), pos.data(), true, want.data(), out_logits, row.data(), spk_pos);
    return 0;
}

// zonos2_logits: every row's logits of one sequence from position 0, [n][ncb*av]
// (src/zonos2-graph.cpp:457-473), with the optional speaker row as o_prefill_spk.
int o_logits(void* model, const int32_t* ids, int n, const float* spk, int spk_pos, const float* delta,
             float* out_logits) {
    OModel* M = (OModel*)model;
    if (spk_pos < 0) spk = nullptr;                  // no speaker (src/zonos2-graph.cpp:36-37)
    if (n < 1 || (spk && spk_pos >= n)) return 1;
    std::vector<float> row;
    if (spk) {
        row.resize((size_t)M->hp.n_embd);
        if (o_spk_row(M, spk, delta, row.data())) return 1;
    }
    OCtx* c = (OCtx*)o_ctx_new(M, 1, n);
    std::vector<int> slots(n, 0), pos(n);
    std::vector<char> want(n, 1);
    for (int i = 0; i < n; ++i) pos[i] = i;
    forward(c, ids, n, slots.data(), pos.data(), true, want.data(), out_logits, spk ? row.data() : nullptr,
            spk ? spk_pos : -1);
    o_ctx_free(c);
    return 0;
}

// zonos2_batch_step for n active slots: slot[i] at position n_past[i] fed ids[i] -> logits [n][ncb*av]
int o_step(void* ctx, const int32_t* slots, const int32_t* n_past, const int32_t* ids, int n, float* out_logits) {
    OCtx* c = (OCtx*)ctx;
    for (int i = 0; i < n; ++i) if (slots[i] < 0 || slots[i] >= c->n_slots || n_past[i] < 0 || n_past[i] >= c->cap) return 1;
    std::vector<char> want(n, 1);
    forward(c, ids, n, slots, n_past, false, want.data(), out_logits);
    return 0;
}

// Routing of the last call: sel [n_moe_layers][n][k] (k = top-k of those layers).
int o_last_sel(void* ctx, int32_t* out, int cap) {
    OCtx* c = (OCtx*)ctx;
    const int n = std::min<int>(cap, (int)c->sel_log.size());
    for (int i = 0; i < n; ++i) out[i] = c->sel_log[i];
    return (int)c->sel_log.size();
}

// Fill positions [0, n) of a slot's cache with pseudo-random f16 values (timing runs that
// need long contexts without computing their prefill).
void o_ctx_fake_fill(void* ctx, int slot, int n, uint32_t seed) {
    OCtx* c = (OCtx*)ctx;
    const OHp& hp = c->m->hp;
    const size_t row = (size_t)hp.n_head_kv * hp.head_dim;
#pragma omp parallel for schedule(dynamic)
    for (int L = 0; L < hp.n_layer; ++L) {
        std::mt19937 g(seed * 1000u + (uint32_t)L);
        std::normal_distribution<float> nd(0.0f, 1.0f);
        for (int p = 0; p < n && p < c->cap; ++p)
            for (size_t i = 0; i < row; ++i) {
                const size_t at = ((size_t)slot * c->cap + p) * row + i;
                c->K[L][at] = f2h(nd(g));
                c->V[L][at] = f2h(nd(g));
            }
    }
}

// Fill positions [0, n) of a slot's cache with a portable integer hash of (seed, layer,
// K/V, position, kv head, dim) mapped to k / 1024, k in [-2048, 2048): exact in f16. The
// product library's debug fill (z2b_debug_fill_kv) computes the same values, so the GPU
// and this oracle hold identical long contexts without computing a prefill.
static uint16_t kv_hash_f16(uint32_t seed, int layer, int kv, int pos, int head, int dim) {
    uint64_t x = (((((uint64_t)seed * 256u + (uint64_t)layer) * 2u + (uint64_t)kv) * 1048576u + (uint64_t)pos) * 64u +
                  (uint64_t)head) * 1024u + (uint64_t)dim;
    x += 0x9E3779B97F4A7C15ull;                      // splitmix64 finaliser
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    x ^= x >> 31;
    const int v = (int)((x >> 40) & 0xFFFu) - 2048;
    return f2h((float)v / 1024.0f);
}

void o_ctx_hash_fill(void* ctx, int slot, int n, uint32_t seed) {
    OCtx* c = (OCtx*)ctx;
    const OHp& hp = c->m->hp;
#pragma omp parallel for schedule(dynamic)
    for (int L = 0; L < hp.n_layer; ++L)
        for (int p = 0; p < n && p < c->cap; ++p)
            for (int h = 0; h < hp.n_head_kv; ++h)
                for (int i = 0; i < hp.head_dim; ++i) {
                    const size_t at = (((size_t)slot * c->cap + p) * hp.n_head_kv + h) * hp.head_dim + i;
                    c->K[L][at] = kv_hash_f16(seed, L, 0, p, h, i);
                    c->V[L][at] = kv_hash_f16(seed, L, 1, p, h, i);
                }
}

// The router of MoE layer `layer` on given residual rows res[n][d] (ffn_norm applied here)
// and the previous MoE layer's state state_in[n][rd] (NULL: none, the first MoE layer):
// sel[n][k], weights w[n][k] and the new state state_out[n][rd] (may be NULL).
int o_router(void* model, int layer, const float* res, const float* state_in, int n, int32_t* sel_out, float* w_out,
             float* state_out) {
    OModel* M = (OModel*)model;
    if (layer < 0 || layer >= M->hp.n_layer || !M->L[layer].is_moe || n < 1) return 1;
    const OLayer& ly = M->L[layer];
    const int d = M->hp.n_embd, rd = (int)ly.rdown.ne1;
    const std::vector<float> fn = small(ly.ffn_norm);
    std::vector<float> cur((size_t)n * d);
    for (int t = 0; t < n; ++t) rms_norm(res + (size_t)t * d, d, M->hp.rms_eps, fn.data(), &cur[(size_t)t * d]);
    std::vector<float> rstate;
    if (state_in) rstate.assign(state_in, state_in + (size_t)n * rd);
    std::vector<int> sel;
    std::vector<float> w, probs;
    router(*M, ly, cur.data(), n, rstate, state_in != nullptr, sel, w, probs);
    std::copy(sel.begin(), sel.end(), sel_out);
    std::copy(w.begin(), w.end(), w_out);
    if (state_out) std::copy(rstate.begin(), rstate.end(), state_out);
    return 0;
}

void o_dequant(uint32_t type, const void* data, int64_t n, float* out) { deq(type, (const uint8_t*)data, out, n); }

// ---- sampler
void* o_sampler_new(float temperature, int top_k, float top_p, float min_p, float rep_penalty, int rep_window,
                    int rep_codebooks, uint32_t seed, int greedy, int n_codebooks) {
    OSampler* s = new OSampler();
    s->temperature = temperature; s->top_k = top_k; s->top_p = top_p; s->min_p = min_p;
    s->rep_penalty = rep_penalty; s->rep_window = rep_window; s->rep_codebooks = rep_codebooks;
    s->greedy = greedy; s->rng.seed(seed);
    s->hist.assign(n_codebooks, {});
    return s;
}
void o_sampler_free(void* s) { delete (OSampler*)s; }
// sample one frame (all codebooks) from logits [ncb][vocab] and push it into the history
void o_sample_frame(void* sp, const float* logits, int ncb, int vocab, int32_t* codes) {
    OSampler* s = (OSampler*)sp;
    for (int cb = 0; cb < ncb; ++cb) codes[cb] = sample_one(*s, logits + (size_t)cb * vocab, cb, vocab);
    for (int cb = 0; cb < ncb; ++cb) {
        s->hist[cb].push_back(codes[cb]);
        while ((int)s->hist[cb].size() > s->rep_window) s->hist[cb].pop_front();
    }
}

}  // extern "C"
