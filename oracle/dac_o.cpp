// dac_o.cpp — CPU oracle for the DAC decoder (codes -> waveform).
//
// TEST INFRASTRUCTURE ONLY: a plain restatement of the reference's ggml CPU graph for the
// DAC decode, used by tests/ and bench.py's CPU legs as the checker; no product code path
// links or calls it.
//
// Restated from the reference (paths relative to the zonos2.cpp project):
//   dac_build_idx      src/dac.cpp:205-219   shear_up (pad 1025 past H), clamp to [0, 1023]
//   from_codes         src/dac.cpp:228-238   sum of the folded tables in codebook order + bias
//   conv1d             src/dac.cpp:104-116   im2col with f16 patches, weights converted to f16
//                                            by ggml's f16 dot; + bias
//   convt1d            src/dac.cpp:118-163   f32 GEMM per input frame + overlap-add fold
//                                            (kernel 2s, crop s/2 each side); + bias
//   snake              src/dac.cpp:166-171   x + sin(alpha x)^2 * inv_alpha
//   res_unit           src/dac.cpp:177-184   x + conv2(snake2(conv1(snake1(x)))), dil 1/3/9
//   dec_block          src/dac.cpp:186-195
//   dac_run_decoder    src/dac.cpp:240-245   conv_in, blocks, snake_out, conv_out, tanh
// Dot products accumulate in double (the reference sums f16 products in f32 vector lanes);
// every elementwise step is one f32 operation in the reference's order
// (-ffp-contract=off). An exact mode skips the f16 rounding of conv operands, to pin the
// graph's structure against a restatement at f32 precision.
//
// Parity is pinned against a torch restatement of the published DAC decoder (torch's
// conv1d / conv_transpose1d) in the tests, on both a synthetic model and the reference's
// own dummy-dac.gguf fixture when it is readable; the reference's ggml build itself cannot
// run here (its ggml submodule is not vendored).
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

namespace {

// round to the nearest f16 (ties to even), as ggml converts f32 to f16; identity in the
// exact mode
bool g_f16 = true;
float r16(float f) { return g_f16 ? (float)(_Float16)f : f; }

using Mat = std::vector<float>;   // time-major [rows][channels]

// x: [L][IC]; w numpy [OC][IC][K]; y[t][o] = b[o] + sum h(x[t + k dil - pad][i]) h(w[o][i][k])
Mat conv1d(const Mat& x, int L, int IC, const float* w, const float* b, int OC, int K, int dil) {
    const int pad = (K / 2) * dil;
    std::vector<float> wt((size_t)OC * K * IC);        // [o][k][i], f16-rounded
    for (int o = 0; o < OC; ++o)
        for (int i = 0; i < IC; ++i)
            for (int k = 0; k < K; ++k) wt[((size_t)o * K + k) * IC + i] = r16(w[((size_t)o * IC + i) * K + k]);
    std::vector<float> xh(x.size());
    for (size_t i = 0; i < x.size(); ++i) xh[i] = r16(x[i]);
    Mat y((size_t)L * OC);
#pragma omp parallel for schedule(static)
    for (int t = 0; t < L; ++t)
        for (int o = 0; o < OC; ++o) {
            double acc = 0.0;
            for (int k = 0; k < K; ++k) {
                const int r = t + k * dil - pad;
                if (r < 0 || r >= L) continue;
                const float* xr = &xh[(size_t)r * IC];
                const float* wr = &wt[((size_t)o * K + k) * IC];
                for (int i = 0; i < IC; ++i) acc += (double)xr[i] * (double)wr[i];
            }
            y[(size_t)t * OC + o] = (float)acc + b[o];
        }
    return y;
}

// ConvTranspose1d, kernel 2s, stride s, crop s/2 each side: x [L][IC], w numpy [IC][OC][2s]
// -> y [L s][OC]; y[t] = b + lower(x[u / s]) + upper(x[u / s - 1]) at u = t + s/2.
Mat convt1d(const Mat& x, int L, int IC, const float* w, const float* b, int OC, int s) {
    const int K = 2 * s, h = s / 2;
    std::vector<float> wt((size_t)K * OC * IC);        // [k][o][i]
    for (int i = 0; i < IC; ++i)
        for (int o = 0; o < OC; ++o)
            for (int k = 0; k < K; ++k) wt[((size_t)k * OC + o) * IC + i] = w[((size_t)i * OC + o) * K + k];
    Mat y((size_t)L * s * OC);
#pragma omp parallel for schedule(static)
    for (int t = 0; t < L * s; ++t) {
        const int u = t + h, bb = u / s, p = u % s;
        for (int o = 0; o < OC; ++o) {
            // the reference adds the two folded halves (each an f32 GEMM result), then the bias
            float lo = 0.0f, up = 0.0f;
            if (bb < L) {
                double a = 0.0;
                const float* xr = &x[(size_t)bb * IC];
                const float* wr = &wt[((size_t)p * OC + o) * IC];
                for (int i = 0; i < IC; ++i) a += (double)xr[i] * (double)wr[i];
                lo = (float)a;
            }
            if (bb >= 1) {
                double a = 0.0;
                const float* xr = &x[(size_t)(bb - 1) * IC];
                const float* wr = &wt[((size_t)(p + s) * OC + o) * IC];
                for (int i = 0; i < IC; ++i) a += (double)xr[i] * (double)wr[i];
                up = (float)a;
            }
            y[(size_t)t * OC + o] = (lo + up) + b[o];
        }
    }
    return y;
}

Mat snake(const Mat& x, int L, int C, const float* alpha, const float* inv) {
    Mat y(x.size());
#pragma omp parallel for schedule(static)
    for (int t = 0; t < L; ++t)
        for (int c = 0; c < C; ++c) {
            const float v = x[(size_t)t * C + c];
            const float sn = std::sin(v * alpha[c]);
            const float s2 = sn * sn;
            y[(size_t)t * C + c] = v + s2 * inv[c];
        }
    return y;
}

}  // namespace

extern "C" {

struct ODac {
    int n_cb, cb_size, latent, dec_dim, n_blocks, pad_id;
    int f16;                 // 1: conv operands rounded to f16 as the reference; 0: exact f32 inputs
    int rates[8];
    const float* const* t;   // tensors in the order documented in oracle/dac_oracle.py
};

// Decode the latent frames [a, b) of raw codes [H][n_cb]; writes (b - a) * prod(rates)
// samples to out. Returns 0, or -1 on bad arguments.
int o_dac_decode(const ODac* m, const int32_t* codes, int H, int a, int b, float* out) {
    if (!m || b <= a || a < 0 || m->n_blocks > 8) return -1;
    g_f16 = m->f16 != 0;
    const int L0 = b - a, ncb = m->n_cb, lat = m->latent;
    const float* const* T = m->t;
    int ti = 0;
    const float* const* tables = T;
    ti += ncb;
    const float* qbias = T[ti++];
    // from_codes
    Mat z((size_t)L0 * lat);
    for (int l = 0; l < L0; ++l) {
        int idx[16];
        for (int j = 0; j < ncb; ++j) {
            const int t = a + l;
            int v = (t + j < H) ? codes[(size_t)(t + j) * ncb + j] : m->pad_id;
            if (v > 1023) v = 1023;
            if (v < 0) v = 0;
            idx[j] = v;
        }
        for (int c = 0; c < lat; ++c) {
            float s = tables[0][(size_t)idx[0] * lat + c];
            for (int j = 1; j < ncb; ++j) s = s + tables[j][(size_t)idx[j] * lat + c];
            z[(size_t)l * lat + c] = s + qbias[c];
        }
    }
    int L = L0, C = m->dec_dim;
    const float* w = T[ti++];
    const float* bi = T[ti++];
    Mat h = conv1d(z, L, lat, w, bi, C, 7, 1);
    static const int dils[3] = {1, 3, 9};
    for (int blk = 0; blk < m->n_blocks; ++blk) {
        const int s = m->rates[blk], Co = C / 2;
        const float* sa = T[ti++];
        const float* si = T[ti++];
        const float* cw = T[ti++];
        const float* cb = T[ti++];
        Mat y = snake(h, L, C, sa, si);
        h = convt1d(y, L, C, cw, cb, Co, s);
        L *= s;
        C = Co;
        for (int r = 0; r < 3; ++r) {
            const float* a1 = T[ti++];
            const float* i1 = T[ti++];
            const float* w1 = T[ti++];
            const float* b1 = T[ti++];
            const float* a2 = T[ti++];
            const float* i2 = T[ti++];
            const float* w2 = T[ti++];
            const float* b2 = T[ti++];
            Mat u = snake(h, L, C, a1, i1);
            u = conv1d(u, L, C, w1, b1, C, 7, dils[r]);
            u = snake(u, L, C, a2, i2);
            u = conv1d(u, L, C, w2, b2, C, 1, 1);
            for (size_t i = 0; i < h.size(); ++i) h[i] = h[i] + u[i];
        }
    }
    const float* ao = T[ti++];
    const float* io = T[ti++];
    const float* wo = T[ti++];
    const float* bo = T[ti++];
    h = snake(h, L, C, ao, io);
    h = conv1d(h, L, C, wo, bo, 1, 7, 1);
    for (int t = 0; t < L; ++t) out[t] = std::tanh(h[t]);
    return 0;
}

}  // extern "C"
