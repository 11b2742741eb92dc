// capi_dac.cpp — extern "C" entry points declared in include/z2b_dac.h.
#include "dac.h"
#include "runtime.h"
#include "z2b_dac.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <new>

using namespace z2b;

struct z2b_dac { DacModel m; };

namespace {

int decode(z2b_dac* dac, const std::vector<DacWin>& wins, float* audio, int64_t cap) {
    std::string err;
    const int rc = dac_decode_batch(dac->m, wins, audio, cap, err);
    if (rc != Z2B_OK) set_error(err);
    return rc;
}

// The window of dac_decode_window (src/dac.cpp:280-299): latent frames [f_lo - Lc (>= 0),
// f_hi + Rc), samples of frames [f_lo, f_hi) kept.
DacWin window(const DacModel& m, const int32_t* codes, int H, int f_lo, int f_hi, int Lc, int Rc) {
    const int64_t spf = m.samples_per_frame();
    DacWin w;
    w.codes = codes;
    w.H = H;
    w.a = std::max(0, f_lo - Lc);
    w.b = f_hi + Rc;
    w.s0 = (int64_t)(f_lo - w.a) * spf;
    w.s1 = (int64_t)(f_hi - w.a) * spf;
    return w;
}

bool window_args_ok(int H, int f_lo, int f_hi, int Lc, int Rc) {
    return H >= 0 && f_lo >= 0 && Lc >= 0 && Rc >= 0 && (int64_t)f_hi + Rc < (1 << 30);
}

}  // namespace

extern "C" {

int z2b_dac_load(const char* path, int device, z2b_dac** out) {
    if (!path || !out) { set_error("null argument"); return Z2B_ERR_ARG; }
    int n_dev = 0;
    if (cudaGetDeviceCount(&n_dev) != cudaSuccess || n_dev == 0) { set_error("no CUDA device"); return Z2B_ERR_CUDA; }
    if (device < 0 || device >= n_dev) { set_error("device index out of range"); return Z2B_ERR_ARG; }
    z2b_dac* d = new (std::nothrow) z2b_dac;
    if (!d) { set_error("out of host memory"); return Z2B_ERR_OOM; }
    std::string err;
    const int rc = dac_load(d->m, path, device, err);
    if (rc != Z2B_OK) {
        dac_free(d->m);
        delete d;
        set_error(err);
        return rc;
    }
    *out = d;
    return Z2B_OK;
}

int z2b_dac_free(z2b_dac* dac) {
    if (!dac) return Z2B_OK;
    dac_free(dac->m);
    delete dac;
    return Z2B_OK;
}

int z2b_dac_get_hparams(const z2b_dac* dac, z2b_dac_hparams* out) {
    if (!dac || !out) { set_error("null argument"); return Z2B_ERR_ARG; }
    const DacModel& m = dac->m;
    std::memset(out, 0, sizeof(*out));
    out->n_codebooks = m.n_codebooks;
    out->codebook_size = m.codebook_size;
    out->latent_dim = m.latent;
    out->decoder_dim = m.decoder_dim;
    out->sample_rate = m.sample_rate;
    out->hop_length = m.hop;
    out->audio_pad_id = m.pad_id;
    out->n_rates = (int32_t)std::min<size_t>(m.rates.size(), 8);
    for (int i = 0; i < out->n_rates; ++i) out->rates[i] = m.rates[i];
    out->samples_per_frame = m.samples_per_frame();
    return Z2B_OK;
}

int z2b_dac_decode(z2b_dac* dac, const int32_t* codes, int H, int W, int eos, float* audio, int64_t cap,
                   int64_t* n_samples) {
    if (!dac || !n_samples || (H > 0 && !codes)) { set_error("null argument"); return Z2B_ERR_ARG; }
    *n_samples = 0;
    if (W != dac->m.n_codebooks) {
        set_error("dac: codes have " + std::to_string(W) + " codebooks, expected " + std::to_string(dac->m.n_codebooks));
        return Z2B_ERR_ARG;
    }
    const int E = eos >= 0 ? std::min(eos, H) : H;     // rows after shear_up + truncate
    if (E <= 0) { set_error("dac: no frames to decode"); return Z2B_ERR_ARG; }
    DacWin w;
    w.codes = codes;
    w.H = H;
    w.a = 0;
    w.b = E;
    w.s0 = 0;
    w.s1 = (int64_t)E * dac->m.samples_per_frame();
    if (!audio && w.s1 > 0) { set_error("null argument"); return Z2B_ERR_ARG; }
    const int rc = decode(dac, {w}, audio, cap);
    if (rc == Z2B_OK) *n_samples = w.s1;
    return rc;
}

int z2b_dac_decode_window(z2b_dac* dac, const int32_t* codes, int H, int f_lo, int f_hi, int Lc, int Rc,
                          float* audio, int64_t cap, int64_t* n_samples) {
    if (!dac || !n_samples || (H > 0 && !codes)) { set_error("null argument"); return Z2B_ERR_ARG; }
    *n_samples = 0;
    if (f_hi <= f_lo) return Z2B_OK;
    if (!window_args_ok(H, f_lo, f_hi, Lc, Rc)) { set_error("dac: bad window"); return Z2B_ERR_ARG; }
    const DacWin w = window(dac->m, codes, H, f_lo, f_hi, Lc, Rc);
    if (!audio) { set_error("null argument"); return Z2B_ERR_ARG; }
    const int rc = decode(dac, {w}, audio, cap);
    if (rc == Z2B_OK) *n_samples = w.s1 - w.s0;
    return rc;
}

int z2b_dac_decode_windows(z2b_dac* dac, const z2b_dac_window* windows, int n, float* audio, int64_t cap,
                           int64_t* n_samples) {
    if (!dac || n < 0 || (n > 0 && (!windows || !n_samples))) { set_error("null argument"); return Z2B_ERR_ARG; }
    std::vector<DacWin> wins;
    wins.reserve(n);
    for (int i = 0; i < n; ++i) {
        const z2b_dac_window& x = windows[i];
        n_samples[i] = 0;
        if (x.f_hi <= x.f_lo) continue;
        if (!window_args_ok(x.H, x.f_lo, x.f_hi, x.Lc, x.Rc) || (x.H > 0 && !x.codes)) {
            set_error("dac: bad window " + std::to_string(i));
            return Z2B_ERR_ARG;
        }
        wins.push_back(window(dac->m, x.codes, x.H, x.f_lo, x.f_hi, x.Lc, x.Rc));
    }
    if (wins.empty()) return Z2B_OK;
    if (!audio) { set_error("null argument"); return Z2B_ERR_ARG; }
    const int rc = decode(dac, wins, audio, cap);
    if (rc != Z2B_OK) return rc;
    for (int i = 0, j = 0; i < n; ++i)
        if (windows[i].f_hi > windows[i].f_lo) { n_samples[i] = wins[j].s1 - wins[j].s0; ++j; }
    return Z2B_OK;
}

long z2b_dac_last_launches(const z2b_dac* dac) { return dac ? dac->m.last_launches : -1; }

void* z2b_dac_stream(z2b_dac* dac) { return dac ? (void*)dac->m.stream : nullptr; }

int64_t z2b_dac_wav_bytes(const float* audio, int64_t n, int sample_rate, uint8_t* out, int64_t cap) {
    if (n < 0 || (n > 0 && !audio)) return -1;
    const int64_t size = 44 + 2 * n;
    if (!out || cap < size) return size;
    const uint32_t sr = (uint32_t)sample_rate, data = (uint32_t)(2 * n);
    uint8_t* p = out;
    auto put = [&](const void* src, size_t k) { std::memcpy(p, src, k); p += k; };
    auto u32 = [&](uint32_t v) { const uint8_t b[4] = {uint8_t(v), uint8_t(v >> 8), uint8_t(v >> 16), uint8_t(v >> 24)}; put(b, 4); };
    auto u16 = [&](uint16_t v) { const uint8_t b[2] = {uint8_t(v), uint8_t(v >> 8)}; put(b, 2); };
    put("RIFF", 4); u32(36 + data); put("WAVE", 4);
    put("fmt ", 4); u32(16); u16(1); u16(1); u32(sr); u32(sr * 2); u16(2); u16(16);
    put("data", 4); u32(data);
    for (int64_t i = 0; i < n; ++i) {
        const float v = std::min(1.0f, std::max(-1.0f, audio[i]));
        u16((uint16_t)(int16_t)lrintf(v * 32767.0f));
    }
    return size;
}

}  // extern "C"
