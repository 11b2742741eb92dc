// dac.cpp — DAC decoder: GGUF loading, weight layout for the tcgen05 convolutions, and the
// batched window decode.
//
// Replaces src/dac.cpp:25-102 (dac_load / dac_free: the same GGUF keys and tensor names,
// weights f32 as the reference's converter writes them, models/convert-dac-to-gguf.py) and
// src/dac.cpp:199-315 (dac_run_decoder, dac_decode, dac_decode_window). One call decodes a
// batch of windows (streams) through a single launch sequence instead of one ggml graph
// per window.
#include "dac.h"

#include "gguf.h"
#include "../../include/z2b.h"

#include <cuda_runtime.h>
#include <algorithm>
#include <cmath>
#include <cstring>

namespace z2b {

namespace {

int round_up(int x, int m) { return (x + m - 1) / m * m; }

// f32 (or f16) tensor data of `name` as floats, with its ne; false if missing.
bool read_f32(const GGUFFile& f, const std::string& name, std::vector<float>& out, int64_t ne[4],
              std::string& err) {
    const GTensor* t = f.tensor(name);
    if (!t) { err = "dac: missing tensor '" + name + "'"; return false; }
    const int64_t n = t->nelements();
    out.resize((size_t)n);
    if (t->type == GT_F32) {
        std::memcpy(out.data(), t->data, (size_t)n * 4);
    } else if (t->type == GT_F16) {
        const __half* h = reinterpret_cast<const __half*>(t->data);
        for (int64_t i = 0; i < n; ++i) out[(size_t)i] = __half2float(h[i]);
    } else {
        err = "dac: tensor '" + name + "' has type " + gtype_name(t->type) + " (f32 or f16 expected)";
        return false;
    }
    for (int i = 0; i < 4; ++i) ne[i] = t->ne[i];
    return true;
}

template <class T>
T* upload(DacModel& m, const std::vector<T>& v, std::string& err) {
    void* d = nullptr;
    if (cudaMalloc(&d, std::max<size_t>(v.size(), 1) * sizeof(T)) != cudaSuccess ||
        cudaMemcpy(d, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice) != cudaSuccess) {
        err = "dac: device allocation failed";
        if (d) cudaFree(d);
        m.load_oom = true;
        return nullptr;
    }
    m.allocs.push_back(d);
    return static_cast<T*>(d);
}

bool load_snake(DacModel& m, const GGUFFile& f, const std::string& p, int c, DacSnake& s, std::string& err) {
    std::vector<float> a, inv;
    int64_t ne[4];
    if (!read_f32(f, p + ".alpha", a, ne, err) || !read_f32(f, p + ".inv_alpha", inv, ne, err)) return false;
    if ((int)a.size() != c || (int)inv.size() != c) { err = "dac: " + p + " has the wrong channel count"; return false; }
    s.alpha = upload(m, a, err);
    s.inv = upload(m, inv, err);
    return s.alpha && s.inv;
}

// Conv1d weight, ggml ne [K, IC, OC] (numpy [OC][IC][K]) -> [oc_pad][K][ic_pad] f16.
bool load_conv(DacModel& m, const GGUFFile& f, const std::string& p, int ic, int oc, int k, int dil, DacConv& c,
               std::string& err) {
    std::vector<float> w, b;
    int64_t ne[4], nb[4];
    if (!read_f32(f, p + ".weight", w, ne, err) || !read_f32(f, p + ".bias", b, nb, err)) return false;
    if (ne[0] != k || ne[1] != ic || ne[2] != oc || (int)b.size() != oc) {
        err = "dac: " + p + " has shape [" + std::to_string(ne[0]) + ", " + std::to_string(ne[1]) + ", " +
              std::to_string(ne[2]) + "], expected [" + std::to_string(k) + ", " + std::to_string(ic) + ", " +
              std::to_string(oc) + "]";
        return false;
    }
    c.ic = ic; c.oc = oc; c.ic_pad = round_up(ic, 64); c.oc_pad = round_up(oc, 128);
    c.taps = k; c.dil = dil; c.pad = (k / 2) * dil; c.phases = 1; c.stride = 1;
    std::vector<__half> d((size_t)c.oc_pad * k * c.ic_pad, __float2half(0.0f));
    for (int o = 0; o < oc; ++o)
        for (int i = 0; i < ic; ++i)
            for (int t = 0; t < k; ++t)
                d[((size_t)o * k + t) * c.ic_pad + i] = __float2half_rn(w[((size_t)o * ic + i) * k + t]);
    c.w = upload(m, d, err);
    c.b = upload(m, b, err);
    if (!c.w || !c.b) return false;
    if (!dac_make_wmap(c)) { err = "dac: tensor map for " + p + " failed"; return false; }
    return true;
}

// ConvTranspose1d weight, ggml ne [2s, OC, IC] (numpy [IC][OC][2s]) -> phases
// [s][oc_pad][2][ic_pad] f16 with W_p[o][j][i] = w[i][o][p + j*s].
bool load_convt(DacModel& m, const GGUFFile& f, const std::string& p, int ic, int oc, int s, DacConv& c,
                std::string& err) {
    std::vector<float> w, b;
    int64_t ne[4], nb[4];
    if (!read_f32(f, p + ".weight", w, ne, err) || !read_f32(f, p + ".bias", b, nb, err)) return false;
    if (ne[0] != 2 * s || ne[1] != oc || ne[2] != ic || (int)b.size() != oc || s % 2) {
        err = "dac: " + p + " must be a transposed conv with kernel 2 x stride " + std::to_string(s) +
              " (even), [" + std::to_string(2 * s) + ", " + std::to_string(oc) + ", " + std::to_string(ic) + "]";
        return false;
    }
    c.ic = ic; c.oc = oc; c.ic_pad = round_up(ic, 64); c.oc_pad = round_up(oc, 128);
    c.taps = 2; c.dil = -1; c.pad = 0; c.phases = s; c.stride = s;
    std::vector<__half> d((size_t)s * c.oc_pad * 2 * c.ic_pad, __float2half(0.0f));
    for (int ph = 0; ph < s; ++ph)
        for (int o = 0; o < oc; ++o)
            for (int j = 0; j < 2; ++j)
                for (int i = 0; i < ic; ++i)
                    d[(((size_t)ph * c.oc_pad + o) * 2 + j) * c.ic_pad + i] =
                        __float2half_rn(w[((size_t)i * oc + o) * (2 * s) + ph + j * s]);
    c.w = upload(m, d, err);
    c.b = upload(m, b, err);
    if (!c.w || !c.b) return false;
    if (!dac_make_wmap(c)) { err = "dac: tensor map for " + p + " failed"; return false; }
    return true;
}

uint32_t kv_u32(const GGUFFile& f, const char* k, uint32_t dflt) {
    const GKV* v = f.kv(k);
    return v ? (uint32_t)v->u : dflt;
}

// Grow-only device buffer.
template <class T>
bool ensure(T*& p, size_t& cap, size_t n) {
    if (n <= cap && p) return true;
    if (p) cudaFree(p);
    p = nullptr;
    cap = 0;
    if (cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)) != cudaSuccess) { p = nullptr; return false; }
    cap = n;
    return true;
}

}  // namespace

int DacModel::samples_per_frame() const {
    int spf = 1;
    for (int r : rates) spf *= r;
    return spf;
}

int dac_load(DacModel& m, const char* path, int device, std::string& err) {
    GGUFFile f;
    if (!f.open(path, err)) { err = "dac: cannot open gguf '" + std::string(path) + "': " + err; return Z2B_ERR_IO; }
    if (cudaSetDevice(device) != cudaSuccess) { err = "dac: bad device"; return Z2B_ERR_CUDA; }
    m.device = device;
    m.n_codebooks = (int)kv_u32(f, "dac.n_codebooks", 9);
    m.codebook_size = (int)kv_u32(f, "dac.codebook_size", 1024);
    m.latent = (int)kv_u32(f, "dac.latent_dim", 1024);
    m.decoder_dim = (int)kv_u32(f, "dac.decoder_dim", 1536);
    m.sample_rate = (int)kv_u32(f, "dac.sample_rate", 44100);
    m.hop = (int)kv_u32(f, "dac.hop_length", 512);
    m.pad_id = (int)kv_u32(f, "dac.audio_pad_id", 1025);
    m.rates = {8, 8, 4, 2};
    if (const GKV* r = f.kv("dac.decoder_rates"); r && r->type == GV_ARR && !r->ai.empty())
        m.rates.assign(r->ai.begin(), r->ai.end());
    if (m.n_codebooks < 1 || m.n_codebooks > 16 || m.codebook_size < 1 || m.latent < 1 || m.decoder_dim < 1) {
        err = "dac: unsupported hyperparameters";
        return m.load_oom ? Z2B_ERR_OOM : Z2B_ERR_FORMAT;
    }
    for (int r : m.rates)
        if (r < 2 || r % 2) { err = "dac: decoder rates must be even"; return m.load_oom ? Z2B_ERR_OOM : Z2B_ERR_FORMAT; }
    if ((m.decoder_dim >> m.rates.size()) << m.rates.size() != m.decoder_dim) {
        err = "dac: decoder_dim must divide by 2^blocks";
        return m.load_oom ? Z2B_ERR_OOM : Z2B_ERR_FORMAT;
    }

    // quantizer: tables ne [latent, codebook] -> [codebook][latent], then every codebook
    std::vector<float> all, t, b;
    int64_t ne[4];
    all.reserve((size_t)m.n_codebooks * m.codebook_size * m.latent);
    for (int i = 0; i < m.n_codebooks; ++i) {
        const std::string n = "quant." + std::to_string(i) + ".table";
        if (!read_f32(f, n, t, ne, err)) return m.load_oom ? Z2B_ERR_OOM : Z2B_ERR_FORMAT;
        if (ne[0] != m.latent || ne[1] != m.codebook_size) { err = "dac: " + n + " has the wrong shape"; return m.load_oom ? Z2B_ERR_OOM : Z2B_ERR_FORMAT; }
        all.insert(all.end(), t.begin(), t.end());
    }
    if (!read_f32(f, "quant.bias", b, ne, err)) return m.load_oom ? Z2B_ERR_OOM : Z2B_ERR_FORMAT;
    if ((int)b.size() != m.latent) { err = "dac: quant.bias has the wrong length"; return m.load_oom ? Z2B_ERR_OOM : Z2B_ERR_FORMAT; }
    if (!(m.tables = upload(m, all, err)) || !(m.qbias = upload(m, b, err))) return m.load_oom ? Z2B_ERR_OOM : Z2B_ERR_FORMAT;

    if (!load_conv(m, f, "dec.conv_in", m.latent, m.decoder_dim, 7, 1, m.conv_in, err)) return m.load_oom ? Z2B_ERR_OOM : Z2B_ERR_FORMAT;
    m.blocks.resize(m.rates.size());
    for (size_t bi = 0; bi < m.rates.size(); ++bi) {
        DacBlock& B = m.blocks[bi];
        const std::string p = "dec.b" + std::to_string(bi);
        B.stride = m.rates[bi];
        B.c_in = m.decoder_dim >> bi;
        B.c_out = m.decoder_dim >> (bi + 1);
        if (!load_snake(m, f, p + ".snake", B.c_in, B.snake, err)) return m.load_oom ? Z2B_ERR_OOM : Z2B_ERR_FORMAT;
        if (!load_convt(m, f, p + ".convt", B.c_in, B.c_out, B.stride, B.convt, err)) return m.load_oom ? Z2B_ERR_OOM : Z2B_ERR_FORMAT;
        static const int dils[3] = {1, 3, 9};
        for (int r = 0; r < 3; ++r) {
            const std::string q = p + ".res" + std::to_string(r);
            DacRes& R = B.res[r];
            if (!load_snake(m, f, q + ".snake1", B.c_out, R.s1, err) ||
                !load_conv(m, f, q + ".conv1", B.c_out, B.c_out, 7, dils[r], R.c1, err) ||
                !load_snake(m, f, q + ".snake2", B.c_out, R.s2, err) ||
                !load_conv(m, f, q + ".conv2", B.c_out, B.c_out, 1, 1, R.c2, err))
                return m.load_oom ? Z2B_ERR_OOM : Z2B_ERR_FORMAT;
        }
    }
    m.c_fin = m.decoder_dim >> m.rates.size();
    if (!load_snake(m, f, "dec.snake_out", m.c_fin, m.snake_out, err)) return m.load_oom ? Z2B_ERR_OOM : Z2B_ERR_FORMAT;
    {
        std::vector<float> w, bo;
        int64_t nw[4], nb[4];
        if (!read_f32(f, "dec.conv_out.weight", w, nw, err) || !read_f32(f, "dec.conv_out.bias", bo, nb, err))
            return m.load_oom ? Z2B_ERR_OOM : Z2B_ERR_FORMAT;
        if (nw[0] != 7 || nw[1] != m.c_fin || nw[2] != 1 || bo.size() != 1) {
            err = "dac: dec.conv_out has the wrong shape";
            return m.load_oom ? Z2B_ERR_OOM : Z2B_ERR_FORMAT;
        }
        std::vector<float> wt((size_t)7 * m.c_fin);
        for (int c = 0; c < m.c_fin; ++c)
            for (int k = 0; k < 7; ++k) wt[(size_t)k * m.c_fin + c] = w[(size_t)c * 7 + k];
        if (!(m.w_out = upload(m, wt, err))) return m.load_oom ? Z2B_ERR_OOM : Z2B_ERR_FORMAT;
        m.b_out = bo[0];
    }
    if (cudaStreamCreateWithFlags(&m.stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&m.err, sizeof(uint32_t)) != cudaSuccess) {
        err = "dac: stream or error word allocation failed";
        return Z2B_ERR_CUDA;
    }
    return Z2B_OK;
}

void dac_free(DacModel& m) {
    if (m.device >= 0) cudaSetDevice(m.device);
    if (m.stream) cudaStreamSynchronize(m.stream);
    auto free_conv = [](DacConv& c) { free(c.wmap); c.wmap = nullptr; };
    free_conv(m.conv_in);
    for (DacBlock& B : m.blocks) {
        free_conv(B.convt);
        for (DacRes& R : B.res) { free_conv(R.c1); free_conv(R.c2); }
    }
    for (void* p : m.allocs) cudaFree(p);
    m.allocs.clear();
    for (__half*& s : m.S) { if (s) cudaFree(s); s = nullptr; }
    if (m.X) cudaFree(m.X);
    if (m.audio) cudaFree(m.audio);
    if (m.codes) cudaFree(m.codes);
    if (m.err) cudaFree(m.err);
    if (m.h_stage) cudaFreeHost(m.h_stage);
    if (m.stream) cudaStreamDestroy(m.stream);
    m.X = nullptr; m.audio = nullptr; m.codes = nullptr; m.err = nullptr; m.h_stage = nullptr; m.stream = nullptr;
    m.cap_s[0] = m.cap_s[1] = m.cap_x = m.cap_audio = m.cap_codes = m.cap_h = 0;
}

int dac_decode_batch(DacModel& m, const std::vector<DacWin>& wins, float* audio, int64_t cap, std::string& err,
                      bool audio_on_device) {
    const int n = (int)wins.size();
    if (n == 0) return Z2B_OK;
    if (cudaSetDevice(m.device) != cudaSuccess) { err = "dac: bad device"; return Z2B_ERR_CUDA; }
    const int spf = m.samples_per_frame(), W = m.n_codebooks, nb = (int)m.blocks.size();
    int lmax = 0;
    int64_t total = 0, max_span = 0;
    size_t code_rows = 0;
    std::vector<int> rows(n);
    for (int i = 0; i < n; ++i) {
        const DacWin& w = wins[i];
        if (w.a < 0 || w.b <= w.a || w.H < 0 || (w.H > 0 && !w.codes) || w.s0 < 0 || w.s1 < w.s0 ||
            w.s1 > (int64_t)(w.b - w.a) * spf) {
            err = "dac: bad window " + std::to_string(i);
            return Z2B_ERR_ARG;
        }
        lmax = std::max(lmax, w.b - w.a);
        total += w.s1 - w.s0;
        max_span = std::max<int64_t>(max_span, w.s1 - w.s0);
        rows[i] = std::max(0, std::min(w.H, w.b + W - 1) - w.a);   // code rows the shear reads
        code_rows += rows[i];
    }
    if (total > cap) { err = "dac: output buffer too small"; return Z2B_ERR_ARG; }
    if (total == 0) return Z2B_OK;

    // stage lengths (rows per window) and channel strides
    std::vector<int> L(nb + 1), st(nb + 1);
    L[0] = lmax;
    st[0] = m.conv_in.oc_pad;
    for (int b = 0; b < nb; ++b) {
        if ((int64_t)L[b] * m.blocks[b].stride > (1 << 30)) { err = "dac: window too long"; return Z2B_ERR_ARG; }
        L[b + 1] = L[b] * m.blocks[b].stride;
        st[b + 1] = m.blocks[b].convt.oc_pad;
    }
    const int st_lat = round_up(m.latent, 128);
    size_t need_s = (size_t)n * lmax * std::max(st_lat, st[0]), need_x = 0;
    for (int b = 1; b <= nb; ++b) {
        need_s = std::max(need_s, (size_t)n * L[b] * st[b]);
        need_x = std::max(need_x, (size_t)n * L[b] * st[b]);
    }
    // upload block: codes | window ints [4n] | valid rows per stage [(nb+1) n] | spans int64 [3n]
    const size_t n_int = code_rows * W + 4 * (size_t)n + (size_t)(nb + 1) * n;
    const size_t n_int_al = (n_int + 1) & ~(size_t)1;
    const size_t up_bytes = n_int_al * 4 + (size_t)3 * n * 8;
    if (!ensure(m.S[0], m.cap_s[0], need_s) || !ensure(m.S[1], m.cap_s[1], need_s) ||
        !ensure(m.X, m.cap_x, std::max<size_t>(need_x, 1)) || !ensure(m.audio, m.cap_audio, (size_t)total) ||
        !ensure(m.codes, m.cap_codes, up_bytes / 4)) {
        err = "dac: workspace allocation failed";
        return Z2B_ERR_OOM;
    }
    if (up_bytes > m.cap_h) {
        if (m.h_stage) cudaFreeHost(m.h_stage);
        m.h_stage = nullptr;
        m.cap_h = 0;
        if (cudaHostAlloc(&m.h_stage, up_bytes, cudaHostAllocDefault) != cudaSuccess) {
            err = "dac: pinned staging allocation failed";
            return Z2B_ERR_OOM;
        }
        m.cap_h = up_bytes;
    }
    int32_t* hi = static_cast<int32_t*>(m.h_stage);
    int64_t* hs = reinterpret_cast<int64_t*>(hi + n_int_al);
    int32_t* hwin = hi + code_rows * W;
    int32_t* hlw = hwin + 4 * n;
    size_t off = 0;
    int64_t aoff = 0;
    for (int i = 0; i < n; ++i) {
        const DacWin& w = wins[i];
        if (rows[i] > 0) std::memcpy(hi + off * W, w.codes + (size_t)w.a * W, (size_t)rows[i] * W * 4);
        hwin[4 * i + 0] = (int32_t)off;
        hwin[4 * i + 1] = rows[i];
        hwin[4 * i + 2] = w.a;
        hwin[4 * i + 3] = w.b - w.a;
        int64_t lw = w.b - w.a;
        hlw[i] = (int32_t)lw;
        for (int b = 0; b < nb; ++b) {
            lw *= m.blocks[b].stride;
            hlw[(b + 1) * n + i] = (int32_t)lw;
        }
        hs[3 * i + 0] = w.s0;
        hs[3 * i + 1] = w.s1 - w.s0;
        hs[3 * i + 2] = aoff;
        aoff += w.s1 - w.s0;
        off += rows[i];
    }
    cudaStream_t s = m.stream;
    const int32_t* d_codes = m.codes;
    const int* d_win = m.codes + code_rows * W;
    const int* d_lw = d_win + 4 * n;
    const int64_t* d_spans = reinterpret_cast<const int64_t*>(m.codes + n_int_al);
    long launches = 0;
    bool ok = cudaMemsetAsync(m.err, 0, sizeof(uint32_t), s) == cudaSuccess &&
              cudaMemcpyAsync(m.codes, m.h_stage, up_bytes, cudaMemcpyHostToDevice, s) == cudaSuccess;

    __half* cur = m.S[0];
    __half* nxt = m.S[1];
    ok = ok && launch_dac_latent(m, d_codes, d_win, n, L[0], st_lat, cur, s);
    ++launches;
    auto conv = [&](const DacConv& c, int lin, int c_in_st, int lout, int c_out_st, const int* lw, const float* xres,
                    float* xout, const DacSnake* sn) {
        if (!ok) return;
        DacConvIO io;
        io.in = cur; io.lin = lin; io.c_in_st = c_in_st; io.n_win = n;
        io.xres = xres; io.xout = xout; io.sout = nxt; io.lout = lout; io.c_out_st = c_out_st;
        io.snake = sn; io.lw_out = lw; io.err = m.err;
        ok = launch_dac_conv(c, io, s);
        ++launches;
        std::swap(cur, nxt);
    };
    conv(m.conv_in, L[0], st_lat, L[0], st[0], d_lw, nullptr, nullptr, nb ? &m.blocks[0].snake : &m.snake_out);
    for (int b = 0; b < nb; ++b) {
        const DacBlock& B = m.blocks[b];
        const int* lw = d_lw + (size_t)(b + 1) * n;
        conv(B.convt, L[b], st[b], L[b + 1], st[b + 1], lw, nullptr, m.X, &B.res[0].s1);
        for (int r = 0; r < 3; ++r) {
            const DacSnake* next = r < 2 ? &B.res[r + 1].s1 : (b + 1 < nb ? &m.blocks[b + 1].snake : &m.snake_out);
            conv(B.res[r].c1, L[b + 1], st[b + 1], L[b + 1], st[b + 1], lw, nullptr, nullptr, &B.res[r].s2);
            conv(B.res[r].c2, L[b + 1], st[b + 1], L[b + 1], st[b + 1], lw, m.X, r < 2 ? m.X : nullptr, next);
        }
    }
    ok = ok && launch_dac_out(m, cur, L[nb], st[nb], n, d_spans, max_span, m.audio, s);
    ++launches;
    m.last_launches = launches;
    if (!ok) {
        cudaStreamSynchronize(s);
        err = "dac: launch failed: " + std::string(cudaGetErrorString(cudaGetLastError()));
        return Z2B_ERR_CUDA;
    }
    uint32_t derr = 0;
    ok = cudaMemcpyAsync(audio, m.audio, (size_t)total * 4,
                         audio_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, s) == cudaSuccess &&
         cudaMemcpyAsync(&derr, m.err, sizeof(uint32_t), cudaMemcpyDeviceToHost, s) == cudaSuccess &&
         cudaStreamSynchronize(s) == cudaSuccess;
    if (!ok) { err = "dac: " + std::string(cudaGetErrorString(cudaGetLastError())); return Z2B_ERR_CUDA; }
    if (derr) { err = "dac: device error " + std::to_string(derr); return Z2B_ERR_DEVICE; }
    return Z2B_OK;
}

}  // namespace z2b
