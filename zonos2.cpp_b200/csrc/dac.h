// dac.h — DAC 44 kHz decoder (codes -> waveform) on the GPU.
//
// Replaces the reference's ggml DAC port (src/dac.h:14-52, src/dac.cpp:199-315): the
// quantizer's folded lookup tables, the conv decoder (conv_in, four upsampling blocks of a
// transposed conv and three dilated residual units, snake activations, conv_out) and tanh.
// The convolutions run as implicit GEMMs on the tcgen05 tensor cores (k_dac.cu); a
// transposed conv with kernel 2s and stride s becomes s phase GEMMs of two taps each.
//
// Device layout: activations time-major per window, [window][rows][channels] with the
// channel stride rounded up to 128; a batch of windows is decoded in one pass, every window
// padded to the longest one's row count (rows past a window's own length hold zeros, as the
// reference's zero padding at the window's end).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <string>
#include <vector>

namespace z2b {

struct DacConv {
    __half* w = nullptr;       // [phases][oc_pad][taps][ic_pad] f16
    float* b = nullptr;        // [oc_pad]
    int ic = 0, oc = 0, ic_pad = 0, oc_pad = 0;
    int taps = 1, dil = 1, pad = 0, phases = 1, stride = 1;
    void* wmap = nullptr;      // host copy of the weight tensor map (CUtensorMap, 128 bytes)
};

struct DacSnake {
    float* alpha = nullptr;    // [c_pad]
    float* inv = nullptr;      // [c_pad]
};

struct DacRes {
    DacSnake s1, s2;
    DacConv c1, c2;
};

struct DacBlock {
    DacSnake snake;
    DacConv convt;
    DacRes res[3];
    int stride = 1, c_in = 0, c_out = 0;
};

// One window of latent frames [a, b) of a stream's sheared codes; samples [s0, s1) of its
// decoded audio are kept.
struct DacWin {
    const int32_t* codes = nullptr;   // raw codes [H][n_codebooks], host
    int H = 0, a = 0, b = 0;
    int64_t s0 = 0, s1 = 0;
};

struct DacModel {
    int device = 0;
    int n_codebooks = 9, codebook_size = 1024, latent = 1024, decoder_dim = 1536;
    int sample_rate = 44100, hop = 512, pad_id = 1025;
    std::vector<int> rates;
    float* tables = nullptr;          // [n_codebooks][codebook_size][latent] f32
    float* qbias = nullptr;           // [latent]
    DacConv conv_in;
    std::vector<DacBlock> blocks;
    DacSnake snake_out;
    float* w_out = nullptr;           // [7][c_fin] f32
    float b_out = 0.0f;
    int c_fin = 0;
    std::vector<void*> allocs;        // every weight allocation, freed together
    // workspace (grown on demand)
    cudaStream_t stream = nullptr;
    __half* S[2] = {nullptr, nullptr};
    float* X = nullptr;
    float* audio = nullptr;
    int32_t* codes = nullptr;         // upload block: codes, per-window tables (dac.cpp)
    uint32_t* err = nullptr;
    size_t cap_s[2] = {0, 0}, cap_x = 0, cap_audio = 0, cap_codes = 0;
    void* h_stage = nullptr;          // pinned host staging
    size_t cap_h = 0;
    long last_launches = 0;
    bool load_oom = false;            // a device allocation failed while loading
    int samples_per_frame() const;
};

// Returns Z2B_OK or a Z2B_ERR_* code (IO: unreadable file, FORMAT: not a usable DAC GGUF,
// OOM: device memory, CUDA: device set-up) with err set.
int dac_load(DacModel& m, const char* path, int device, std::string& err);
void dac_free(DacModel& m);
// Decode the windows in one batched pass; audio receives each window's kept samples in order.
// Returns Z2B_OK or a Z2B_ERR_* code (include/z2b.h) with err set.
int dac_decode_batch(DacModel& m, const std::vector<DacWin>& wins, float* audio, int64_t cap,
                     std::string& err, bool audio_on_device = false);

// ---- kernel launchers (k_dac.cu) ----

// Inputs and outputs of one convolution over a batch of windows.
struct DacConvIO {
    const __half* in = nullptr;   // [n_win][lin][c_in_st] f16 (already snake-activated)
    int lin = 0, c_in_st = 0, n_win = 0;
    const float* xres = nullptr;  // residual added to the output, [n_win][lout][c_out_st] f32 (may alias xout)
    float* xout = nullptr;        // f32 output (the residual stream; rows past lw_out and padding
                                  // channels are left unwritten, as nothing reads them), or null
    __half* sout = nullptr;       // f16 output after the next snake (or as is), [n_win][lout][c_out_st]
    int lout = 0, c_out_st = 0;
    const DacSnake* snake = nullptr;
    const int* lw_out = nullptr;  // [n_win] valid output rows per window; sout rows past it are written as 0
    uint32_t* err = nullptr;
};

// Weight tensor map of a convolution, encoded once at load.
bool dac_make_wmap(DacConv& c);
bool launch_dac_conv(const DacConv& c, const DacConvIO& io, cudaStream_t s);
// Sheared, clamped codes -> latent z (sum of the folded tables + bias), f16, [n_win][lat_rows][c_st].
// Per-window table: win[4 * w + 0..3] = codes offset (rows), rows available, latent frame a, frames.
bool launch_dac_latent(const DacModel& m, const int32_t* codes, const int* win, int n_win, int lat_rows, int c_st,
                       __half* out, cudaStream_t s);
// conv_out (k 7, one output channel) + tanh over the kept samples of each window.
// Per-window device table: spans[3 * w + 0..2] = first kept sample, kept samples, output offset.
bool launch_dac_out(const DacModel& m, const __half* in, int lin, int c_st, int n_win, const int64_t* spans,
                    int64_t max_span, float* audio, cudaStream_t s);

}  // namespace z2b
