/* z2b_dac.h — C ABI of the B200 DAC decoder (codes -> waveform) in libz2b.so.
 *
 * Drop-in for the reference's DAC port, src/dac.h:28-52 (dac_load, dac_free, dac_decode,
 * dac_decode_window, dac_wav_bytes), reading the same GGUF files
 * (models/convert-dac-to-gguf.py). The decoder's convolutions run on the tcgen05 tensor
 * cores; z2b_dac_decode_windows decodes many streams' windows in one pass, which the
 * reference's server does one window per DAC lane thread (src/server.cpp:935-1008).
 * Return codes and z2b_last_error() as in z2b.h. A z2b_dac is used by one thread at a time.
 */
#ifndef Z2B_DAC_H
#define Z2B_DAC_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct z2b_dac z2b_dac;

/* dac_model's hyper-parameters (src/dac.h:21-24), from the GGUF keys dac.*. */
typedef struct z2b_dac_hparams {
    int32_t n_codebooks, codebook_size, latent_dim, decoder_dim;
    int32_t sample_rate, hop_length, audio_pad_id;
    int32_t n_rates, rates[8];         /* decoder upsampling factors */
    int32_t samples_per_frame;         /* product of the rates */
} z2b_dac_hparams;

/* One stream's window, as dac_decode_window's arguments (src/dac.h:37-45): output frames
 * [f_lo, f_hi) of the raw codes [H][n_codebooks], decoded over the latent frames
 * [max(0, f_lo - Lc), f_hi + Rc) (frames at or past H read as the pad code). */
typedef struct z2b_dac_window {
    const int32_t* codes;
    int32_t H, f_lo, f_hi, Lc, Rc;
} z2b_dac_window;

/* Replaces dac_load (src/dac.h:28-29). */
int z2b_dac_load(const char* path, int device, z2b_dac** out);
/* Replaces dac_free (src/dac.h:30). */
int z2b_dac_free(z2b_dac* dac);
int z2b_dac_get_hparams(const z2b_dac* dac, z2b_dac_hparams* out);

/* Replaces dac_decode (src/dac.h:32-35): raw codes [H][W] -> shear_up -> truncate at eos
 * (eos < 0: all H rows) -> clamp -> decoder -> tanh. Writes min(eos, H) * samples_per_frame
 * samples to audio (capacity cap) and their count to *n_samples. No frames to decode
 * (eos == 0 or H == 0) is an error, as in the reference. */
int z2b_dac_decode(z2b_dac* dac, const int32_t* codes, int H, int W, int eos, float* audio, int64_t cap,
                   int64_t* n_samples);

/* Replaces dac_decode_window (src/dac.h:37-45): the samples of output frames [f_lo, f_hi)
 * (none when f_hi <= f_lo). */
int z2b_dac_decode_window(z2b_dac* dac, const int32_t* codes, int H, int f_lo, int f_hi, int Lc, int Rc,
                          float* audio, int64_t cap, int64_t* n_samples);

/* Batched form: n windows decoded in one pass; audio receives each window's samples in
 * order, n_samples[i] their counts. A window decodes exactly as z2b_dac_decode_window
 * would decode it alone, bit for bit. */
int z2b_dac_decode_windows(z2b_dac* dac, const z2b_dac_window* windows, int n, float* audio, int64_t cap,
                           int64_t* n_samples);

/* Kernels launched by the last decode call. */
long z2b_dac_last_launches(const z2b_dac* dac);

/* The CUDA stream (cudaStream_t) the decoder's kernels and copies run on. */
void* z2b_dac_stream(z2b_dac* dac);

/* Replaces dac_wav_bytes (src/dac.h:47-48): a 16-bit PCM mono RIFF/WAVE image of audio
 * (clamped to [-1, 1], scaled by 32767 and rounded to nearest). Returns the image size
 * (44 + 2 n); writes it to out when cap is large enough. */
int64_t z2b_dac_wav_bytes(const float* audio, int64_t n, int sample_rate, uint8_t* out, int64_t cap);

#ifdef __cplusplus
}
#endif

#endif /* Z2B_DAC_H */
