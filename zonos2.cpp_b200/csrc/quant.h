// quant.h — host-side GGUF block encoders/decoders for the synthetic model writer,
// the load-time repack and the CPU-side layout checks.
//
// Block formats (third-party gguf-py 0.19.0, gguf/quants.py; ggml-quants.c):
//   Q8_0: 32 weights  = f16 d, int8 qs[32]                          w = qs*d
//   Q4_K: 256 weights = f16 d, f16 dmin, u8 scales[12], u8 qs[128]  w = (d*sc)*q - (dmin*m)
//   Q6_K: 256 weights = u8 ql[128], u8 qh[64], i8 scales[16], f16 d w = (d*sc)*(q-32)
#pragma once

#include <cstddef>
#include <cstdint>

namespace z2b {

// Q8_0 encoder, bit-exact with gguf-py Q8_0.quantize_blocks (quants.py:382-394):
// d = amax/127 in f32, q = round-half-away(x * (1/d)), d stored as f16.
void quantize_row_q8_0(const float* x, uint8_t* out, int64_t n);
// Q4_K / Q6_K encoders (round-to-nearest with per-sub-block scale search kept simple).
// Any valid block encoding is acceptable: parity is defined on the decoded values.
void quantize_row_q4_k(const float* x, uint8_t* out, int64_t n);
void quantize_row_q6_k(const float* x, uint8_t* out, int64_t n);
void quantize_row_f16(const float* x, uint8_t* out, int64_t n);
// Encodes n values of `type` (GType); returns false for unsupported types.
bool quantize_row(uint32_t type, const float* x, uint8_t* out, int64_t n);

// Decoders with the gguf-py rounding order (product rounded to f32, then the
// subtraction): bit-exact with gguf.quants.dequantize.
void dequant_row(uint32_t type, const uint8_t* in, float* out, int64_t n);

// Q4_K 6-bit scale/min unpack for sub-block j (gguf-py Q4_K.get_scale_min).
inline void q4k_scale_min(const uint8_t* s, int j, int* sc, int* m) {
    if (j < 4) { *sc = s[j] & 63; *m = s[j + 4] & 63; }
    else {
        *sc = (s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4);
        *m  = (s[j + 4] >> 4)   | ((s[j] >> 6) << 4);
    }
}

}  // namespace z2b
