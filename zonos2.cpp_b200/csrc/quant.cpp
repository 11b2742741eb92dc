// quant.cpp — host-side block encoders/decoders (see quant.h).
// Compiled with -ffp-contract=off so a*b-c never fuses: the decoders must round
// exactly like numpy does in gguf-py.
#include "quant.h"
#include "gguf.h"

#include <algorithm>
#include <cmath>
#include <cstring>

namespace z2b {

static inline float round_half_away(float v) { return std::round(v); }

void quantize_row_q8_0(const float* x, uint8_t* out, int64_t n) {
    for (int64_t b = 0; b < n / 32; ++b) {
        const float* xb = x + b * 32;
        uint8_t* o = out + b * 34;
        float amax = 0.0f;
        for (int i = 0; i < 32; ++i) amax = std::max(amax, std::fabs(xb[i]));
        const float d = amax / 127.0f;
        const float id = d == 0.0f ? 0.0f : 1.0f / d;
        const uint16_t dh = f32_to_f16(d);
        std::memcpy(o, &dh, 2);
        for (int i = 0; i < 32; ++i) {
            const float q = round_half_away(xb[i] * id);
            o[2 + i] = (uint8_t)(int8_t)q;
        }
    }
}

void quantize_row_q4_k(const float* x, uint8_t* out, int64_t n) {
    for (int64_t b = 0; b < n / 256; ++b) {
        const float* xb = x + b * 256;
        uint8_t* o = out + b * 144;
        float scale[8], mins[8];
        for (int j = 0; j < 8; ++j) {
            float mn = 0.0f, mx = -INFINITY;
            for (int i = 0; i < 32; ++i) { mn = std::min(mn, xb[j * 32 + i]); mx = std::max(mx, xb[j * 32 + i]); }
            scale[j] = (mx - mn) / 15.0f;
            mins[j] = -mn;
        }
        float smax = 0.0f, mmax = 0.0f;
        for (int j = 0; j < 8; ++j) { smax = std::max(smax, scale[j]); mmax = std::max(mmax, mins[j]); }
        const uint16_t dh = f32_to_f16(smax / 63.0f), dmh = f32_to_f16(mmax / 63.0f);
        const float d = f16_to_f32(dh), dmin = f16_to_f32(dmh);
        int sc[8], mq[8];
        for (int j = 0; j < 8; ++j) {
            sc[j] = d > 0.0f ? std::min(63, std::max(0, (int)std::lround(scale[j] / d))) : 0;
            mq[j] = dmin > 0.0f ? std::min(63, std::max(0, (int)std::lround(mins[j] / dmin))) : 0;
        }
        std::memcpy(o, &dh, 2);
        std::memcpy(o + 2, &dmh, 2);
        uint8_t* s = o + 4;
        for (int j = 0; j < 4; ++j) {
            s[j]     = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
            s[j + 4] = (uint8_t)((mq[j] & 63) | ((mq[j + 4] >> 4) << 6));
            s[j + 8] = (uint8_t)((sc[j + 4] & 15) | ((mq[j + 4] & 15) << 4));
        }
        uint8_t* qs = o + 16;
        std::memset(qs, 0, 128);
        for (int j = 0; j < 8; ++j) {
            const float ds = d * (float)sc[j], dm = dmin * (float)mq[j];
            for (int i = 0; i < 32; ++i) {
                int q = 0;
                if (ds > 0.0f) q = std::min(15, std::max(0, (int)std::lround((xb[j * 32 + i] + dm) / ds)));
                // sub-block j lives in byte group j/2, low nibble for even j, high for odd j
                qs[(j / 2) * 32 + i] |= (uint8_t)(q << (4 * (j & 1)));
            }
        }
    }
}

void quantize_row_q6_k(const float* x, uint8_t* out, int64_t n) {
    for (int64_t b = 0; b < n / 256; ++b) {
        const float* xb = x + b * 256;
        uint8_t* o = out + b * 210;
        float sub[16];
        for (int j = 0; j < 16; ++j) {
            float amax = 0.0f;
            for (int i = 0; i < 16; ++i) amax = std::max(amax, std::fabs(xb[j * 16 + i]));
            sub[j] = amax / 31.0f;
        }
        float smax = 0.0f;
        for (int j = 0; j < 16; ++j) smax = std::max(smax, sub[j]);
        const uint16_t dh = f32_to_f16(smax / 127.0f);
        const float d = f16_to_f32(dh);
        int8_t sc[16];
        for (int j = 0; j < 16; ++j) sc[j] = (int8_t)(d > 0.0f ? std::min(127, std::max(-128, (int)std::lround(sub[j] / d))) : 0);
        uint8_t* ql = o;
        uint8_t* qh = o + 128;
        std::memset(ql, 0, 128);
        std::memset(qh, 0, 64);
        for (int e = 0; e < 256; ++e) {
            const float ds = d * (float)sc[e / 16];
            int q = 32;
            if (ds > 0.0f) q = std::min(63, std::max(0, (int)std::lround(xb[e] / ds) + 32));
            const int g = e / 32, i = e % 32;
            ql[(g / 4) * 64 + (g % 2) * 32 + i] |= (uint8_t)((q & 15) << (4 * ((g % 4) / 2)));
            qh[(g / 4) * 32 + i] |= (uint8_t)((q >> 4) << (2 * (g % 4)));
        }
        std::memcpy(o + 192, sc, 16);
        std::memcpy(o + 208, &dh, 2);
    }
}

void quantize_row_f16(const float* x, uint8_t* out, int64_t n) {
    uint16_t* o = (uint16_t*)out;
    for (int64_t i = 0; i < n; ++i) o[i] = f32_to_f16(x[i]);
}

bool quantize_row(uint32_t type, const float* x, uint8_t* out, int64_t n) {
    switch (type) {
        case GT_F32: std::memcpy(out, x, (size_t)n * 4); return true;
        case GT_F16: quantize_row_f16(x, out, n); return true;
        case GT_Q8_0: quantize_row_q8_0(x, out, n); return true;
        case GT_Q4_K: quantize_row_q4_k(x, out, n); return true;
        case GT_Q6_K: quantize_row_q6_k(x, out, n); return true;
        default: return false;
    }
}

void dequant_row(uint32_t type, const uint8_t* in, float* out, int64_t n) {
    switch (type) {
        case GT_F32: std::memcpy(out, in, (size_t)n * 4); break;
        case GT_F16: for (int64_t i = 0; i < n; ++i) { uint16_t h; std::memcpy(&h, in + 2 * i, 2); out[i] = f16_to_f32(h); } break;
        case GT_BF16: for (int64_t i = 0; i < n; ++i) { uint16_t h; std::memcpy(&h, in + 2 * i, 2); uint32_t u = (uint32_t)h << 16; std::memcpy(out + i, &u, 4); } break;
        case GT_Q8_0:
            for (int64_t b = 0; b < n / 32; ++b) {
                uint16_t dh; std::memcpy(&dh, in + b * 34, 2);
                const float d = f16_to_f32(dh);
                for (int i = 0; i < 32; ++i) out[b * 32 + i] = (float)(int8_t)in[b * 34 + 2 + i] * d;
            }
            break;
        case GT_Q4_K:
            for (int64_t b = 0; b < n / 256; ++b) {
                const uint8_t* blk = in + b * 144;
                uint16_t dh, mh; std::memcpy(&dh, blk, 2); std::memcpy(&mh, blk + 2, 2);
                const float d = f16_to_f32(dh), dmin = f16_to_f32(mh);
                for (int j = 0; j < 8; ++j) {
                    int sc, m; q4k_scale_min(blk + 4, j, &sc, &m);
                    const float ds = d * (float)sc, dm = dmin * (float)m;
                    for (int i = 0; i < 32; ++i) {
                        const int q = (blk[16 + (j / 2) * 32 + i] >> (4 * (j & 1))) & 15;
                        const float p = ds * (float)q;
                        out[b * 256 + j * 32 + i] = p - dm;
                    }
                }
            }
            break;
        case GT_Q6_K:
            for (int64_t b = 0; b < n / 256; ++b) {
                const uint8_t* blk = in + b * 210;
                uint16_t dh; std::memcpy(&dh, blk + 208, 2);
                const float d = f16_to_f32(dh);
                for (int e = 0; e < 256; ++e) {
                    const int g = e / 32, i = e % 32;
                    const int lo = (blk[(g / 4) * 64 + (g % 2) * 32 + i] >> (4 * ((g % 4) / 2))) & 15;
                    const int hi = (blk[128 + (g / 4) * 32 + i] >> (2 * (g % 4))) & 3;
                    const float ds = d * (float)(int8_t)blk[192 + e / 16];
                    out[b * 256 + e] = ds * (float)((lo | (hi << 4)) - 32);
                }
            }
            break;
        default: break;
    }
}

}  // namespace z2b
