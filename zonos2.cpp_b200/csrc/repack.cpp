// repack.cpp — GGUF rows -> device tile layout (tile_layout.h), and the host-side
// inverse used to check the layout without a GPU.
#include "repack.h"
#include "gguf.h"
#include "quant.h"
#include "tile_layout.h"
#include "../../include/z2b_tools.h"

#include <cstring>
#include <vector>

namespace z2b {

namespace {

inline int q4k_nib(const uint8_t* blk, int n) {            // element n of a Q4_K block
    const int j = n / 32, i = n % 32;
    return (blk[16 + (j / 2) * 32 + i] >> (4 * (j & 1))) & 15;
}
inline int q6k_val(const uint8_t* blk, int n) {             // 6-bit value (before -32)
    const int g = n / 32, i = n % 32;
    const int lo = (blk[(g / 4) * 64 + (g % 2) * 32 + i] >> (4 * ((g % 4) / 2))) & 15;
    const int hi = (blk[128 + (g / 4) * 32 + i] >> (2 * (g % 4))) & 3;
    return lo | (hi << 4);
}
// nibble word for k-steps (s, s+1) given e(s, j) = f(s, j)
template <class F> inline uint32_t nib_word(int s, F f) {
    uint32_t w = 0;
    for (int t = 0; t < 2; ++t) {
        const int sh = 8 * t;
        w |= (uint32_t)(f(s + t, 0) & 15) << (0 + sh);
        w |= (uint32_t)(f(s + t, 1) & 15) << (16 + sh);
        w |= (uint32_t)(f(s + t, 2) & 15) << (4 + sh);
        w |= (uint32_t)(f(s + t, 3) & 15) << (20 + sh);
    }
    return w;
}
template <class F> inline int nib_get(uint32_t w, int t, int j) {  // inverse of nib_word
    static const int pos[4] = {0, 16, 4, 20};
    return (int)((w >> (pos[j] + 8 * t)) & 15);
}

}  // namespace

int64_t tiles_bytes(uint32_t type, int64_t rows, int64_t K) {
    TileGeom g;
    if (!tile_geom(type, K, &g)) return -1;
    return ((rows + TILE_ROWS - 1) / TILE_ROWS) * g.chunks * g.tile_bytes;
}

bool repack_rows(uint32_t type, int64_t rows, int64_t K, const uint8_t* src, uint8_t* dst) {
    TileGeom g;
    if (!tile_geom(type, K, &g)) return false;
    const size_t rb = gtype_row_bytes(type, K);
    const int64_t ntiles = (rows + TILE_ROWS - 1) / TILE_ROWS;
    std::vector<uint8_t> zero(rb, 0);
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < ntiles; ++t) {
        const uint8_t* rowp[16];
        for (int rr = 0; rr < 16; ++rr) {
            const int64_t R = t * 16 + rr;
            rowp[rr] = R < rows ? src + (size_t)R * rb : zero.data();
        }
        for (int64_t c = 0; c < g.chunks; ++c) {
            uint8_t* T = dst + ((size_t)t * g.chunks + c) * g.tile_bytes;
            std::memset(T, 0, g.tile_bytes);
            if (type == GT_Q4_K) {
                for (int rr = 0; rr < 16; ++rr) {
                    const uint8_t* blk = rowp[rr] + c * 144;
                    uint8_t* h = T + rr * 16;
                    std::memcpy(h, blk, 4);                      // d, dmin
                    uint8_t bits[12] = {0};
                    for (int q = 0; q < 4; ++q) {
                        int sc0, m0, sc1, m1;
                        q4k_scale_min(blk + 4, 2 * q, &sc0, &m0);
                        q4k_scale_min(blk + 4, 2 * q + 1, &sc1, &m1);
                        const uint32_t f = (uint32_t)sc0 | ((uint32_t)sc1 << 6) | ((uint32_t)m0 << 12) | ((uint32_t)m1 << 18);
                        for (int b = 0; b < 24; ++b)
                            if (f >> b & 1) { const int p = 24 * q + b; bits[p / 8] |= (uint8_t)(1u << (p % 8)); }
                    }
                    std::memcpy(h + 4, bits, 12);
                }
                for (int u = 0; u < 4; ++u)
                    for (int lane = 0; lane < 32; ++lane) {
                        const int r = lane / 4, q = lane % 4;
                        uint32_t w[4];
                        for (int half = 0; half < 2; ++half) {
                            const uint8_t* blk = rowp[r + 8 * half] + c * 144;
                            auto f = [&](int s, int j) { return q4k_nib(blk, 64 * q + 4 * s + j); };
                            w[2 * half + 0] = nib_word(4 * u, f);
                            w[2 * half + 1] = nib_word(4 * u + 2, f);
                        }
                        std::memcpy(T + Q4K_HDR + (u * 32 + lane) * 16, w, 16);
                    }
            } else if (type == GT_Q6_K) {
                for (int rr = 0; rr < 16; ++rr) {
                    const uint8_t* blk = rowp[rr] + c * 210;
                    std::memcpy(T + rr * 16, blk + 192, 16);          // int8 scales
                    std::memcpy(T + 256 + rr * 2, blk + 208, 2);      // d
                }
                for (int lane = 0; lane < 32; ++lane) {
                    const int r = lane / 4, q = lane % 4;
                    for (int u = 0; u < 4; ++u) {
                        uint32_t w[4];
                        for (int half = 0; half < 2; ++half) {
                            const uint8_t* blk = rowp[r + 8 * half] + c * 210;
                            auto f = [&](int s, int j) { return q6k_val(blk, 64 * q + 4 * s + j) & 15; };
                            w[2 * half + 0] = nib_word(4 * u, f);
                            w[2 * half + 1] = nib_word(4 * u + 2, f);
                        }
                        std::memcpy(T + Q6K_HDR + (u * 32 + lane) * 16, w, 16);
                    }
                    for (int gg = 0; gg < 2; ++gg) {
                        uint32_t w[4];
                        for (int half = 0; half < 2; ++half) {
                            const uint8_t* blk = rowp[r + 8 * half] + c * 210;
                            for (int gi = 0; gi < 2; ++gi) {
                                const int G = 2 * gg + gi;
                                uint32_t hw = 0;
                                for (int j = 0; j < 4; ++j) {
                                    const int s = 4 * G + j, k0 = 64 * q + 4 * s;
                                    hw |= (uint32_t)(q6k_val(blk, k0 + 0) >> 4) << (4 * j);
                                    hw |= (uint32_t)(q6k_val(blk, k0 + 2) >> 4) << (4 * j + 2);
                                    hw |= (uint32_t)(q6k_val(blk, k0 + 1) >> 4) << (16 + 4 * j);
                                    hw |= (uint32_t)(q6k_val(blk, k0 + 3) >> 4) << (16 + 4 * j + 2);
                                }
                                w[2 * half + gi] = hw;
                            }
                        }
                        std::memcpy(T + Q6K_HDR + Q6K_LO + (gg * 32 + lane) * 16, w, 16);
                    }
                }
            } else if (type == GT_Q8_0) {
                for (int rr = 0; rr < 16; ++rr)
                    for (int q = 0; q < 4; ++q)
                        std::memcpy(T + (rr * 4 + q) * 2, rowp[rr] + (c * 4 + q) * 34, 2);
                for (int u = 0; u < 4; ++u)
                    for (int lane = 0; lane < 32; ++lane) {
                        const int r = lane / 4, q = lane % 4;
                        uint8_t b[16];
                        for (int half = 0; half < 2; ++half) {
                            const uint8_t* blk = rowp[r + 8 * half] + (c * 4 + q) * 34;
                            for (int t2 = 0; t2 < 2; ++t2) {
                                const int s = 2 * u + t2;
                                for (int j = 0; j < 4; ++j)
                                    b[half * 8 + t2 * 4 + j] = (uint8_t)(blk[2 + 4 * s + j] ^ 0x80u);
                            }
                        }
                        std::memcpy(T + Q80_HDR + (u * 32 + lane) * 16, b, 16);
                    }
            } else if (type == GT_F16) {
                const int S = g.steps;
                for (int s = 0; s < S; ++s)
                    for (int lane = 0; lane < 32; ++lane) {
                        const int r = lane / 4, q = lane % 4;
                        uint16_t v[8];
                        for (int half = 0; half < 2; ++half) {
                            const uint16_t* row = (const uint16_t*)rowp[r + 8 * half];
                            for (int j = 0; j < 4; ++j) v[half * 4 + j] = row[c * g.kc + 4 * S * q + 4 * s + j];
                        }
                        std::memcpy(T + (s * 32 + lane) * 16, v, 16);
                    }
            }
        }
    }
    return true;
}

bool unpack_tiles(uint32_t type, int64_t rows, int64_t K, const uint8_t* tiles, float* out) {
    TileGeom g;
    if (!tile_geom(type, K, &g)) return false;
    const int64_t ntiles = (rows + TILE_ROWS - 1) / TILE_ROWS;
    for (int64_t t = 0; t < ntiles; ++t)
        for (int64_t c = 0; c < g.chunks; ++c) {
            const uint8_t* T = tiles + ((size_t)t * g.chunks + c) * g.tile_bytes;
            for (int lane = 0; lane < 32; ++lane) {
                const int r = lane / 4, q = lane % 4;
                for (int half = 0; half < 2; ++half) {
                    const int rr = r + 8 * half;
                    const int64_t R = t * 16 + rr;
                    if (R >= rows) continue;
                    float* orow = out + (size_t)R * K + c * g.kc;
                    if (type == GT_Q4_K) {
                        uint16_t dh, mh; std::memcpy(&dh, T + rr * 16, 2); std::memcpy(&mh, T + rr * 16 + 2, 2);
                        uint8_t bits[12]; std::memcpy(bits, T + rr * 16 + 4, 12);
                        uint32_t f = 0;
                        for (int b = 0; b < 24; ++b) { const int p = 24 * q + b; f |= (uint32_t)((bits[p / 8] >> (p % 8)) & 1) << b; }
                        const int sc[2] = {(int)(f & 63), (int)((f >> 6) & 63)}, mm[2] = {(int)((f >> 12) & 63), (int)((f >> 18) & 63)};
                        const float d = f16_to_f32(dh), dmin = f16_to_f32(mh);
                        for (int u = 0; u < 4; ++u) {
                            uint32_t w[4]; std::memcpy(w, T + Q4K_HDR + (u * 32 + lane) * 16, 16);
                            for (int wi = 0; wi < 2; ++wi)
                                for (int t2 = 0; t2 < 2; ++t2)
                                    for (int j = 0; j < 4; ++j) {
                                        const int s = 4 * u + 2 * wi + t2;
                                        const int e = nib_get<int>(w[2 * half + wi], t2, j);
                                        const int sb = s / 8;              // sub-block 2q + sb
                                        const float ds = d * (float)sc[sb], dm = dmin * (float)mm[sb];
                                        const float p = ds * (float)e;
                                        orow[64 * q + 4 * s + j] = p - dm;
                                    }
                        }
                    } else if (type == GT_Q6_K) {
                        int8_t sc[16]; std::memcpy(sc, T + rr * 16, 16);
                        uint16_t dh; std::memcpy(&dh, T + 256 + rr * 2, 2);
                        const float d = f16_to_f32(dh);
                        for (int s = 0; s < 16; ++s) {
                            uint32_t w[4]; std::memcpy(w, T + Q6K_HDR + ((s / 4) * 32 + lane) * 16, 16);
                            const uint32_t nw = w[2 * half + (s % 4) / 2];
                            uint32_t hv[4]; std::memcpy(hv, T + Q6K_HDR + Q6K_LO + ((s / 8) * 32 + lane) * 16, 16);
                            const uint32_t hw = hv[2 * half + (s / 4) % 2];
                            const int j4 = s % 4;
                            for (int j = 0; j < 4; ++j) {
                                const int lo = nib_get<int>(nw, s % 2, j);
                                static const int hpos[4] = {0, 16, 2, 18};
                                const int hi = (int)((hw >> (hpos[j] + 4 * j4)) & 3);
                                const int k = 64 * q + 4 * s + j;
                                const float ds = d * (float)sc[k / 16];
                                orow[k] = ds * (float)((lo | (hi << 4)) - 32);
                            }
                        }
                    } else if (type == GT_Q8_0) {
                        uint16_t dh; std::memcpy(&dh, T + (rr * 4 + q) * 2, 2);
                        const float d = f16_to_f32(dh);
                        for (int u = 0; u < 4; ++u) {
                            uint8_t b[16]; std::memcpy(b, T + Q80_HDR + (u * 32 + lane) * 16, 16);
                            for (int t2 = 0; t2 < 2; ++t2)
                                for (int j = 0; j < 4; ++j) {
                                    const int s = 2 * u + t2;
                                    orow[32 * q + 4 * s + j] = (float)((int)b[half * 8 + t2 * 4 + j] - 128) * d;
                                }
                        }
                    } else if (type == GT_F16) {
                        const int S = g.steps;
                        for (int s = 0; s < S; ++s) {
                            uint16_t v[8]; std::memcpy(v, T + (s * 32 + lane) * 16, 16);
                            for (int j = 0; j < 4; ++j) orow[4 * S * q + 4 * s + j] = f16_to_f32(v[half * 4 + j]);
                        }
                    }
                }
            }
        }
    return true;
}

}  // namespace z2b

extern "C" int64_t z2b_host_tiles_bytes(uint32_t type, int64_t rows, int64_t k) {
    return z2b::tiles_bytes(type, rows, k);
}
extern "C" int z2b_host_repack(uint32_t type, int64_t rows, int64_t k, const void* src, void* dst) {
    return z2b::repack_rows(type, rows, k, (const uint8_t*)src, (uint8_t*)dst) ? 0 : 1;
}
extern "C" int z2b_host_unpack_tiles(uint32_t type, int64_t rows, int64_t k, const void* tiles, float* out) {
    return z2b::unpack_tiles(type, rows, k, (const uint8_t*)tiles, out) ? 0 : 1;
}
