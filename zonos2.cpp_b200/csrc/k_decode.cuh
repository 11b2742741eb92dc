// k_decode.cuh — in-register decoders of the weight tile layout (tile_layout.h): each
// builds the mma.sync m16n8k16 A fragment of one k-step of a 16-row tile, with the
// weight values rounded once to f16. Shared by the tile GEMV and the tcgen05 GEMM.
#pragma once

#include "common.cuh"
#include "gguf.h"
#include "tile_layout.h"

namespace z2b {

constexpr int MAXKS = 16;    // k-steps per warp per item (register budget for B)

__device__ __forceinline__ __half2 hc(uint16_t bits) { return __half2half2(__ushort_as_half(bits)); }

template <int N> __device__ __forceinline__ uint32_t shr_signed(uint32_t x) {
    if constexpr (N >= 0) return x >> N; else return x << (-N);
}

// ---- per-type decoders: prep() reads the chunk's scales, frag() builds A for k-step S ----
template <int WT> struct Dec;

// Q4_K: w = (d*sc)*q - dmin*m, decoded per pair as hfma2(q, S, -M) with q recovered
// exactly from the magic-number extraction (1024 + q, or 1024 + 16 q for the high
// nibbles). Rounding the centred value q*S - M once keeps the weight error relative to
// the weight itself (rounding q*S alone and subtracting the min later doubles it).
template <> struct Dec<GT_Q4_K> {
    static constexpr int KS = 16, KC = 256;
    __half2 S[2][2], M[2][2];                 // [sub-block 0/1][row r / r+8], M holds -min
    // Scales without the conversion pipe: the 6-bit fields become exact halves through
    // the 0x6400 exponent (1024 + v, minus 1024), and d * sc (exact in f32, 17 bits) is
    // rounded once by the half multiply, the same value __float2half_rn(d * sc) gives.
    __device__ __forceinline__ void prep(const uint8_t* T, int lane) {
        const int r = lane >> 2, q = lane & 3;
        const __half2 k1024 = hc(0x6400);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint4 hd = *(const uint4*)(T + (r + 8 * h) * 16);
            const __half2 dd = u2h(prmt(hd.x, 0u, 0x1010u));          // (d, d)
            const __half2 nm = u2h(prmt(hd.x, 0u, 0x3232u) ^ 0x80008000u);   // (-dmin, -dmin)
            // quad q's 24 bits start at bit 24q of (y, z, w): selects, no divergent branch
            const uint32_t lo = q < 2 ? hd.y : (q == 2 ? hd.z : hd.w);
            const uint32_t hi = q < 2 ? hd.z : (q == 2 ? hd.w : 0u);
            const uint32_t f = __funnelshift_r(lo, hi, (32 - 8 * q) & 31);
            // (sc0, sc1) and (m0, m1) as 1024 + v halves
            const uint32_t sc = lop3_and_or(f, 0x3Fu, lop3_and_or(f << 10, 0x003F0000u, 0x64006400u));
            const uint32_t mn = lop3_and_or(f >> 12, 0x3Fu, lop3_and_or(f >> 2, 0x003F0000u, 0x64006400u));
            const __half2 s01 = __hmul2(__hsub2(u2h(sc), k1024), dd);
            const __half2 m01 = __hmul2(__hsub2(u2h(mn), k1024), nm);
            S[0][h] = u2h(prmt(h2u(s01), 0u, 0x1010u));
            S[1][h] = u2h(prmt(h2u(s01), 0u, 0x3232u));
            M[0][h] = u2h(prmt(h2u(m01), 0u, 0x1010u));
            M[1][h] = u2h(prmt(h2u(m01), 0u, 0x3232u));
        }
    }
    template <int s> __device__ __forceinline__ void frag(const uint8_t* T, int lane, uint32_t a[4]) const {
        const uint4 w = *(const uint4*)(T + Q4K_HDR + ((s >> 2) * 32 + lane) * 16);
        uint32_t v0 = (s & 2) ? w.y : w.x, v1 = (s & 2) ? w.w : w.z;
        if (s & 1) { v0 >>= 8; v1 >>= 8; }
        constexpr int sb = s >> 3;
        const __half2 k1024 = hc(0x6400), k16 = hc(0x2C00), km64 = hc(0xD400);
        a[0] = h2u(__hfma2(__hsub2(u2h(lop3_and_or(v0, 0x000F000Fu, 0x64006400u)), k1024), S[sb][0], M[sb][0]));
        a[1] = h2u(__hfma2(__hsub2(u2h(lop3_and_or(v1, 0x000F000Fu, 0x64006400u)), k1024), S[sb][1], M[sb][1]));
        a[2] = h2u(__hfma2(__hfma2(u2h(lop3_and_or(v0, 0x00F000F0u, 0x64006400u)), k16, km64), S[sb][0], M[sb][0]));
        a[3] = h2u(__hfma2(__hfma2(u2h(lop3_and_or(v1, 0x00F000F0u, 0x64006400u)), k16, km64), S[sb][1], M[sb][1]));
    }
};

template <> struct Dec<GT_Q6_K> {
    static constexpr int KS = 16, KC = 256;
    __half2 S[4][2];
    // int8 scales as exact halves (1152 + sc - 1152 via the 0x6400 exponent: the byte is
    // biased by 128), times d rounded once by the half multiply (d * sc is exact in f32).
    __device__ __forceinline__ void prep(const uint8_t* T, int lane) {
        const int r = lane >> 2, q = lane & 3;
        const __half2 k1152 = hc(0x6480);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t sc = *(const uint32_t*)(T + (r + 8 * h) * 16 + 4 * q) ^ 0x80808080u;   // sc + 128
            const uint16_t dbits = *(const uint16_t*)(T + 256 + 2 * (r + 8 * h));
            const __half2 dd = u2h((uint32_t)dbits * 0x10001u);
            const __half2 s01 = __hmul2(__hsub2(u2h(prmt(sc, 0x64646464u, 0x4140u)), k1152), dd);   // bytes 0, 1
            const __half2 s23 = __hmul2(__hsub2(u2h(prmt(sc, 0x64646464u, 0x4342u)), k1152), dd);   // bytes 2, 3
            S[0][h] = u2h(prmt(h2u(s01), 0u, 0x1010u));
            S[1][h] = u2h(prmt(h2u(s01), 0u, 0x3232u));
            S[2][h] = u2h(prmt(h2u(s23), 0u, 0x1010u));
            S[3][h] = u2h(prmt(h2u(s23), 0u, 0x3232u));
        }
    }
    template <int s> __device__ __forceinline__ void frag(const uint8_t* T, int lane, uint32_t a[4]) const {
        const uint4 w = *(const uint4*)(T + Q6K_HDR + ((s >> 2) * 32 + lane) * 16);
        const uint4 hv = *(const uint4*)(T + Q6K_HDR + Q6K_LO + ((s >> 3) * 32 + lane) * 16);
        uint32_t v0 = (s & 2) ? w.y : w.x, v1 = (s & 2) ? w.w : w.z;
        if (s & 1) { v0 >>= 8; v1 >>= 8; }
        const uint32_t h0 = ((s >> 2) & 1) ? hv.y : hv.x, h1 = ((s >> 2) & 1) ? hv.w : hv.z;
        constexpr int j4 = s & 3, j = s >> 2;
        const __half2 k1056 = hc(0x6420), k16 = hc(0x2C00), km96 = hc(0xD600);
        const uint32_t x0 = lop3_and_or(shr_signed<4 * j4 - 4>(h0), 0x00300030u, lop3_and_or(v0, 0x000F000Fu, 0x64006400u));
        const uint32_t x1 = lop3_and_or(shr_signed<4 * j4 - 4>(h1), 0x00300030u, lop3_and_or(v1, 0x000F000Fu, 0x64006400u));
        const uint32_t y0 = lop3_and_or(shr_signed<4 * j4 - 6>(h0), 0x03000300u, lop3_and_or(v0, 0x00F000F0u, 0x64006400u));
        const uint32_t y1 = lop3_and_or(shr_signed<4 * j4 - 6>(h1), 0x03000300u, lop3_and_or(v1, 0x00F000F0u, 0x64006400u));
        a[0] = h2u(__hmul2(__hsub2(u2h(x0), k1056), S[j][0]));
        a[1] = h2u(__hmul2(__hsub2(u2h(x1), k1056), S[j][1]));
        a[2] = h2u(__hmul2(__hfma2(u2h(y0), k16, km96), S[j][0]));
        a[3] = h2u(__hmul2(__hfma2(u2h(y1), k16, km96), S[j][1]));
    }
};

template <> struct Dec<GT_Q8_0> {
    static constexpr int KS = 8, KC = 128;
    __half2 D[2];
    __device__ __forceinline__ void prep(const uint8_t* T, int lane) {
        const int r = lane >> 2, q = lane & 3;
        D[0] = __half2half2(*(const __half*)(T + (r * 4 + q) * 2));
        D[1] = __half2half2(*(const __half*)(T + ((r + 8) * 4 + q) * 2));
    }
    template <int s> __device__ __forceinline__ void frag(const uint8_t* T, int lane, uint32_t a[4]) const {
        const uint4 w = *(const uint4*)(T + Q80_HDR + ((s >> 1) * 32 + lane) * 16);
        const uint32_t v0 = (s & 1) ? w.y : w.x, v1 = (s & 1) ? w.w : w.z;
        const __half2 k1152 = hc(0x6480);
        a[0] = h2u(__hmul2(__hsub2(u2h(prmt(v0, 0x64646464u, 0x4140u)), k1152), D[0]));
        a[1] = h2u(__hmul2(__hsub2(u2h(prmt(v1, 0x64646464u, 0x4140u)), k1152), D[1]));
        a[2] = h2u(__hmul2(__hsub2(u2h(prmt(v0, 0x64646464u, 0x4342u)), k1152), D[0]));
        a[3] = h2u(__hmul2(__hsub2(u2h(prmt(v1, 0x64646464u, 0x4342u)), k1152), D[1]));
    }
};

// F16 with KS k-steps per chunk (KS = 4, 2, 1)
template <int KS_> struct DecF16 {
    static constexpr int KS = KS_, KC = 16 * KS_;
    __device__ __forceinline__ void prep(const uint8_t*, int) {}
    template <int s> __device__ __forceinline__ void frag(const uint8_t* T, int lane, uint32_t a[4]) const {
        const uint4 w = *(const uint4*)(T + (s * 32 + lane) * 16);
        a[0] = w.x; a[1] = w.z; a[2] = w.y; a[3] = w.w;
    }
};

template <int WT, int KSF> struct DecSel { using T = Dec<WT>; };
template <int KSF> struct DecSel<GT_F16, KSF> { using T = DecF16<KSF>; };


}  // namespace z2b
