// tile_layout.h — device weight layout shared by the host repack and the kernels.
//
// A weight matrix W[N rows][K] (ggml ne = {K, N}) is stored as row-tiles of 16 rows;
// each row-tile is a run of k-chunks, each chunk a self-contained "tile" holding every
// byte needed to multiply those 16 rows over KC consecutive k. Tiles are stored
// [row_tile][chunk], so one row-tile's K-range is contiguous and a warp can pull any
// run of chunks with one bulk copy. The byte count equals the GGUF block bytes of the
// same weights (only rows padded up to a multiple of 16 add bytes).
//
// Inside a tile every byte sits where one lane of a warp needs it as an operand of
// mma.sync.m16n8k16 (A = weights, row-major 16x16 per k-step). Lane l = 4*r + q holds
// rows r and r+8; the mma k-index is permuted so that lane-quad q owns the contiguous
// physical k-range [q*KC/4, (q+1)*KC/4) of the chunk. With that permutation the
// activation operand B is read with one 8-byte load per k-step from a plain row-major
// [token][K] f16 buffer: lane (token n = l/4, quad q) at k-step s reads k = 64q+4s..+3
// (Q4_K/Q6_K), 32q+4s.. (Q8_0) or 4Sq+4s.. (F16), and the weight words below decode
// into exactly the matching A registers:
//   a0 = (row r,   k+0,k+1)  a1 = (row r+8, k+0,k+1)
//   a2 = (row r,   k+2,k+3)  a3 = (row r+8, k+2,k+3)
//
// Nibble word (Q4_K, and the low 4 bits of Q6_K): one u32 covers k-steps s, s+1 of one
// row for one lane; with e(s,j) the value at k = base+4s+j:
//   bits 0-3 e(s,0)   16-19 e(s,1)   4-7 e(s,2)   20-23 e(s,3)
//   bits 8-11 e(s+1,0) 24-27 e(s+1,1) 12-15 e(s+1,2) 28-31 e(s+1,3)
// so (w & 0x000F000F) | 0x64006400 is the half2 (1024+e0, 1024+e1), (w & 0x00F000F0) |
// 0x64006400 is (1024+16e2, 1024+16e3), and w>>8 exposes k-step s+1 the same way.
#pragma once

#include <cstdint>

namespace z2b {

constexpr int TILE_ROWS = 16;

// ---- Q4_K: KC = 256 (16 k-steps), lane quad q covers sub-blocks 2q, 2q+1 ----
// header [16 rows][16 B]: f16 d, f16 dmin, then 96 bits of 6-bit fields where quad q's
//        24 bits start at bit 24q: sc[2q], sc[2q+1], m[2q], m[2q+1] (6 bits each);
// body   [u=0..3][lane][16 B] = {row r word(4u,4u+1), row r word(4u+2,4u+3),
//                                 row r+8 word(4u,4u+1), row r+8 word(4u+2,4u+3)}.
constexpr int Q4K_KC = 256, Q4K_TILE = 2304, Q4K_HDR = 256;

// ---- Q6_K: KC = 256, lane quad q covers 16-element sub-blocks 4q..4q+3 ----
// header scales [16 rows][16 x int8] (GGUF order), then d [16 rows] f16  (288 B);
// low nibbles as Q4_K body (2048 B);
// high bits [g=0..1][lane][16 B] = {row r hw(2g), row r hw(2g+1), row r+8 hw(2g), row r+8 hw(2g+1)}
//   hw(G) covers k-steps s = 4G+j (j=0..3): hi(s,0) at bits 4j, hi(s,2) at 4j+2,
//   hi(s,1) at 16+4j, hi(s,3) at 16+4j+2 (2 bits each).
constexpr int Q6K_KC = 256, Q6K_TILE = 3360, Q6K_HDR = 288, Q6K_LO = 2048;

// ---- Q8_0: KC = 128 (8 k-steps), lane quad q covers GGUF block (4*chunk + q) ----
// header d [16 rows][4] f16 (128 B); body [u=0..3][lane][16 B] =
//   {row r w(2u), row r w(2u+1), row r+8 w(2u), row r+8 w(2u+1)}, w(s) = 4 bytes
//   (q+128) for k = 32q+4s+0..3.
constexpr int Q80_KC = 128, Q80_TILE = 2176, Q80_HDR = 128;

// ---- F16: KC = 16*S (S = 4, 2 or 1 k-steps, the largest dividing K) ----
// body [s][lane][16 B] = {row r (k0,k1), row r (k2,k3), row r+8 (k0,k1), row r+8 (k2,k3)}
//   with k = 4S*q + 4s + j.
inline int f16_steps(int64_t K) { return (K % 64 == 0) ? 4 : (K % 32 == 0) ? 2 : 1; }

// Tile geometry for a type/K pair; returns false if the shape is not supported.
struct TileGeom { int kc; int tile_bytes; int steps; int64_t chunks; };
inline bool tile_geom(uint32_t type, int64_t K, TileGeom* g) {
    switch (type) {
        case 12: if (K % 256) return false; *g = {Q4K_KC, Q4K_TILE, 16, K / 256}; return true;
        case 14: if (K % 256) return false; *g = {Q6K_KC, Q6K_TILE, 16, K / 256}; return true;
        case 8:  if (K % 128) return false; *g = {Q80_KC, Q80_TILE, 8, K / 128}; return true;
        case 1: {
            if (K % 16) return false;
            const int s = f16_steps(K);
            *g = {16 * s, 512 * s, s, K / (16 * s)};
            return true;
        }
        default: return false;
    }
}

}  // namespace z2b
