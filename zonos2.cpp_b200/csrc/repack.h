// repack.h — GGUF block rows <-> device tile layout (see tile_layout.h).
#pragma once

#include <cstdint>

namespace z2b {

// Bytes of the tile image of a [rows][K] matrix of `type`; -1 if unsupported.
int64_t tiles_bytes(uint32_t type, int64_t rows, int64_t K);
// src: `rows` GGUF rows of K weights; dst: tiles_bytes(...) bytes.
bool repack_rows(uint32_t type, int64_t rows, int64_t K, const uint8_t* src, uint8_t* dst);
// Inverse, decoding to f32 with gguf-py's rounding order (bit-exact dequant).
bool unpack_tiles(uint32_t type, int64_t rows, int64_t K, const uint8_t* tiles, float* out);

}  // namespace z2b
