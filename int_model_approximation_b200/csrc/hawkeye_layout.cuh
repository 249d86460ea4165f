// Staged operand layout of the direct Hawkeye replay (written by ima_hawkeye_prepare and
// ima_hawkeye_quantize_prepare, read by ima_hawkeye_replay).  One buffer per operand
// (activations and weights alike), rows padded to `pitch` (a multiple of 128).  The buffer
// is a sequence of blocks, one per (group g of 32 k, tile t of 128 rows), block index
// g * (pitch / 128) + t, HK_BLOCK bytes each, so that one bulk copy moves everything the
// replay needs of one operand for one group:
//
//   +0        rec[k][r]    uint2 { bits(|s| 2^e) (0 when s == 0), sign mask (0 or ~0) },
//                          k < 32, r < 128 (1 KB per k)
//   +32768    pw[r][32]    bf16 exponent powers 2^(8 (e - 8) + 1) of the 32 k (0 when the
//                          element is absent: s == 0 or k >= K), 64 bytes per row with the
//                          16-byte chunks permuted by the 64-byte swizzle (chunk c at
//                          c ^ ((r >> 1) & 3)): a K-major SWIZZLE_64B tensor-core operand
//   +40960    sg[r]        sign bits of the group (bit j = sign of k = 32 g + j)
//
// The replay multiplies the power tiles of A and B on the tensor cores: for one output and
// group the fp32 sum of 2^(8 (ea + eb) - 126) over the present products has exponent field
// 8 max(ea + eb) + 1 + r with 0 <= r <= 5 (at most 32 terms), so the field >> 3 is the
// group's maximum exponent sum exactly.
#pragma once

#include "ima_common.cuh"

constexpr int HK_GROUP = 32;
constexpr int HK_TILE_ROWS = 128;
constexpr int HK_BLK_POW = HK_GROUP * HK_TILE_ROWS * 8;         // 32,768
constexpr int HK_BLK_SG = HK_BLK_POW + HK_TILE_ROWS * 64;       // 40,960
constexpr int HK_BLOCK = HK_BLK_SG + HK_TILE_ROWS * 4;          // 41,472 bytes per (group, tile)

// bf16 bits of 2^(8 (e - 8) + 1), e in 1 .. 15 (an effective e4m3 exponent), or 0.
IMA_DEVINL uint32_t hk_pow_bits(bool present, int e) { return present ? (uint32_t)(8 * e + 64) << 7 : 0u; }

// The block holding row r of group g.
IMA_DEVINL unsigned char* hk_block(unsigned char* base, int64_t g, int64_t r, int64_t pitch) {
    return base + (g * (pitch / HK_TILE_ROWS) + (r / HK_TILE_ROWS)) * (int64_t)HK_BLOCK;
}

// Store everything of one (group, row): its 32 records, its 32 powers (packed two per word,
// k = 2i low, 2i + 1 high) and its sign word.
IMA_DEVINL void hk_store_row(unsigned char* base, int64_t g, int64_t r, int64_t pitch, const uint2 (&rec)[32],
                             const uint32_t (&w)[16], uint32_t signs) {
    unsigned char* blk = hk_block(base, g, r, pitch);
    const uint32_t rl = (uint32_t)(r % HK_TILE_ROWS);
#pragma unroll
    for (int j = 0; j < HK_GROUP; ++j) reinterpret_cast<uint2*>(blk)[j * HK_TILE_ROWS + rl] = rec[j];
    unsigned char* row = blk + HK_BLK_POW + rl * 64;
    const uint32_t sw = (rl >> 1) & 3u;
#pragma unroll
    for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(row + ((c ^ sw) << 4)) = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
    reinterpret_cast<uint32_t*>(blk + HK_BLK_SG)[rl] = signs;
}
