// Staged operand layout of the direct Hawkeye replay (written by ima_hawkeye_prepare and
// ima_hawkeye_quantize_prepare, read by ima_hawkeye_replay).  One buffer per operand
// (activations and weights alike), rows padded to `pitch` (a multiple of 128):
//
//   rec[k][r]        uint2 { bits(|s| 2^e) (0 when s == 0), sign mask (0 or ~0) }
//   pw[g][r][32]     bf16 exponent powers 2^(8 (e - 8) + 1) of the 32 k of group g
//                    (0 when the element is absent: s == 0 or k >= K), 64 bytes per
//                    (group, row) with the 16-byte chunks permuted by the 64-byte swizzle
//                    (chunk c at c ^ ((r >> 1) & 3)), so that one 8 KB bulk copy of 128 rows
//                    is a K-major SWIZZLE_64B tensor-core operand
//   sg[g][r]         sign bits of group g (bit j = sign of k = 32 g + j)
//
// The replay multiplies the power tiles of A and B on the tensor cores: for one output and
// group the fp32 sum of 2^(8 (ea + eb) - 126) over the present products has exponent field
// 8 max(ea + eb) + 1 + r with 0 <= r <= 5 (at most 32 terms), so the field >> 3 is the
// group's maximum exponent sum exactly.
#pragma once

#include "ima_common.cuh"

constexpr int HK_GROUP = 32;

// bf16 bits of 2^(8 (e - 8) + 1), e in 1 .. 15 (an effective e4m3 exponent), or 0.
IMA_DEVINL uint32_t hk_pow_bits(bool present, int e) { return present ? (uint32_t)(8 * e + 64) << 7 : 0u; }

// Byte offset of (group g, row r) in the power array; chunk c of the row lies at
// hk_pow_row(g, r, pitch) + ((c ^ ((r >> 1) & 3)) << 4).
IMA_DEVINL int64_t hk_pow_row(int64_t g, int64_t r, int64_t pitch) { return (g * pitch + r) * 64; }

// Store the 32 powers of one (group, row), packed two per word (k = 2i low, 2i + 1 high).
IMA_DEVINL void hk_store_pow(unsigned char* pw, int64_t g, int64_t r, int64_t pitch, const uint32_t (&w)[16]) {
    unsigned char* row = pw + hk_pow_row(g, r, pitch);
    const uint32_t sw = (uint32_t)(r >> 1) & 3u;
#pragma unroll
    for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(row + ((c ^ sw) << 4)) = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
}
