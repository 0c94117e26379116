// Device access to the GGUF block formats this backend computes with in their stored layout
// (q4_1, q5_1, q4_K, q5_K, q6_K: the GGUF bytes uploaded unchanged) and the codes of the two it
// expands at load (q5_0, iq4_nl -> the Q8_0 tiled layout). Layouts, per unit of 32 or 256 values:
//
//   q4_1   [d f16][m f16][16 B]            value j: low nibble of byte j, value j + 16: high nibble
//   q5_1   [d f16][m f16][qh u32][16 B]    bit 4 of value j: bit j of qh
//   q5_0   [d f16][qh u32][16 B]           values q - 16
//   iq4_nl [d f16][16 B]                   values iq4nl_value(nibble), a fixed 16-entry table
//   q4_K   [d f16][dmin f16][12 B scales/mins][128 B]   8 sub-blocks of 32: value 32j + l is nibble
//          j % 2 of byte 32 (j / 2) + l; w = d sc_j q - dmin m_j with 6-bit sc_j, m_j
//   q5_K   [d f16][dmin f16][12 B][32 B qh][128 B]      bit 4 of value 32j + l: bit j of qh[l]
//   q6_K   [128 B low nibbles][64 B high 2 bits][16 x int8 scales][d f16]   16 sub-blocks of 16,
//          w = d sc_j (q - 32)
//
// (ggml's block_q4_1 ... block_q6_K, as gguf-py gguf/quants.py restates them.)
#pragma once

#include <cstdint>

#include "../gc_types.h"
#include "gc_math.cuh"

namespace gcb {

__device__ __forceinline__ uint32_t ld16(const uint8_t *p) { return *(const uint16_t *)p; }
// 32 bits from a 2-byte aligned address (q6_K super-blocks are 210 bytes apart)
__device__ __forceinline__ uint32_t ld32a2(const uint8_t *p) { return ld16(p) | (ld16(p + 2) << 16); }
__device__ __forceinline__ uint32_t ld32(const uint8_t *p) { return *(const uint32_t *)p; }

// bits 0..3 of b -> bit 4 of bytes 0..3
__device__ __forceinline__ uint32_t spread4(uint32_t b) {
    return ((b & 1u) << 4) | ((b & 2u) << 11) | ((b & 4u) << 18) | ((b & 8u) << 25);
}

__device__ __forceinline__ int iq4nl_value(int i) {
    const int8_t t[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};
    return t[i & 15];
}

// q4_K / q5_K: 6-bit scale and min of sub-block j from the 12 packed bytes
__device__ __forceinline__ void kq_scale_min(const uint8_t *s, int j, int &sc, int &m) {
    if (j < 4) {
        sc = s[j] & 63;
        m = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
        m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

__device__ __forceinline__ int unit_values(int type) { return (type == T_Q4_1 || type == T_Q5_1) ? 32 : 256; }
__device__ __forceinline__ int unit_bytes(int type) {
    switch (type) {
        case T_Q4_1: return 20;
        case T_Q5_1: return 24;
        case T_Q4_K: return 144;
        case T_Q5_K: return 176;
        default: return 210;  // q6_K
    }
}

// Element i of a row stored in one of the raw formats, as ggml's dequantize_row_* computes it
// (every product and difference one IEEE-rounded step).
__device__ __forceinline__ float dequant_raw(int type, const uint8_t *row, int64_t i) {
    const int un = unit_values(type);
    const uint8_t *blk = row + (i / un) * unit_bytes(type);
    const int v = (int)(i % un);
    if (type == T_Q4_1 || type == T_Q5_1) {
        const uint8_t byte = blk[(type == T_Q4_1 ? 4 : 8) + (v & 15)];
        int q = v < 16 ? (byte & 15) : (byte >> 4);
        if (type == T_Q5_1) q |= (int)((ld32(blk + 4) >> v) & 1u) << 4;
        return __fadd_rn(__fmul_rn(h2f((uint16_t)ld16(blk)), (float)q), h2f((uint16_t)ld16(blk + 2)));
    }
    if (type == T_Q6_K) {
        const int h = v / 128, r = v % 128;
        const int lo = (blk[64 * h + r % 64] >> (4 * (r / 64))) & 15;
        const int hi = (blk[128 + 32 * h + r % 32] >> (2 * (r / 32))) & 3;
        const float d = h2f((uint16_t)ld16(blk + 208));
        return __fmul_rn(__fmul_rn(d, (float)(int8_t)blk[192 + v / 16]), (float)((lo | (hi << 4)) - 32));
    }
    const int j = v / 32, l = v % 32;
    int q;
    if (type == T_Q4_K) {
        q = (blk[16 + 32 * (j / 2) + l] >> (4 * (j % 2))) & 15;
    } else {
        q = ((blk[48 + 32 * (j / 2) + l] >> (4 * (j % 2))) & 15) | (((blk[16 + l] >> j) & 1) << 4);
    }
    int sc, m;
    kq_scale_min(blk + 4, j, sc, m);
    const float d1 = __fmul_rn(h2f((uint16_t)ld16(blk)), (float)sc);
    const float m1 = __fmul_rn(h2f((uint16_t)ld16(blk + 2)), (float)m);
    return __fsub_rn(__fmul_rn(d1, (float)q), m1);
}

}  // namespace gcb
