#include "gc_types.h"

#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

namespace gcb {

namespace {
// Block sizes of the GGUF types (gguf-py gguf/constants.py GGML_QUANT_SIZES).
const TypeTraits kTraits[] = {
    {T_F32, "f32", 1, 4},        {T_F16, "f16", 1, 2},         {T_Q4_0, "q4_0", 32, 18},
    {T_Q4_1, "q4_1", 32, 20},    {T_Q5_0, "q5_0", 32, 22},     {T_Q5_1, "q5_1", 32, 24},
    {T_Q8_0, "q8_0", 32, 34},    {T_Q8_1, "q8_1", 32, 40},     {T_Q2_K, "q2_K", 256, 84},
    {T_Q3_K, "q3_K", 256, 110},  {T_Q4_K, "q4_K", 256, 144},   {T_Q5_K, "q5_K", 256, 176},
    {T_Q6_K, "q6_K", 256, 210},  {T_Q8_K, "q8_K", 256, 292},   {T_IQ2_XXS, "iq2_xxs", 256, 66},
    {T_IQ2_XS, "iq2_xs", 256, 74}, {T_IQ3_XXS, "iq3_xxs", 256, 98}, {T_IQ1_S, "iq1_s", 256, 50},
    {T_IQ4_NL, "iq4_nl", 32, 18}, {T_IQ3_S, "iq3_s", 256, 110}, {T_IQ2_S, "iq2_s", 256, 82},
    {T_IQ4_XS, "iq4_xs", 256, 136}, {T_I8, "i8", 1, 1},        {T_I16, "i16", 1, 2},
    {T_I32, "i32", 1, 4},        {T_I64, "i64", 1, 8},         {T_F64, "f64", 1, 8},
    {T_IQ1_M, "iq1_m", 256, 56}, {T_BF16, "bf16", 1, 2},       {T_TQ1_0, "tq1_0", 256, 54},
    {T_TQ2_0, "tq2_0", 256, 66}, {T_MXFP4, "mxfp4", 32, 17},
};
}  // namespace

const TypeTraits *type_traits(Type t) {
    for (const auto &tr : kTraits)
        if (tr.type == t) return &tr;
    return nullptr;
}

const TypeTraits *type_by_name(const std::string &name) {
    for (const auto &tr : kTraits)
        if (name == tr.name) return &tr;
    return nullptr;
}

const char *type_name(Type t) {
    const TypeTraits *tr = type_traits(t);
    return tr ? tr->name : "?";
}

size_t row_size(Type t, int64_t n) {
    const TypeTraits *tr = type_traits(t);
    if (!tr) return 0;
    return (size_t)(n / tr->block) * tr->block_size;
}

uint16_t f32_to_f16(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);  // NaN -> quiet NaN
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  // rounds to >= 65520: inf
    if (ax < 0x38800000u) {                                    // below the smallest normal half
        if (ax < 0x33000000u) return (uint16_t)sign;           // < 2^-25: rounds to 0
        // subnormal half: value = m * 2^-24, m = round(ax_value * 2^24)
        const uint32_t e = ax >> 23;
        const uint32_t mant = (ax & 0x7fffffu) | 0x800000u;
        const int shift = (int)(126 - e);  // 2^(e-127) * mant/2^23 * 2^24 = mant >> (126 - e + ... )
        // value * 2^24 = mant * 2^(e - 127 - 23 + 24) = mant * 2^(e - 126) -> shift right by 126 - e
        const uint32_t q = mant >> shift;
        const uint32_t rem = mant & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1);
        uint32_t r = q + ((rem > half || (rem == half && (q & 1u))) ? 1u : 0u);
        return (uint16_t)(sign | r);
    }
    // normal: rebias exponent, round mantissa from 23 to 10 bits (nearest even)
    uint32_t r = ax - 0x38000000u;  // exponent 127 -> 15 bias
    const uint32_t rem = r & 0x1fffu;
    r >>= 13;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r += 1;  // may carry into the exponent: fine
    return (uint16_t)(sign | r);
}

float f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    uint32_t x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else {  // subnormal: normalise
            int ee = -1;
            do {
                ee++;
                m <<= 1;
            } while ((m & 0x400u) == 0);
            x = sign | ((uint32_t)(127 - 15 - ee) << 23) | ((m & 0x3ffu) << 13);
        }
    } else if (e == 31) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    std::memcpy(&f, &x, 4);
    return f;
}

uint16_t f32_to_bf16(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 64u);  // quiet NaN
    return (uint16_t)((x + (0x7fffu + ((x >> 16) & 1u))) >> 16);
}

// Q8_0: d = amax / 127, codes round(x / d) half away from zero (ggml quantize_row_q8_0_ref).
void quantize_row_q8_0(const float *x, uint8_t *dst, int64_t n) {
    for (int64_t b = 0; b < n / QK; b++) {
        const float *xb = x + b * QK;
        uint8_t *yb = dst + b * Q8_0_BYTES;
        float amax = 0.0f;
        for (int j = 0; j < QK; j++) amax = std::fmax(amax, std::fabs(xb[j]));
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        const uint16_t dh = f32_to_f16(d);
        std::memcpy(yb, &dh, 2);
        for (int j = 0; j < QK; j++) {
            const float v = xb[j] * id;
            yb[2 + j] = (uint8_t)(int8_t)std::roundf(v);
        }
    }
}

// Q4_0: the signed value of largest magnitude (first one on ties) sets d = max / -8; codes
// min(15, trunc(x / d + 8.5)) (ggml quantize_row_q4_0_ref).
void quantize_row_q4_0(const float *x, uint8_t *dst, int64_t n) {
    for (int64_t b = 0; b < n / QK; b++) {
        const float *xb = x + b * QK;
        uint8_t *yb = dst + b * Q4_0_BYTES;
        float amax = 0.0f, max = 0.0f;
        for (int j = 0; j < QK; j++) {
            const float v = xb[j];
            if (amax < std::fabs(v)) {
                amax = std::fabs(v);
                max = v;
            }
        }
        const float d = max / -8.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        const uint16_t dh = f32_to_f16(d);
        std::memcpy(yb, &dh, 2);
        for (int j = 0; j < QK / 2; j++) {
            const float x0 = xb[j] * id;
            const float x1 = xb[QK / 2 + j] * id;
            int q0 = (int)(x0 + 8.5f);
            int q1 = (int)(x1 + 8.5f);
            q0 = q0 < 0 ? 0 : (q0 > 15 ? 15 : q0);
            q1 = q1 < 0 ? 0 : (q1 > 15 ? 15 : q1);
            yb[2 + j] = (uint8_t)(q0 | (q1 << 4));
        }
    }
}

// Q4_1 / Q5_1: d = (max - min) / 15 or / 31, the block minimum as an fp16 offset, unsigned codes
// min(top, trunc((x - min) / d + 0.5)) (ggml quantize_row_q4_1_ref / quantize_row_q5_1_ref). Q5_1
// stores bit 4 of code j in bit j of a 32-bit word after the two scales.
void quantize_row_q_min(const float *x, uint8_t *dst, int64_t n, int bits) {
    const int bs = bits == 4 ? 20 : 24, top = (1 << bits) - 1;
    for (int64_t b = 0; b < n / QK; b++) {
        const float *xb = x + b * QK;
        uint8_t *yb = dst + b * bs;
        float lo = xb[0], hi = xb[0];
        for (int j = 1; j < QK; j++) {
            lo = xb[j] < lo ? xb[j] : lo;
            hi = xb[j] > hi ? xb[j] : hi;
        }
        const float d = (hi - lo) / (float)top;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        const uint16_t dh = f32_to_f16(d), mh = f32_to_f16(lo);
        std::memcpy(yb, &dh, 2);
        std::memcpy(yb + 2, &mh, 2);
        uint32_t qh = 0;
        uint8_t *qs = yb + (bits == 4 ? 4 : 8);
        for (int j = 0; j < QK / 2; j++) {
            int q0 = (int)std::trunc((xb[j] - lo) * id + 0.5f);
            int q1 = (int)std::trunc((xb[QK / 2 + j] - lo) * id + 0.5f);
            q0 = q0 < 0 ? 0 : (q0 > top ? top : q0);
            q1 = q1 < 0 ? 0 : (q1 > top ? top : q1);
            qs[j] = (uint8_t)((q0 & 15) | ((q1 & 15) << 4));
            qh |= (uint32_t)(q0 >> 4) << j;
            qh |= (uint32_t)(q1 >> 4) << (j + QK / 2);
        }
        if (bits == 5) std::memcpy(yb + 4, &qh, 4);
    }
}

// Q5_0: the signed value of largest magnitude (first on ties) sets d = max / -16; codes
// min(31, trunc(x / d + 16.5)), bit 4 of code j in bit j of the word after the scale
// (ggml quantize_row_q5_0_ref).
void quantize_row_q5_0(const float *x, uint8_t *dst, int64_t n) {
    for (int64_t b = 0; b < n / QK; b++) {
        const float *xb = x + b * QK;
        uint8_t *yb = dst + b * 22;
        float amax = 0.0f, max = 0.0f;
        for (int j = 0; j < QK; j++)
            if (amax < std::fabs(xb[j])) {
                amax = std::fabs(xb[j]);
                max = xb[j];
            }
        const float d = max / -16.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        const uint16_t dh = f32_to_f16(d);
        std::memcpy(yb, &dh, 2);
        uint32_t qh = 0;
        for (int j = 0; j < QK / 2; j++) {
            int q0 = (int)(xb[j] * id + 16.5f);
            int q1 = (int)(xb[QK / 2 + j] * id + 16.5f);
            q0 = q0 < 0 ? 0 : (q0 > 31 ? 31 : q0);
            q1 = q1 < 0 ? 0 : (q1 > 31 ? 31 : q1);
            yb[6 + j] = (uint8_t)((q0 & 15) | ((q1 & 15) << 4));
            qh |= (uint32_t)(q0 >> 4) << j;
            qh |= (uint32_t)(q1 >> 4) << (j + QK / 2);
        }
        std::memcpy(yb + 2, &qh, 4);
    }
}

size_t quantize_rows(Type t, const float *src, int64_t nrows, int64_t n, uint8_t *dst) {
    const size_t rb = row_size(t, n);
    auto work = [&](int64_t r0, int64_t r1) {
        for (int64_t r = r0; r < r1; r++) {
            const float *x = src + r * n;
            uint8_t *y = dst + (size_t)r * rb;
            switch (t) {
                case T_Q8_0: quantize_row_q8_0(x, y, n); break;
                case T_Q4_0: quantize_row_q4_0(x, y, n); break;
                case T_Q4_1: quantize_row_q_min(x, y, n, 4); break;
                case T_Q5_1: quantize_row_q_min(x, y, n, 5); break;
                case T_Q5_0: quantize_row_q5_0(x, y, n); break;
                case T_F32: std::memcpy(y, x, (size_t)n * 4); break;
                case T_F16:
                    for (int64_t i = 0; i < n; i++) {
                        const uint16_t h = f32_to_f16(x[i]);
                        std::memcpy(y + 2 * i, &h, 2);
                    }
                    break;
                case T_BF16:
                    for (int64_t i = 0; i < n; i++) {
                        const uint16_t h = f32_to_bf16(x[i]);
                        std::memcpy(y + 2 * i, &h, 2);
                    }
                    break;
                default: break;
            }
        }
    };
    const int64_t work_elems = nrows * n;
    unsigned nt = std::thread::hardware_concurrency();
    if (nt == 0) nt = 1;
    if (work_elems < (1 << 20) || nrows < 2 || nt == 1) {
        work(0, nrows);
    } else {
        nt = (unsigned)std::min<int64_t>((int64_t)nt, nrows);
        std::vector<std::thread> th;
        for (unsigned i = 0; i < nt; i++) {
            const int64_t r0 = nrows * i / nt, r1 = nrows * (i + 1) / nt;
            th.emplace_back(work, r0, r1);
        }
        for (auto &x : th) x.join();
    }
    return rb * (size_t)nrows;
}

}  // namespace gcb
