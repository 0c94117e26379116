// Tensor element types of ggml-compiler programs and GGUF files, and their storage sizes.
//
// The numeric ids are the GGUF on-disk type ids (the `ggml_type` enum that gguf-py mirrors in
// gguf/constants.py GGMLQuantizationType); the names are the ones the program JSON uses
// (reference runtime/src/program.cpp:12-20 resolves them through ggml_type_name). Only the block
// sizes are needed to lay out any type; this backend computes on f32, f16, i32, q4_0 and q8_0.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>

namespace gcb {

enum Type : int {
    T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8, T_Q8_1 = 9,
    T_Q2_K = 10, T_Q3_K = 11, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14, T_Q8_K = 15,
    T_IQ2_XXS = 16, T_IQ2_XS = 17, T_IQ3_XXS = 18, T_IQ1_S = 19, T_IQ4_NL = 20, T_IQ3_S = 21,
    T_IQ2_S = 22, T_IQ4_XS = 23, T_I8 = 24, T_I16 = 25, T_I32 = 26, T_I64 = 27, T_F64 = 28,
    T_IQ1_M = 29, T_BF16 = 30, T_TQ1_0 = 34, T_TQ2_0 = 35, T_MXFP4 = 39,
    T_INVALID = -1,
};

struct TypeTraits {
    Type        type;
    const char *name;
    int64_t     block;      // elements per block
    size_t      block_size; // bytes per block
};

const TypeTraits *type_traits(Type t);       // nullptr for an unknown id
const TypeTraits *type_by_name(const std::string &name);  // nullptr if unknown
inline bool is_quantized(Type t) { return t != T_F32 && t != T_F16 && t != T_BF16 && t != T_I32 && t != T_I8 &&
                                          t != T_I16 && t != T_I64 && t != T_F64; }
size_t row_size(Type t, int64_t n);          // bytes of n elements (n a multiple of the block)
const char *type_name(Type t);

// Q4_0 / Q8_0 block geometry (ggml: 32 values per block behind one fp16 scale).
constexpr int QK = 32;
constexpr size_t Q4_0_BYTES = 18;  // fp16 d + 16 bytes: byte j holds element j (low nibble), j+16 (high)
constexpr size_t Q8_0_BYTES = 34;  // fp16 d + 32 int8 codes

// IEEE half <-> float, round to nearest even (ggml's GGML_FP32_TO_FP16 rounding).
uint16_t f32_to_f16(float f);
float f16_to_f32(uint16_t h);
uint16_t f32_to_bf16(float f);

// Encoders, byte-exact with ggml's reference quantizers (gguf-py 0.19 gguf/quants.py Q4_0 :220-252,
// Q8_0 :378-402, which state bit-equality with ggml-quants.c). Rows are n elements, n % 32 == 0.
void quantize_row_q8_0(const float *x, uint8_t *dst, int64_t n);
void quantize_row_q4_0(const float *x, uint8_t *dst, int64_t n);
void quantize_row_q_min(const float *x, uint8_t *dst, int64_t n, int bits);  // q4_1 (4), q5_1 (5)
void quantize_row_q5_0(const float *x, uint8_t *dst, int64_t n);
// Multithreaded over rows; returns bytes written.
size_t quantize_rows(Type t, const float *src, int64_t nrows, int64_t n, uint8_t *dst);

}  // namespace gcb
