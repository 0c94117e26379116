// Device tensor descriptors and the host launchers of every CUDA kernel of the backend.
//
// A TD is a strided view in ggml's layout: ne innermost first, nb byte strides. A quantized weight
// (Q4_0 / Q8_0) is stored on the device in the tiled layout of kernels/gc_qweight.cuh (8-row tiles
// cut into 128-block segments, codes then scales per piece), repacked from the GGUF blocks at load;
// `data` points at it and nb[1] is the code bytes of one row (a nominal stride: quantized tensors
// are only viewed row for row).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "gc_types.h"

namespace gcb {

struct TD {
    char *data = nullptr;
    uint16_t *scales = nullptr;  // quantized types only
    Type type = T_F32;
    int64_t ne[4] = {1, 1, 1, 1};
    int64_t nb[4] = {0, 0, 0, 0};
    // Planning only: storage id in the call site's arena (-1: data is an absolute pointer) and
    // byte offset into that storage.
    int sid = -1;
    size_t off = 0;

    int64_t nelements() const { return ne[0] * ne[1] * ne[2] * ne[3]; }
    int64_t nrows() const { return ne[1] * ne[2] * ne[3]; }
    size_t elsize() const;  // bytes per element (non-quantized types)
    bool contiguous() const;
    size_t nbytes() const;  // bytes spanned by a contiguous tensor of this shape
};

// Contiguous strides for a shape (quantized: code bytes of a row in nb[1]).
void set_contiguous(TD &t);
size_t quant_code_bytes(Type t);  // code bytes per 32-block: Q4_0 16, Q8_0 32

namespace k {

// Repack raw GGUF Q4_0/Q8_0 rows into the tiled device layout of quant_device_bytes bytes.
size_t quant_device_bytes(Type t, int64_t rows, int64_t K);
void repack_quant(Type t, const uint8_t *raw, int64_t nrows, int64_t K, char *dst, cudaStream_t s);

// The other GGUF block formats (kernels/gc_blockq.cu). q5_0 and iq4_nl are expanded at load into
// the Q8_0 tiled layout (quant_device_bytes(T_Q8_0, ...) bytes) and then are Q8_0 weights; q4_1,
// q5_1, q4_K, q5_K and q6_K stay in their GGUF layout (nb[0] = unit bytes, nb[1] = row bytes) and
// multiply through mul_mat_block.
bool expands_to_q8_0(Type t);
bool raw_block_type(Type t);
void expand_to_q8_0(Type t, const uint8_t *raw, int64_t nrows, int64_t K, char *dst, cudaStream_t s);
size_t mul_mat_block_scratch_bytes(const TD &a, const TD &b);
void mul_mat_block(const TD &a, const TD &b, const TD &out, void *scratch, cudaStream_t s);

// Elementwise and row ops (generic strides).
void copy(const TD &src, const TD &dst, cudaStream_t s);  // cont / cpy / cast (f32, f16, bf16, i32)
enum BinOp { ADD = 0, SUB = 1, MUL = 2, DIV = 3 };
void binary(int op, const TD &a, const TD &b, const TD &out, cudaStream_t s);
enum UnOp {
    SCALE = 0, CLAMP, SILU, NEG, ABS, SQR, SQRT, EXP, LOG, RELU, TANH, SIGMOID, STEP, SIN, COS, SOFTPLUS,
    GELU_TANH, GELU_ERF,
};
void unary(int op, const TD &x, const TD &out, float p0, float p1, cudaStream_t s);
void rms_norm(const TD &x, const TD &out, float eps, cudaStream_t s);
void norm(const TD &x, const TD &out, float eps, cudaStream_t s);
void soft_max(const TD &x, const TD *mask, const TD &out, float scale, cudaStream_t s);
void rope_neox(const TD &x, const TD &pos, const TD &out, int n_dims, const float *table, int64_t table_npos,
               float theta_scale, float freq_scale, float attn_factor, const float *freq_factors, cudaStream_t s);
void rope_norm(const TD &x, const TD &pos, const TD &out, int n_dims, const float *table, int64_t table_npos,
               float theta_scale, float freq_scale, float attn_factor, const float *freq_factors, cudaStream_t s);
void get_rows(const TD &table, const TD &idx, const TD &out, cudaStream_t s);
void set_rows(const TD &dst, const TD &src, const TD &idx, int *err, cudaStream_t s);
// Quantized mul_mat of 9+ activation rows on the tensor cores (gc_gemm_tc.cu): shapes it takes, and
// the launch over activation codes / fp16 scales as act_quant writes them.
bool gemm_tc_ok(const TD &a, const TD &b);
void gemm_tc(const TD &a, int64_t M, const int8_t *qx, const uint16_t *dx, float *out, int *err, cudaStream_t s);

// Activation rows from which a quantized mul_mat sums its blocks in order (GEMM) rather than into 32
// lane partials and a butterfly (GEMV); the CPU checker uses the same rule.
constexpr int64_t GEMM_MIN_ROWS = 9;

void argmax(const TD &x, const TD &out, cudaStream_t s);
// Long f32 rows: slices per row (0: use argmax), then the split form with scratch of rows x parts
// float2 pairs and rows zeroed counters (reset by the kernel).
int argmax_split_parts(const TD &x);
void argmax_split(const TD &x, const TD &out, void *scratch, int *counters, cudaStream_t s);
void swiglu(const TD &g, const TD &u, const TD &out, cudaStream_t s);
void sum_rows(const TD &x, const TD &out, float scale, cudaStream_t s);  // scale = 1/n for mean
void repeat(const TD &x, const TD &out, cudaStream_t s);
void concat(const TD &a, const TD &b, const TD &out, int dim, cudaStream_t s);
void arange(const TD &out, float start, float step, cudaStream_t s);
void fill_f32(float *dst, int64_t n, float v, cudaStream_t s);

// A driver loop's per-iteration bookkeeping on the device (gc_loop.cu). Pointers are device
// memory; `iter` is the index of the iteration about to run, `start` the counters' start values.
constexpr int LOOP_MAX = 4;      // counters, masks, scalars, slices, collects and stop tests per loop
constexpr int LOOP_MAX_IDS = 8;  // stop ids per test
struct LoopDev {
    int32_t *iter = nullptr, *stop = nullptr, *end = nullptr;  // end: iterations to run before pausing
    const int32_t *start = nullptr;
    int n_counters = 0;
    int32_t *counter[LOOP_MAX] = {};
    int n_masks = 0;
    float *mask[LOOP_MAX] = {};
    int64_t mask_n[LOOP_MAX] = {}, mask_row[LOOP_MAX] = {};
    int mask_counter[LOOP_MAX] = {};
    int n_scalars = 0;
    float *scalar[LOOP_MAX] = {};
    int64_t scalar_n[LOOP_MAX] = {};
    const float *scalar_vals[LOOP_MAX] = {};  // [trips] per scalar
    int n_slices = 0;
    char *slice_dst[LOOP_MAX] = {};
    const char *slice_src[LOOP_MAX] = {};
    int64_t slice_bytes[LOOP_MAX] = {};
    int n_collect = 0;
    char *collect_dst[LOOP_MAX] = {};
    const char *collect_src[LOOP_MAX] = {};
    int64_t collect_bytes[LOOP_MAX] = {};
    int n_until = 0;
    const int32_t *until_val[LOOP_MAX] = {};
    int32_t until_ids[LOOP_MAX][LOOP_MAX_IDS] = {};
    int n_ids[LOOP_MAX] = {};
};
void loop_begin(const LoopDev &L, cudaStream_t s);
// `use_cond`: also set `cond` (the loop's WHILE node) for the next iteration.
void loop_end(const LoopDev &L, cudaGraphConditionalHandle cond, bool use_cond, cudaStream_t s);
void loop_guard(const LoopDev &L, cudaGraphConditionalHandle cond, cudaStream_t s);
// Batched decode bookkeeping (kernels/gc_loop.cu): the causal mask of each sequence's row
// ([n][window] f16: 0 for keys up to pos[i], -inf after), and one greedy step's hand-over (tok :=
// next, pos += 1, out[step][i] := next, step += 1).
void batch_mask(__half *mask, const int32_t *pos, int n, int64_t window, cudaStream_t s);
void batch_advance(int32_t *tok, int32_t *pos, const int32_t *next, int32_t *out, int32_t *step, int n, cudaStream_t s);

// mul_mat(a, b): out[n, m, i2, i3] = sum_k a[k, n, i2/r2, i3/r3] * b[k, m, i2, i3].
// `scratch` must hold mul_mat_scratch_bytes(a, b) bytes.
size_t mul_mat_scratch_bytes(const TD &a, const TD &b);
void mul_mat(const TD &a, const TD &b, const TD &out, void *scratch, cudaStream_t s, int *err = nullptr);

// flash_attn_ext: q [D, Sq, H, B] f32, k/v [D, n_kv, Hkv, B] f16, mask [n_kv, >=Sq, ...] f16 (nullable)
// -> out [D, H, Sq, B] f32.
void flash_attn(const TD &q, const TD &k, const TD &v, const TD *mask, const TD &out, float scale, cudaStream_t s);

// Split-KV flash attention (gc_flash.cu): head size <= 256 and a multiple of 32; same result as
// flash_attn. `counters` (flash_split_counters ints) must be zero before the first launch and are
// left zero by every launch; `scratch` holds flash_split_scratch_bytes.
bool flash_split_ok(const TD &q);
size_t flash_split_scratch_bytes(const TD &q, const TD &k);
size_t flash_split_counters(const TD &q, const TD &k);
// kv_pos (one query row; cluster kernel only): the positions [batch] of the K/V rows the kernel
// launched before this one writes. The cluster kernel then copies the chunk's K/V before its
// dependent-launch wait (the other rows were written by earlier launches that completed before
// the kernel before it started: a graph launch or loop iteration boundary) and reads that row
// again after the wait. Null: every copy after the wait.
void flash_attn_split(const TD &q, const TD &k, const TD &v, const TD *mask, const TD &out, float scale, void *scratch,
                      int *counters, int *err, cudaStream_t s, uint64_t *trace = nullptr, char *act_out = nullptr,
                      const int32_t *kv_pos = nullptr, bool prefill_tc = false);
size_t flash_split_ctas(const TD &q, const TD &k);  // CTAs of one split launch (trace slots)
// One decode row of 2-16 chunks runs as thread-block clusters (one per K/V head, chunk partials
// merged through distributed shared memory) when such clusters fit; this asks once, outside any
// stream capture, and says whether they do. GCB_ATTN_CLUSTER=0 keeps the split kernel.
bool flash_split_prepare(const TD &q, const TD &k, const TD &v, const TD &out);
// act_out (one query row, one batch): the merged row's Q8_0 blocks in the GEMV staging layout
// (gemv_act_bytes(1, H x D) bytes) for the GEMV that reads it (FusedArgs::PRO_Q8).
// The same result for prefill calls (16+ query rows, head size 64 or 128, K/V rows contiguous):
// one CTA per 64 (row, head) pairs over every chunk, merge in the CTA (gc_flash_prefill.cu).
bool flash_prefill_ok(const TD &q, const TD &k, const TD &v, const TD &out);
void flash_prefill(const TD &q, const TD &k, const TD &v, const TD *mask, const TD &out, float scale, int *err,
                   cudaStream_t s);
// The same shapes on the tensor cores (gc_flash_prefill_tc.cu): within tolerance of the checker, not
// bit-exact; flash_attn_split takes it instead of flash_prefill when asked (prefill_tc: the model
// was loaded with GGML_COMPILER_B200_PREFILL_ATTN=tc).
void flash_prefill_tc(const TD &q, const TD &k, const TD &v, const TD *mask, const TD &out, float scale, cudaStream_t s);

// Tensor-parallel exchange (gc_tp.cu). A window is TP_FLAG_BYTES of flag words (one per sender)
// followed by two slots of slot_bytes; every rank maps every window.
constexpr int TP_MAX = 8;
constexpr int64_t TP_FLAG_BYTES = 256;
struct TpExchange {
    char *buf = nullptr;  // the local buffer: `rows` rows at a stride of `ld` bytes
    int64_t rows = 0, ld = 0, row_bytes = 0;
    int64_t col[TP_MAX + 1] = {};  // rank r computed bytes [col[r], col[r + 1]) of every row
    int rank = 0, world = 1;
    char *win[TP_MAX] = {};  // the window of every rank (this rank's included)
    int64_t slot_bytes = 0;
    unsigned *seq = nullptr;  // exchanges done by this rank (device word)
    unsigned *done = nullptr; // CTAs of the running exchange that finished (device word, left at 0)
    int *err = nullptr;
    uint64_t timeout_ns = 0;
};
bool tp_exchange_ok(const TpExchange &x);  // geometry (the buffer's alignment is checked at launch)
void tp_exchange(const TpExchange &x, cudaStream_t s);

}  // namespace k
}  // namespace gcb
