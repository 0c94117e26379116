/*
 * ggml_oracle.c - TEST INFRASTRUCTURE ONLY. A CPU restatement of the arithmetic that the
 * reference (khanhnd61-vr/ggml-compiler) runs through ggml's CPU backend for the LLM op subset.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it, and only
 * as the checker or as the timed CPU baseline. The product library never links or calls it.
 *
 * What is restated, and from where:
 * - Q4_0 / Q8_0 block encoders: ggml's reference quantizers as gguf-py 0.19 restates them
 *   (gguf/quants.py Q4_0.quantize_blocks :220-252, Q8_0.quantize_blocks :378-402; the reference
 *   calls them through ggml_compiler_quantize, runtime/src/ggml_compiler_rt.cpp:859-876).
 *   Pinned bit-exact against gguf-py by tests/test_quant.py.
 * - mul_mat with a Q4_0/Q8_0 weight (reference runtime/src/ops.cpp:107-119 ->
 *   runtime/include/ggml_compiler_ops.h:116-122 -> ggml_mul_mat): ggml's CPU backend converts the
 *   f32 activation row to Q8_0 blocks (the x86 AVX2 from_float rule: d = amax/127 stored as fp16,
 *   codes = round-to-nearest-even(x * 127/amax)), then sums per-block integer dot products scaled
 *   by d_w * d_x in f32.
 * - mul_mat with an f16 weight converts the activation to f16 first (ggml's vec_dot_type for f16);
 *   products are then exact in f32.
 * - The other block formats the reference stores weights in (ggml_compiler/quant/types.py:6-19):
 *   q4_1, q5_0, q5_1 encoders (gguf-py quants.py Q4_1 / Q5_0 / Q5_1 quantize_blocks); the layouts
 *   of all seven (gguf-py dequantize_blocks, pinned bit for bit by tests/test_block_formats.py);
 *   q5_0 / iq4_nl matmuls as ggml's vec_dot_q5_0_q8_0 / vec_dot_iq4_nl_q8_0 (a Q8_0 block dot of
 *   the expanded codes); q4_1 / q5_1 over Q8_1 activations and q4_K / q5_K / q6_K over Q8_K
 *   activations (ggml quantize_row_q8_1 on x86, quantize_row_q8_K_ref) with the per-unit terms of
 *   ggml's vec_dot_*_q8_1 / vec_dot_*_q8_K.
 * - rms_norm (ops.cpp:144-148): the sum of squares in double, 1/sqrtf(mean + eps) in float.
 * - rope NEOX (ops.cpp:277-291): angles theta_i = p * s^i by repeated float multiplication,
 *   s = powf(base, -2/n_dims), cos/sin from libm, halves rotated together.
 * - soft_max, flash_attn (ops.cpp:217-243, ggml_compiler_ops.h:124-148): scores of Q rounded to f16
 *   against the f16 K cache, f32 accumulation (the reference asks for GGML_PREC_F32), masked
 *   keys (-inf) skipped, output divided by the softmax sum (0 when every key is masked).
 * - swiglu silu(g)*u, argmax (first maximum), get_rows, set_rows: as ggml.
 *
 * ggml's exact float summation order is not visible from the reference tree (ggml is fetched at
 * build time, llama.cpp tag b11223) and differs between its SIMD paths. This restatement fixes one
 * order for every reduction; the B200 kernels follow the same orders, so their decode results can
 * be compared bit for bit. The orders:
 * - 32-lane butterfly: 32 partial sums, then p[i] += p[i ^ off] for off = 16, 8, 4, 2, 1.
 * - other block formats: unit u (32-block, or 256-value super-block for the K-quants) goes to
 *   partial u % 32, then the butterfly, for any number of rows.
 * - quantized dot, up to 8 activation rows: block b goes to partial b % 32
 *   (fmaf(d_w*d_x, isum, p)), then the butterfly; 9 or more rows: every block in order into one sum
 *   (the integer block dots are exact, so only the order of the fmaf chain matters).
 * - float dot: element k goes to partial k % 32 (fmaf), then the butterfly.
 * - head dot (attention, D % 32 == 0): lane l owns elements [l*D/32, (l+1)*D/32), then butterfly.
 * - 256-way double tree (rms_norm, softmax sums): element i goes to partial i % 256, then
 *   p[t] += p[t + off] for off = 128 ... 1.
 * - flash attention: keys in chunks of 64; per chunk max, exp, sum and weighted V in key order;
 *   chunks merged in order with weights exp(m_c - M).
 * - exp: orc_expf below (range reduction by ln 2, degree-7 Taylor polynomial, 2^n by two exact
 *   scalings); the GPU kernels use the same function.
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off, pthreads).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#define QK 32
#define FA_CHUNK 64

enum {
    ORC_F32 = 0, ORC_F16 = 1, ORC_Q4_0 = 2, ORC_Q4_1 = 3, ORC_Q5_0 = 6, ORC_Q5_1 = 7, ORC_Q8_0 = 8,
    ORC_Q4_K = 12, ORC_Q5_K = 13, ORC_Q6_K = 14, ORC_IQ4_NL = 20
};
#define QKK 256

/* ---------------------------------------------------------------------------------------------
 * A static-schedule parallel for over [0, n) on all host threads (ORC_THREADS overrides). */
typedef struct {
    void (*fn)(void *, int64_t, int64_t);
    void *ctx;
    int64_t lo, hi;
} orc_job;

static void *orc_job_run(void *a) {
    orc_job *j = (orc_job *)a;
    j->fn(j->ctx, j->lo, j->hi);
    return NULL;
}

static int orc_n_threads = 0;
void orc_set_threads(int n) { orc_n_threads = n; }
int orc_get_threads(void) {
    if (orc_n_threads > 0) return orc_n_threads;
    const char *e = getenv("ORC_THREADS");
    if (e && atoi(e) > 0) return atoi(e);
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

static void orc_parallel_for(int64_t n, void (*fn)(void *, int64_t, int64_t), void *ctx) {
    int nt = orc_get_threads();
    if (nt > 256) nt = 256;
    if (n < 2 * nt) nt = n > 0 ? (int)(n < nt ? n : nt) : 1;
    if (nt <= 1) {
        fn(ctx, 0, n);
        return;
    }
    pthread_t th[256];
    orc_job jobs[256];
    for (int i = 0; i < nt; i++) {
        jobs[i].fn = fn;
        jobs[i].ctx = ctx;
        jobs[i].lo = n * i / nt;
        jobs[i].hi = n * (i + 1) / nt;
        pthread_create(&th[i], NULL, orc_job_run, &jobs[i]);
    }
    for (int i = 0; i < nt; i++) pthread_join(th[i], NULL);
}


/* fp16 through the compiler's _Float16 (round to nearest even), independent of the product code. */
static inline float h2f(uint16_t h) {
    _Float16 v;
    memcpy(&v, &h, 2);
    return (float)v;
}
static inline uint16_t f2h(float f) {
    _Float16 v = (_Float16)f;
    uint16_t h;
    memcpy(&h, &v, 2);
    return h;
}

float orc_h2f(uint16_t h) { return h2f(h); }
uint16_t orc_f2h(float f) { return f2h(f); }

/* ---------------------------------------------------------------------------------------------
 * Block encoders (gguf-py quants.py :220-252, :378-402). */

static void quant_q8_0_row(const float *x, uint8_t *y, int64_t n) {
    for (int64_t b = 0; b < n / QK; b++) {
        const float *xb = x + b * QK;
        uint8_t *yb = y + b * 34;
        float amax = 0.0f;
        for (int j = 0; j < QK; j++) {
            const float a = fabsf(xb[j]);
            if (a > amax) amax = a;
        }
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        const uint16_t dh = f2h(d);
        memcpy(yb, &dh, 2);
        for (int j = 0; j < QK; j++) {
            /* round half away from zero, as gguf-py's np_roundf and C roundf */
            const float v = xb[j] * id;
            const float a = fabsf(v);
            float r = floorf(a);
            r = r + floorf(2.0f * (a - r));
            yb[2 + j] = (uint8_t)(int8_t)(v < 0 ? -r : r);
        }
    }
}

static void quant_q4_0_row(const float *x, uint8_t *y, int64_t n) {
    for (int64_t b = 0; b < n / QK; b++) {
        const float *xb = x + b * QK;
        uint8_t *yb = y + b * 18;
        int imax = 0;
        float amax = fabsf(xb[0]);
        for (int j = 1; j < QK; j++) {
            if (fabsf(xb[j]) > amax) {
                amax = fabsf(xb[j]);
                imax = j;
            }
        }
        const float d = xb[imax] / -8.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        const uint16_t dh = f2h(d);
        memcpy(yb, &dh, 2);
        uint8_t q[QK];
        for (int j = 0; j < QK; j++) {
            float t = truncf(xb[j] * id + 8.5f);
            int v = (int)t;
            q[j] = (uint8_t)(v < 0 ? 0 : (v > 15 ? 15 : v));
        }
        for (int j = 0; j < QK / 2; j++) yb[2 + j] = (uint8_t)(q[j] | (q[j + QK / 2] << 4));
    }
}

/* Q4_1 / Q5_1: d = (max - min) / (2^bits - 1), codes trunc((x - min) / d + 0.5) clipped, min kept
 * as the block's fp16 offset (gguf-py quants.py Q4_1.quantize_blocks, Q5_1.quantize_blocks). */
static void quant_q_min_row(const float *x, uint8_t *y, int64_t n, int bits) {
    const int bs = bits == 4 ? 20 : 24, top = (1 << bits) - 1;
    for (int64_t b = 0; b < n / QK; b++) {
        const float *xb = x + b * QK;
        uint8_t *yb = y + b * bs;
        float mx = xb[0], mn = xb[0];
        for (int j = 1; j < QK; j++) {
            if (xb[j] > mx) mx = xb[j];
            if (xb[j] < mn) mn = xb[j];
        }
        const float d = (mx - mn) / (float)top;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        const uint16_t dh = f2h(d), mh = f2h(mn);
        memcpy(yb, &dh, 2);
        memcpy(yb + 2, &mh, 2);
        uint8_t q[QK];
        for (int j = 0; j < QK; j++) {
            const float t = truncf((xb[j] - mn) * id + 0.5f);
            const int v = (int)t;
            q[j] = (uint8_t)(v < 0 ? 0 : (v > top ? top : v));
        }
        uint8_t *qs = yb + (bits == 4 ? 4 : 8);
        for (int j = 0; j < QK / 2; j++) qs[j] = (uint8_t)((q[j] & 15) | ((q[j + QK / 2] & 15) << 4));
        if (bits == 5) {
            uint32_t qh = 0;
            for (int j = 0; j < QK; j++) qh |= (uint32_t)(q[j] >> 4) << j;
            memcpy(yb + 4, &qh, 4);
        }
    }
}

/* Q5_0: the value of largest magnitude (first on ties) sets d = max / -16; codes
 * trunc(x / d + 16.5) clipped to 0..31; bit 4 of code j in bit j of qh (gguf-py quants.py
 * Q5_0.quantize_blocks). */
static void quant_q5_0_row(const float *x, uint8_t *y, int64_t n) {
    for (int64_t b = 0; b < n / QK; b++) {
        const float *xb = x + b * QK;
        uint8_t *yb = y + b * 22;
        int imax = 0;
        float amax = fabsf(xb[0]);
        for (int j = 1; j < QK; j++)
            if (fabsf(xb[j]) > amax) {
                amax = fabsf(xb[j]);
                imax = j;
            }
        const float d = xb[imax] / -16.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        const uint16_t dh = f2h(d);
        memcpy(yb, &dh, 2);
        uint8_t q[QK];
        for (int j = 0; j < QK; j++) {
            const int v = (int)truncf(xb[j] * id + 16.5f);
            q[j] = (uint8_t)(v < 0 ? 0 : (v > 31 ? 31 : v));
        }
        uint32_t qh = 0;
        for (int j = 0; j < QK; j++) qh |= (uint32_t)(q[j] >> 4) << j;
        memcpy(yb + 2, &qh, 4);
        for (int j = 0; j < QK / 2; j++) yb[6 + j] = (uint8_t)((q[j] & 15) | ((q[j + QK / 2] & 15) << 4));
    }
}

size_t orc_row_size(int type, int64_t n) {
    switch (type) {
        case ORC_F32: return (size_t)n * 4;
        case ORC_F16: return (size_t)n * 2;
        case ORC_Q4_0: return (size_t)(n / QK) * 18;
        case ORC_Q8_0: return (size_t)(n / QK) * 34;
        case ORC_Q4_1: return (size_t)(n / QK) * 20;
        case ORC_Q5_0: return (size_t)(n / QK) * 22;
        case ORC_Q5_1: return (size_t)(n / QK) * 24;
        case ORC_IQ4_NL: return (size_t)(n / QK) * 18;
        case ORC_Q4_K: return (size_t)(n / QKK) * 144;
        case ORC_Q5_K: return (size_t)(n / QKK) * 176;
        case ORC_Q6_K: return (size_t)(n / QKK) * 210;
        default: return 0;
    }
}

typedef struct {
    int type;
    const float *src;
    int64_t n;
    uint8_t *dst;
    size_t rb;
} quant_ctx;

static void quant_rows(void *c, int64_t r0, int64_t r1) {
    const quant_ctx *q = (const quant_ctx *)c;
    for (int64_t r = r0; r < r1; r++) {
        const float *x = q->src + r * q->n;
        uint8_t *y = q->dst + r * q->rb;
        switch (q->type) {
            case ORC_Q8_0: quant_q8_0_row(x, y, q->n); break;
            case ORC_Q4_0: quant_q4_0_row(x, y, q->n); break;
            case ORC_Q4_1: quant_q_min_row(x, y, q->n, 4); break;
            case ORC_Q5_1: quant_q_min_row(x, y, q->n, 5); break;
            case ORC_Q5_0: quant_q5_0_row(x, y, q->n); break;
            default: break;
        }
    }
}

size_t orc_quantize(int type, const float *src, int64_t nrows, int64_t n, uint8_t *dst) {
    const size_t rb = orc_row_size(type, n);
    if (rb == 0 || n % QK ||
        (type != ORC_Q8_0 && type != ORC_Q4_0 && type != ORC_Q4_1 && type != ORC_Q5_0 && type != ORC_Q5_1))
        return 0;
    quant_ctx c = {type, src, n, dst, rb};
    orc_parallel_for(nrows, quant_rows, &c);
    return rb * (size_t)nrows;
}

/* ---------------------------------------------------------------------------------------------
 * Block layouts (the GGUF bytes; gguf-py quants.py dequantize_blocks restates each one):
 *   q4_1 [d f16][m f16][16 B nibbles]        value j: low nibble of byte j, j + 16: high nibble
 *   q5_0 [d f16][qh u32][16 B nibbles]       bit 4 of value j is bit j of qh; values q - 16
 *   q5_1 [d f16][m f16][qh u32][16 B]
 *   iq4_nl [d f16][16 B nibbles]             values IQ4_NL_VALUES[nibble]
 *   q4_K [d f16][dmin f16][12 B 6-bit scales and mins][128 B nibbles]       256 values, 8 x 32
 *   q5_K [d f16][dmin f16][12 B][32 B qh][128 B nibbles]
 *   q6_K [128 B low nibbles][64 B 2-bit highs][16 int8 scales][d f16]          16 x 16, q - 32
 * The iq4_nl value table is part of the format (gguf-py IQ4_NL.kvalues). */
static const int8_t IQ4_NL_VALUES[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

static inline float blk_h(const uint8_t *p) {
    uint16_t h;
    memcpy(&h, p, 2);
    return h2f(h);
}

/* Codes of one 32-value block as ggml's integer dot sees them: signed for q5_0 / iq4_nl (q4_0 and
 * q8_0 too), unsigned (0..15 / 0..31, the offset m applied separately) for q4_1 / q5_1. */
static void block_codes(int type, const uint8_t *blk, int *c) {
    uint32_t qh = 0;
    const uint8_t *qs;
    switch (type) {
        case ORC_Q4_0: qs = blk + 2; break;
        case ORC_Q4_1: qs = blk + 4; break;
        case ORC_Q5_0: memcpy(&qh, blk + 2, 4); qs = blk + 6; break;
        case ORC_Q5_1: memcpy(&qh, blk + 4, 4); qs = blk + 8; break;
        case ORC_IQ4_NL: qs = blk + 2; break;
        default: /* q8_0 */
            for (int j = 0; j < QK; j++) c[j] = (int8_t)blk[2 + j];
            return;
    }
    for (int j = 0; j < QK / 2; j++) {
        int lo = qs[j] & 15, hi = qs[j] >> 4;
        lo |= (int)((qh >> j) & 1) << 4;
        hi |= (int)((qh >> (j + 16)) & 1) << 4;
        if (type == ORC_IQ4_NL) {
            lo = IQ4_NL_VALUES[lo];
            hi = IQ4_NL_VALUES[hi];
        } else if (type == ORC_Q4_0) {
            lo -= 8;
            hi -= 8;
        } else if (type == ORC_Q5_0) {
            lo -= 16;
            hi -= 16;
        }
        c[j] = lo;
        c[j + 16] = hi;
    }
}

/* q4_K / q5_K sub-block j (0..7): its 6-bit scale and min. */
static void kq_scale_min(const uint8_t *sc12, int j, int *sc, int *m) {
    if (j < 4) {
        *sc = sc12[j] & 63;
        *m = sc12[j + 4] & 63;
    } else {
        *sc = (sc12[j + 4] & 15) | ((sc12[j - 4] >> 6) << 4);
        *m = (sc12[j + 4] >> 4) | ((sc12[j] >> 6) << 4);
    }
}

/* Codes of one 256-value super-block: q4_K / q5_K unsigned (0..15 / 0..31), q6_K signed (q - 32). */
static void kq_codes(int type, const uint8_t *blk, int *c) {
    for (int v = 0; v < QKK; v++) {
        const int j = v / 32, l = v % 32;
        if (type == ORC_Q4_K) {
            c[v] = (blk[16 + 32 * (j / 2) + l] >> (4 * (j % 2))) & 15;
        } else if (type == ORC_Q5_K) {
            c[v] = ((blk[48 + 32 * (j / 2) + l] >> (4 * (j % 2))) & 15) | (((blk[16 + l] >> j) & 1) << 4);
        } else {
            const int h = v / 128, r = v % 128;
            const int lo = (blk[64 * h + r % 64] >> (4 * (r / 64))) & 15;
            const int hi = (blk[128 + 32 * h + r % 32] >> (2 * (r / 32))) & 3;
            c[v] = (lo | (hi << 4)) - 32;
        }
    }
}

void orc_dequantize(int type, const uint8_t *src, int64_t nrows, int64_t n, float *dst) {
    const size_t rb = orc_row_size(type, n);
    const int kq = type == ORC_Q4_K || type == ORC_Q5_K || type == ORC_Q6_K;
    const size_t ub = kq ? orc_row_size(type, QKK) : orc_row_size(type, QK);
    const int64_t un = kq ? QKK : QK;
    for (int64_t r = 0; r < nrows; r++) {
        const uint8_t *x = src + r * rb;
        float *y = dst + r * n;
        for (int64_t u = 0; u < n / un; u++) {
            const uint8_t *blk = x + u * ub;
            float *yu = y + u * un;
            int c[QKK];
            if (!kq) {
                block_codes(type, blk, c);
                const float d = blk_h(blk);
                for (int j = 0; j < QK; j++) {
                    if (type == ORC_Q4_1 || type == ORC_Q5_1) yu[j] = d * (float)c[j] + blk_h(blk + 2);
                    else yu[j] = d * (float)c[j];
                }
            } else if (type == ORC_Q6_K) {
                kq_codes(type, blk, c);
                const float d = blk_h(blk + 208);
                for (int v = 0; v < QKK; v++) yu[v] = (d * (float)(int8_t)blk[192 + v / 16]) * (float)c[v];
            } else {
                kq_codes(type, blk, c);
                const float d = blk_h(blk), dmin = blk_h(blk + 2);
                for (int j = 0; j < 8; j++) {
                    int sc, m;
                    kq_scale_min(blk + 4, j, &sc, &m);
                    const float d1 = d * (float)sc, m1 = dmin * (float)m;
                    for (int l = 0; l < 32; l++) yu[32 * j + l] = d1 * (float)c[32 * j + l] - m1;
                }
            }
        }
    }
}

/* Activation row -> Q8_0 blocks, the rule ggml's x86 CPU backend applies to src1 of mul_mat:
 * d = amax / 127 (stored fp16), codes = nearest-even(x * (127 / amax)). */
void orc_act_q8_0(const float *x, int64_t n, int8_t *q, uint16_t *d) {
    for (int64_t b = 0; b < n / QK; b++) {
        float amax = 0.0f;
        for (int j = 0; j < QK; j++) {
            const float a = fabsf(x[b * QK + j]);
            if (a > amax) amax = a;
        }
        d[b] = f2h(amax / 127.0f);
        const float id = amax != 0.0f ? 127.0f / amax : 0.0f;
        for (int j = 0; j < QK; j++) q[b * QK + j] = (int8_t)(int)rintf(x[b * QK + j] * id);
    }
}

/* Activation row -> Q8_1 blocks (src1 of a q4_1 / q5_1 mul_mat): the Q8_0 codes and scale above,
 * plus s = d * sum(codes) with d = amax / 127 in f32, stored fp16 (ggml's x86 quantize_row_q8_1). */
void orc_act_q8_1(const float *x, int64_t n, int8_t *q, uint16_t *d, uint16_t *s) {
    orc_act_q8_0(x, n, q, d);
    for (int64_t b = 0; b < n / QK; b++) {
        float amax = 0.0f;
        int sum = 0;
        for (int j = 0; j < QK; j++) {
            const float a = fabsf(x[b * QK + j]);
            if (a > amax) amax = a;
            sum += q[b * QK + j];
        }
        s[b] = f2h((amax / 127.0f) * (float)sum);
    }
}

/* Activation row -> Q8_K super-blocks (src1 of a K-quant mul_mat; ggml quantize_row_q8_K_ref): the
 * value of largest magnitude (first on ties) sets iscale = -127 / max; codes nearest-even(iscale * x)
 * capped at 127; d = 1 / iscale in f32; bsums = sums of 16 consecutive codes. */
void orc_act_q8_K(const float *x, int64_t n, int8_t *q, float *d, int16_t *bsums) {
    for (int64_t b = 0; b < n / QKK; b++) {
        const float *xb = x + b * QKK;
        float amax = 0.0f, mx = 0.0f;
        for (int j = 0; j < QKK; j++) {
            const float a = fabsf(xb[j]);
            if (a > amax) {
                amax = a;
                mx = xb[j];
            }
        }
        if (amax == 0.0f) {
            d[b] = 0.0f;
            memset(q + b * QKK, 0, QKK);
            memset(bsums + b * 16, 0, 32);
            continue;
        }
        const float iscale = -127.0f / mx;
        for (int j = 0; j < QKK; j++) {
            const int v = (int)rintf(iscale * xb[j]);
            q[b * QKK + j] = (int8_t)(v > 127 ? 127 : v);
        }
        for (int g = 0; g < 16; g++) {
            int sum = 0;
            for (int j = 0; j < 16; j++) sum += q[b * QKK + 16 * g + j];
            bsums[b * 16 + g] = (int16_t)sum;
        }
        d[b] = 1.0f / iscale;
    }
}

/* ---------------------------------------------------------------------------------------------
 * Canonical reductions. */

static float butterfly32(float *p) {
    float t[32];
    for (int off = 16; off >= 1; off >>= 1) {
        for (int i = 0; i < 32; i++) t[i] = p[i] + p[i ^ off];
        memcpy(p, t, sizeof t);
    }
    return p[0];
}

static double tree256(double *p) {
    for (int off = 128; off >= 1; off >>= 1)
        for (int t = 0; t < off; t++) p[t] = p[t] + p[t + off];
    return p[0];
}

/* exp(x): n = rint(x log2 e), r = x - n ln2 (two-part ln2), e^r by a degree-7 Taylor polynomial in
 * Horner form, then 2^n applied as two exact power-of-two scalings. Same steps on the GPU. */
float orc_expf(float x) {
    if (x != x) return x;
    if (x > 88.72283f) return INFINITY;
    if (x < -103.972084f) return 0.0f;
    const float n = rintf(x * 1.44269504088896341f);
    float r = fmaf(n, -0.693145751953125f, x);
    r = fmaf(n, -1.428606765330187e-06f, r);
    float p = 1.98412698e-4f;          /* 1/5040 */
    p = fmaf(p, r, 1.38888889e-3f);    /* 1/720 */
    p = fmaf(p, r, 8.33333333e-3f);    /* 1/120 */
    p = fmaf(p, r, 4.16666667e-2f);    /* 1/24 */
    p = fmaf(p, r, 1.66666667e-1f);    /* 1/6 */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int ni = (int)n;
    const int a = ni / 2, b = ni - a;
    uint32_t ua = (uint32_t)(a + 127) << 23, ub = (uint32_t)(b + 127) << 23;
    float fa, fb;
    memcpy(&fa, &ua, 4);
    memcpy(&fb, &ub, 4);
    return (p * fa) * fb;
}

float orc_silu(float x) { return x / (1.0f + orc_expf(-x)); }

/* ---------------------------------------------------------------------------------------------
 * mul_mat: Y[m][n] = sum_k X[m][k] * W[n][k]. W rows are w_row_bytes apart; X rows ldx floats,
 * Y rows ldy floats. */

typedef struct {
    int wtype;
    const uint8_t *W;
    size_t wrb;
    int64_t K, M, ldy;
    const int8_t *qx;
    const uint16_t *dx;
    const float *xr;
    float *Y;
} mm_ctx;

/* Block products fma'd into the result in one of two orders (the GPU kernels follow the same):
 * up to GEMM_MIN_ROWS - 1 = 8 activation rows (decode GEMVs), block b into partial b % 32 and the
 * 32 partials reduced by the butterfly; more rows (prefill GEMMs, integer tensor-core MMA per block),
 * every block in order into one sum. */
#define GEMM_MIN_ROWS 9

static void mm_quant_rows(void *cv, int64_t n0, int64_t n1) {
    const mm_ctx *c = (const mm_ctx *)cv;
    const int64_t K = c->K, nb = K / QK;
    const int seq = c->M >= GEMM_MIN_ROWS;
    for (int64_t n = n0; n < n1; n++) {
        const uint8_t *w = c->W + (size_t)n * c->wrb;
        for (int64_t m = 0; m < c->M; m++) {
            float p[32] = {0}, acc = 0.0f;
            const int8_t *xq = c->qx + m * K;
            for (int64_t b = 0; b < nb; b++) {
                int32_t isum = 0;
                uint16_t dwh;
                if (c->wtype == ORC_Q4_0) {
                    const uint8_t *blk = w + b * 18;
                    memcpy(&dwh, blk, 2);
                    for (int j = 0; j < 16; j++) {
                        isum += ((int)(blk[2 + j] & 15) - 8) * xq[b * QK + j];
                        isum += ((int)(blk[2 + j] >> 4) - 8) * xq[b * QK + j + 16];
                    }
                } else {
                    const uint8_t *blk = w + b * 34;
                    memcpy(&dwh, blk, 2);
                    for (int j = 0; j < 32; j++) isum += (int)(int8_t)blk[2 + j] * xq[b * QK + j];
                }
                const float dd = h2f(dwh) * h2f(c->dx[m * nb + b]);
                if (seq) acc = fmaf(dd, (float)isum, acc);
                else p[b & 31] = fmaf(dd, (float)isum, p[b & 31]);
            }
            c->Y[m * c->ldy + n] = seq ? acc : butterfly32(p);
        }
    }
}

static void mm_quant(int wtype, const uint8_t *W, size_t wrb, int64_t N, int64_t K, const float *X, int64_t ldx,
                     int64_t M, float *Y, int64_t ldy) {
    const int64_t nb = K / QK;
    int8_t *qx = (int8_t *)malloc((size_t)(M * K));
    uint16_t *dx = (uint16_t *)malloc((size_t)(M * nb) * 2);
    for (int64_t m = 0; m < M; m++) orc_act_q8_0(X + m * ldx, K, qx + m * K, dx + m * nb);
    mm_ctx c = {wtype, W, wrb, K, M, ldy, qx, dx, NULL, Y};
    orc_parallel_for(N, mm_quant_rows, &c);
    free(qx);
    free(dx);
}

static void mm_float_rows(void *cv, int64_t n0, int64_t n1) {
    const mm_ctx *c = (const mm_ctx *)cv;
    const int64_t K = c->K;
    for (int64_t n = n0; n < n1; n++) {
        const uint8_t *w = c->W + (size_t)n * c->wrb;
        for (int64_t m = 0; m < c->M; m++) {
            float p[32] = {0};
            const float *x = c->xr + m * K;
            for (int64_t k = 0; k < K; k++) {
                float wv;
                if (c->wtype == ORC_F16) {
                    uint16_t h;
                    memcpy(&h, w + 2 * k, 2);
                    wv = h2f(h);
                } else {
                    memcpy(&wv, w + 4 * k, 4);
                }
                p[k & 31] = fmaf(wv, x[k], p[k & 31]);
            }
            c->Y[m * c->ldy + n] = butterfly32(p);
        }
    }
}

static void mm_float(int wtype, const uint8_t *W, size_t wrb, int64_t N, int64_t K, const float *X, int64_t ldx,
                     int64_t M, float *Y, int64_t ldy) {
    float *xr = (float *)malloc((size_t)(M * K) * 4);
    for (int64_t m = 0; m < M; m++)
        for (int64_t k = 0; k < K; k++) {
            const float v = X[m * ldx + k];
            xr[m * K + k] = wtype == ORC_F16 ? h2f(f2h(v)) : v;
        }
    mm_ctx c = {wtype, W, wrb, K, M, ldy, NULL, NULL, xr, Y};
    orc_parallel_for(N, mm_float_rows, &c);
    free(xr);
}

/* q4_1 / q5_1 / q4_K / q5_K / q6_K weights: one unit (a 32-value block, or a 256-value super-block
 * for the K-quants) per step of the lane chains: unit u into partial u % 32, then the butterfly, for
 * any number of activation rows. The integer parts are exact; the float steps per unit:
 *   q4_1, q5_1:  p = fmaf(d_w * d_x, isum, p);  p = fmaf(m_w, s_x, p)
 *   q4_K, q5_K:  p = fmaf(d_w * d_x, sum_j sc_j * isum_j, p);  p = fmaf(-(dmin_w * d_x), sum_j m_j * bsum_j, p)
 *   q6_K:        p = fmaf(d_w * d_x, sum_j sc_j * isum_j, p)
 * (d_x of a Q8_K row is f32; j runs over the 8 sub-blocks of 32, or the 16 of 16 for q6_K). ggml's
 * CPU vec_dot_{q4_1_q8_1, q5_1_q8_1, q4_K_q8_K, q5_K_q8_K, q6_K_q8_K} compute the same per-unit terms. */
typedef struct {
    int wtype;
    const uint8_t *W;
    size_t wrb;
    int64_t K, M, ldy;
    const int8_t *qx;
    const uint16_t *dx, *sx;
    const float *dk;
    const int16_t *bs;
    float *Y;
} mb_ctx;

static void mm_block_rows(void *cv, int64_t n0, int64_t n1) {
    const mb_ctx *c = (const mb_ctx *)cv;
    const int kq = c->wtype == ORC_Q4_K || c->wtype == ORC_Q5_K || c->wtype == ORC_Q6_K;
    const int64_t un = kq ? QKK : QK, nu = c->K / un;
    const size_t ub = orc_row_size(c->wtype, un);
    int codes[QKK];
    for (int64_t n = n0; n < n1; n++) {
        const uint8_t *w = c->W + (size_t)n * c->wrb;
        for (int64_t m = 0; m < c->M; m++) {
            float p[32] = {0};
            const int8_t *xq = c->qx + m * c->K;
            for (int64_t u = 0; u < nu; u++) {
                const uint8_t *blk = w + u * ub;
                const int8_t *xu = xq + u * un;
                float *pp = &p[u & 31];
                if (!kq) {
                    block_codes(c->wtype, blk, codes);
                    int32_t isum = 0;
                    for (int j = 0; j < QK; j++) isum += codes[j] * xu[j];
                    const int64_t bi = m * nu + u;
                    *pp = fmaf(blk_h(blk) * h2f(c->dx[bi]), (float)isum, *pp);
                    *pp = fmaf(blk_h(blk + 2), h2f(c->sx[bi]), *pp);
                    continue;
                }
                kq_codes(c->wtype, blk, codes);
                const float dx = c->dk[m * nu + u];
                int32_t isc = 0, imn = 0;
                if (c->wtype == ORC_Q6_K) {
                    for (int j = 0; j < 16; j++) {
                        int32_t t = 0;
                        for (int l = 0; l < 16; l++) t += codes[16 * j + l] * xu[16 * j + l];
                        isc += (int8_t)blk[192 + j] * t;
                    }
                    *pp = fmaf(blk_h(blk + 208) * dx, (float)isc, *pp);
                    continue;
                }
                const int16_t *bs = c->bs + (m * nu + u) * 16;
                for (int j = 0; j < 8; j++) {
                    int sc, mn;
                    kq_scale_min(blk + 4, j, &sc, &mn);
                    int32_t t = 0;
                    for (int l = 0; l < 32; l++) t += codes[32 * j + l] * xu[32 * j + l];
                    isc += sc * t;
                    imn += mn * (bs[2 * j] + bs[2 * j + 1]);
                }
                *pp = fmaf(blk_h(blk) * dx, (float)isc, *pp);
                *pp = fmaf(-(blk_h(blk + 2) * dx), (float)imn, *pp);
            }
            c->Y[m * c->ldy + n] = butterfly32(p);
        }
    }
}

static void mm_block(int wtype, const uint8_t *W, size_t wrb, int64_t N, int64_t K, const float *X, int64_t ldx,
                     int64_t M, float *Y, int64_t ldy) {
    const int kq = wtype == ORC_Q4_K || wtype == ORC_Q5_K || wtype == ORC_Q6_K;
    const int64_t nu = K / (kq ? QKK : QK);
    int8_t *qx = (int8_t *)malloc((size_t)(M * K));
    uint16_t *dx = (uint16_t *)malloc((size_t)(M * nu) * 2 + 2), *sx = (uint16_t *)malloc((size_t)(M * nu) * 2 + 2);
    float *dk = (float *)malloc((size_t)(M * nu) * 4 + 4);
    int16_t *bs = (int16_t *)malloc((size_t)(M * nu) * 32 + 2);
    for (int64_t m = 0; m < M; m++) {
        if (kq) orc_act_q8_K(X + m * ldx, K, qx + m * K, dk + m * nu, bs + m * nu * 16);
        else orc_act_q8_1(X + m * ldx, K, qx + m * K, dx + m * nu, sx + m * nu);
    }
    mb_ctx c = {wtype, W, wrb, K, M, ldy, qx, dx, sx, dk, bs, Y};
    orc_parallel_for(N, mm_block_rows, &c);
    free(qx);
    free(dx);
    free(sx);
    free(dk);
    free(bs);
}

/* q5_0 / iq4_nl rows -> Q8_0 rows with the same fp16 scale: ggml's vec_dot_q5_0_q8_0 and
 * vec_dot_iq4_nl_q8_0 take exactly the integer dot of these codes with the Q8_0 activation, scaled
 * by d_w * d_x, so a q5_0 / iq4_nl matmul is the Q8_0 matmul of the expanded codes. */
static uint8_t *expand_to_q8_0(int wtype, const uint8_t *W, size_t wrb, int64_t N, int64_t K) {
    const int64_t nb = K / QK;
    const size_t sb = orc_row_size(wtype, QK);
    uint8_t *out = (uint8_t *)malloc((size_t)(N * nb) * 34);
    int c[QK];
    for (int64_t n = 0; n < N; n++)
        for (int64_t b = 0; b < nb; b++) {
            const uint8_t *blk = W + (size_t)n * wrb + b * sb;
            uint8_t *o = out + (size_t)(n * nb + b) * 34;
            block_codes(wtype, blk, c);
            o[0] = blk[0];
            o[1] = blk[1];
            for (int j = 0; j < QK; j++) o[2 + j] = (uint8_t)(int8_t)c[j];
        }
    return out;
}

int orc_mul_mat(int wtype, const void *W, size_t w_row_bytes, int64_t N, int64_t K, const float *X, int64_t ldx,
                int64_t M, float *Y, int64_t ldy) {
    if (wtype == ORC_Q5_0 || wtype == ORC_IQ4_NL) {
        if (K % QK) return -1;
        uint8_t *w8 = expand_to_q8_0(wtype, (const uint8_t *)W, w_row_bytes, N, K);
        mm_quant(ORC_Q8_0, w8, (size_t)(K / QK) * 34, N, K, X, ldx, M, Y, ldy);
        free(w8);
        return 0;
    }
    if (wtype == ORC_Q4_1 || wtype == ORC_Q5_1 || wtype == ORC_Q4_K || wtype == ORC_Q5_K || wtype == ORC_Q6_K) {
        const int64_t un = (wtype == ORC_Q4_1 || wtype == ORC_Q5_1) ? QK : QKK;
        if (K % un) return -1;
        mm_block(wtype, (const uint8_t *)W, w_row_bytes, N, K, X, ldx, M, Y, ldy);
        return 0;
    }
    if (wtype == ORC_Q4_0 || wtype == ORC_Q8_0) {
        if (K % QK) return -1;
        mm_quant(wtype, (const uint8_t *)W, w_row_bytes, N, K, X, ldx, M, Y, ldy);
        return 0;
    }
    if (wtype == ORC_F32 || wtype == ORC_F16) {
        mm_float(wtype, (const uint8_t *)W, w_row_bytes, N, K, X, ldx, M, Y, ldy);
        return 0;
    }
    return -1;
}

/* ---------------------------------------------------------------------------------------------
 * Row ops. */

void orc_rms_norm(const float *x, int64_t n, float eps, float *y) {
    double p[256] = {0};
    for (int64_t i = 0; i < n; i++) p[i & 255] += (double)(x[i] * x[i]);
    const float mean = (float)(tree256(p) / (double)n);
    const float scale = 1.0f / sqrtf(mean + eps);
    for (int64_t i = 0; i < n; i++) y[i] = x[i] * scale;
}

/* y = softmax(x * scale + mask) over one row; mask f32 (nullable). */
void orc_soft_max(const float *x, const float *mask, int64_t n, float scale, float *y) {
    float mx = -INFINITY;
    for (int64_t i = 0; i < n; i++) {
        const float w = x[i] * scale + (mask ? mask[i] : 0.0f);
        y[i] = w;
        if (w > mx) mx = w;
    }
    double p[256] = {0};
    for (int64_t i = 0; i < n; i++) {
        const float e = orc_expf(y[i] - mx);
        y[i] = e;
        p[i & 255] += (double)e;
    }
    const float inv = (float)(1.0 / tree256(p));
    for (int64_t i = 0; i < n; i++) y[i] = y[i] * inv;
}

/* cos/sin table [npos][n_dims/2][2] for rope: theta starts at p and is multiplied by
 * s = powf(base, -2/n_dims) once per frequency (ggml's rope cache), times freq_scale, divided by
 * the optional frequency factors; cos and sin are scaled by attn_factor. */
void orc_rope_table(int n_dims, float freq_base, float freq_scale, float attn_factor, const float *ff, int64_t npos,
                    float *cs) {
    const float theta_scale = powf(freq_base, -2.0f / (float)n_dims);
    for (int64_t p = 0; p < npos; p++) {
        float theta = (float)p;
        for (int i = 0; i < n_dims / 2; i++) {
            const float t = freq_scale * (ff ? theta / ff[i] : theta);
            cs[(p * (n_dims / 2) + i) * 2 + 0] = cosf(t) * attn_factor;
            cs[(p * (n_dims / 2) + i) * 2 + 1] = sinf(t) * attn_factor;
            theta *= theta_scale;
        }
    }
}

/* NEOX rotation of one head row x[D] with the table row for its position. */
void orc_rope_neox(const float *x, int64_t D, int n_dims, const float *cs_row, float *y) {
    const int h = n_dims / 2;
    for (int i = 0; i < h; i++) {
        const float c = cs_row[2 * i], s = cs_row[2 * i + 1];
        const float x0 = x[i], x1 = x[i + h];
        y[i] = x0 * c - x1 * s;
        y[i + h] = x0 * s + x1 * c;
    }
    for (int64_t i = n_dims; i < D; i++) y[i] = x[i];
}

/* Dot of an f16-rounded query row with an f16 key row in the head-dot order. */
static float head_dot(const float *qh, const uint16_t *k, int64_t D) {
    float p[32] = {0};
    if (D % 32 == 0) {
        const int64_t c = D / 32;
        for (int l = 0; l < 32; l++)
            for (int64_t j = 0; j < c; j++) p[l] = fmaf(qh[l * c + j], h2f(k[l * c + j]), p[l]);
    } else {
        for (int64_t d = 0; d < D; d++) p[d & 31] = fmaf(qh[d], h2f(k[d]), p[d & 31]);
    }
    return butterfly32(p);
}

/* One query row of flash attention over n_kv keys. K/V rows are k_stride / v_stride halves
 * apart; mask is f16 per key (nullable). out[D] f32. */
void orc_flash_attn_row(const float *q, const uint16_t *K, int64_t k_stride, const uint16_t *V, int64_t v_stride,
                        int64_t n_kv, int64_t D, const uint16_t *mask, float scale, float *out) {
    float *qh = (float *)malloc((size_t)D * 4);
    float *o = (float *)malloc((size_t)D * 4);
    float *oc = (float *)malloc((size_t)D * 4);
    float s[FA_CHUNK];
    for (int64_t d = 0; d < D; d++) {
        qh[d] = h2f(f2h(q[d]));
        o[d] = 0.0f;
    }
    /* chunk maxima first: the merge weights need the overall maximum */
    const int64_t nch = (n_kv + FA_CHUNK - 1) / FA_CHUNK;
    float M = -INFINITY;
    float *mc = (float *)malloc((size_t)nch * 4);
    float *lc = (float *)malloc((size_t)nch * 4);
    float *oall = (float *)malloc((size_t)(nch * D) * 4);
    for (int64_t c = 0; c < nch; c++) {
        const int64_t j0 = c * FA_CHUNK, j1 = j0 + FA_CHUNK < n_kv ? j0 + FA_CHUNK : n_kv;
        float m = -INFINITY;
        for (int64_t j = j0; j < j1; j++) {
            float v = head_dot(qh, K + j * k_stride, D) * scale;
            v = v + (mask ? h2f(mask[j]) : 0.0f);
            s[j - j0] = v;
            if (v > m) m = v;
        }
        mc[c] = m;
        float l = 0.0f;
        for (int64_t d = 0; d < D; d++) oc[d] = 0.0f;
        if (m != -INFINITY) {
            for (int64_t j = j0; j < j1; j++) {
                const float pj = orc_expf(s[j - j0] - m);
                l = l + pj;
                const uint16_t *vr = V + j * v_stride;
                for (int64_t d = 0; d < D; d++) oc[d] = fmaf(pj, h2f(vr[d]), oc[d]);
            }
        }
        lc[c] = l;
        memcpy(oall + c * D, oc, (size_t)D * 4);
        if (m > M) M = m;
    }
    float L = 0.0f;
    for (int64_t c = 0; c < nch; c++) {
        if (mc[c] == -INFINITY) continue;
        const float w = orc_expf(mc[c] - M);
        L = fmaf(w, lc[c], L);
        for (int64_t d = 0; d < D; d++) o[d] = fmaf(w, oall[c * D + d], o[d]);
    }
    const float inv = L == 0.0f ? 0.0f : 1.0f / L;
    for (int64_t d = 0; d < D; d++) out[d] = o[d] * inv;
    free(qh);
    free(o);
    free(oc);
    free(mc);
    free(lc);
    free(oall);
}

void orc_swiglu(const float *g, const float *u, int64_t n, float *y) {
    for (int64_t i = 0; i < n; i++) y[i] = orc_silu(g[i]) * u[i];
}

int32_t orc_argmax(const float *x, int64_t n) {
    int32_t idx = 0;
    float mx = x[0];
    for (int64_t i = 1; i < n; i++) {
        if (x[i] > mx) {
            mx = x[i];
            idx = (int32_t)i;
        }
    }
    return idx;
}

int orc_version(void) { return 1; }
