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

enum { ORC_F32 = 0, ORC_F16 = 1, ORC_Q4_0 = 2, ORC_Q8_0 = 8 };

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

size_t orc_row_size(int type, int64_t n) {
    switch (type) {
        case ORC_F32: return (size_t)n * 4;
        case ORC_F16: return (size_t)n * 2;
        case ORC_Q4_0: return (size_t)(n / QK) * 18;
        case ORC_Q8_0: return (size_t)(n / QK) * 34;
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
        if (q->type == ORC_Q8_0) quant_q8_0_row(q->src + r * q->n, q->dst + r * q->rb, q->n);
        else if (q->type == ORC_Q4_0) quant_q4_0_row(q->src + r * q->n, q->dst + r * q->rb, q->n);
    }
}

size_t orc_quantize(int type, const float *src, int64_t nrows, int64_t n, uint8_t *dst) {
    const size_t rb = orc_row_size(type, n);
    if (rb == 0 || n % QK || (type != ORC_Q8_0 && type != ORC_Q4_0)) return 0;
    quant_ctx c = {type, src, n, dst, rb};
    orc_parallel_for(nrows, quant_rows, &c);
    return rb * (size_t)nrows;
}

void orc_dequantize(int type, const uint8_t *src, int64_t nrows, int64_t n, float *dst) {
    const size_t rb = orc_row_size(type, n);
    for (int64_t r = 0; r < nrows; r++) {
        const uint8_t *x = src + r * rb;
        float *y = dst + r * n;
        for (int64_t b = 0; b < n / QK; b++) {
            if (type == ORC_Q8_0) {
                uint16_t dh;
                memcpy(&dh, x + b * 34, 2);
                const float d = h2f(dh);
                for (int j = 0; j < QK; j++) y[b * QK + j] = d * (float)(int8_t)x[b * 34 + 2 + j];
            } else {
                uint16_t dh;
                memcpy(&dh, x + b * 18, 2);
                const float d = h2f(dh);
                for (int j = 0; j < QK / 2; j++) {
                    const uint8_t v = x[b * 18 + 2 + j];
                    y[b * QK + j] = d * (float)((int)(v & 15) - 8);
                    y[b * QK + j + 16] = d * (float)((int)(v >> 4) - 8);
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

int orc_mul_mat(int wtype, const void *W, size_t w_row_bytes, int64_t N, int64_t K, const float *X, int64_t ldx,
                int64_t M, float *Y, int64_t ldy) {
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
