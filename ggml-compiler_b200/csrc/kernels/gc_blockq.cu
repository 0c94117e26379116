// mul_mat with a weight in one of the other GGUF block formats the reference can store
// (ggml_compiler/quant/types.py:6-19), and the load-time expansion of q5_0 / iq4_nl.
//
// q5_0 and iq4_nl: ggml's CPU dots (vec_dot_q5_0_q8_0, vec_dot_iq4_nl_q8_0) are the integer dot of
// the block's signed codes (q - 16, or the iq4_nl table value) with the Q8_0 activation codes,
// scaled by d_w * d_x: exactly a Q8_0 x Q8_0 block dot. So these weights are expanded once at load
// into the Q8_0 tiled layout (same fp16 scale, codes as int8) and every Q8_0 kernel (the fused
// decode GEMVs, the tensor-core GEMV and GEMM) runs them with unchanged results.
//
// q4_1, q5_1, q4_K, q5_K, q6_K stay in their GGUF layout. Their activation rows are quantized the
// way ggml's CPU backend quantizes src1 for them (Q8_1: the Q8_0 codes and scale plus the fp16
// s = d * sum(codes); Q8_K: 256-value super-blocks with an f32 scale 1 / (-127 / max) and int16
// sums of 16 codes). A warp takes one weight row and up to 8 activation rows; for each output, unit
// u of the row (a 32-block, or a 256-value super-block) is folded into the chain of lane u % 32 in
// order of u, then the 32 chains are summed by the butterfly. The integer parts of a unit are
// exact; its float steps:
//   q4_1, q5_1:  p = fma(d_w * d_x, isum, p);  p = fma(m_w, s_x, p)
//   q4_K, q5_K:  p = fma(d_w * d_x, sum_j sc_j isum_j, p);  p = fma(-(dmin_w * d_x), sum_j m_j bsum_j, p)
//   q6_K:        p = fma(d_w * d_x, sum_j sc_j isum_j, p)
// These are the per-unit terms of ggml's vec_dot_q4_1_q8_1 ... vec_dot_q6_K_q8_K; the CPU checker
// sums them in the same order.
#include <algorithm>
#include <stdexcept>
#include <string>

#include "../gc_kernels.h"
#include "gc_blockq.cuh"
#include "gc_qweight.cuh"

namespace gcb {
namespace k {

namespace {

void check(const char *what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) throw std::runtime_error(std::string("CUDA launch of ") + what + " failed: " + cudaGetErrorString(e));
}

unsigned grid_for(int64_t threads) {
    int64_t b = (threads + 255) / 256;
    b = std::min<int64_t>(std::max<int64_t>(b, 1), 148 * 32);
    return (unsigned)b;
}

// q5_0 / iq4_nl GGUF rows -> the Q8_0 tiled layout (gc_qweight.cuh), one thread per block.
__global__ void expand_q8_0_kernel(int type, const uint8_t *raw, int64_t rows, int64_t nb, char *dst) {
    const int bs = type == T_Q5_0 ? 22 : 18;
    const QW w{dst, nb, 32};
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < rows * nb; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = t / nb, blk = t % nb;
        const uint8_t *src = raw + t * bs;
        const uint8_t *qs = src + (type == T_Q5_0 ? 6 : 2);
        const uint32_t qh = type == T_Q5_0 ? (uint32_t)src[2] | ((uint32_t)src[3] << 8) | ((uint32_t)src[4] << 16) |
                                                 ((uint32_t)src[5] << 24)
                                           : 0u;
        uint32_t words[8];
        for (int i = 0; i < 8; i++) {
            uint32_t word = 0;
            for (int b = 0; b < 4; b++) {
                const int j = 4 * i + b;  // value j
                const uint8_t byte = qs[j & 15];
                int q = j < 16 ? (byte & 15) : (byte >> 4);
                if (type == T_Q5_0) q = (q | (int)(((qh >> j) & 1u) << 4)) - 16;
                else q = iq4nl_value(q);
                word |= (uint32_t)(uint8_t)(int8_t)q << (8 * b);
            }
            words[i] = word;
        }
        char *code = (char *)qw_code(w, row, blk);
        *(uint4 *)code = make_uint4(words[0], words[1], words[2], words[3]);
        *(uint4 *)(code + 16) = make_uint4(words[4], words[5], words[6], words[7]);
        const int64_t g = blk / QSEG, sb = qw_seg_blocks(nb, g);
        uint16_t *sc = (uint16_t *)(dst + qw_piece_off(nb, 32, row / QTR, g) + QTR * sb * 32);
        sc[(row % QTR) * sb + blk % QSEG] = (uint16_t)(src[0] | (src[1] << 8));
    }
}

struct Act {  // activation rows [K, M, B2, B3] (f32, any strides) and their quantized form
    const char *b;
    int64_t K, M, B2, B3;
    int64_t bnb0, bnb1, bnb2, bnb3;
    int8_t *qx;    // [rows][K] codes
    uint16_t *dx;  // Q8_1: [rows][K/32] fp16 scales
    uint16_t *sx;  // Q8_1: [rows][K/32] fp16 d * sum(codes)
    float *dk;     // Q8_K: [rows][K/256] scales
    int16_t *bs;   // Q8_K: [rows][K/16] sums of 16 codes
};

__device__ __forceinline__ float act_x(const Act &a, int64_t r, int64_t k) {
    const int64_t m = r % a.M, i2 = (r / a.M) % a.B2, i3 = r / (a.M * a.B2);
    return *(const float *)(a.b + m * a.bnb1 + i2 * a.bnb2 + i3 * a.bnb3 + k * a.bnb0);
}

// Q8_1 (ggml's x86 quantize_row_q8_1): one warp per 32-block; d = amax / 127 (fp16), codes
// nearest-even(x * (127 / amax)), s = fp16((amax / 127) * sum(codes)).
__global__ void act_q8_1_kernel(Act a) {
    const int lane = threadIdx.x & 31;
    const int64_t nb = a.K / 32, nblk = nb * a.M * a.B2 * a.B3;
    for (int64_t w = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; w < nblk; w += ((int64_t)gridDim.x * blockDim.x) >> 5) {
        const int64_t r = w / nb, blk = w % nb;
        const float x = act_x(a, r, blk * 32 + lane);
        const float amax = warp_max(fabsf(x));
        const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
        const int q = __float2int_rn(__fmul_rn(x, id));
        a.qx[r * a.K + blk * 32 + lane] = (int8_t)q;
        const int sum = __reduce_add_sync(0xffffffffu, q);
        if (lane == 0) {
            const float d = __fdiv_rn(amax, 127.0f);
            a.dx[r * nb + blk] = f2h(d);
            a.sx[r * nb + blk] = f2h(__fmul_rn(d, __int2float_rn(sum)));
        }
    }
}

// Q8_K (ggml quantize_row_q8_K_ref): one warp per 256 values, lane l owns values 8l .. 8l + 7. The
// value of largest magnitude (first on ties) sets iscale = -127 / max; codes min(127,
// nearest-even(iscale * x)); d = 1 / iscale; an all-zero super-block gets d = 0 and zero codes.
__global__ void act_q8_K_kernel(Act a) {
    const int lane = threadIdx.x & 31;
    const int64_t nsb = a.K / 256, n = nsb * a.M * a.B2 * a.B3;
    for (int64_t w = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; w < n; w += ((int64_t)gridDim.x * blockDim.x) >> 5) {
        const int64_t r = w / nsb, sb = w % nsb;
        float x[8], amax = 0.0f, mx = 0.0f;
        for (int i = 0; i < 8; i++) {
            x[i] = act_x(a, r, sb * 256 + lane * 8 + i);
            if (fabsf(x[i]) > amax) {
                amax = fabsf(x[i]);
                mx = x[i];
            }
        }
        int at = lane;  // the winning lane: larger magnitude, the lower lane (earlier values) on ties
        for (int off = 16; off >= 1; off >>= 1) {
            const float oa = __shfl_xor_sync(0xffffffffu, amax, off), om = __shfl_xor_sync(0xffffffffu, mx, off);
            const int ol = __shfl_xor_sync(0xffffffffu, at, off);
            if (oa > amax || (oa == amax && ol < at)) {
                amax = oa;
                mx = om;
                at = ol;
            }
        }
        int8_t *q = a.qx + r * a.K + sb * 256 + lane * 8;
        int sum = 0;
        if (amax == 0.0f) {
            for (int i = 0; i < 8; i++) q[i] = 0;
        } else {
            const float iscale = __fdiv_rn(-127.0f, mx);
            for (int i = 0; i < 8; i++) {
                const int v = min(127, __float2int_rn(__fmul_rn(iscale, x[i])));
                q[i] = (int8_t)v;
                sum += v;
            }
            if (lane == 0) a.dk[r * nsb + sb] = __fdiv_rn(1.0f, iscale);
        }
        if (amax == 0.0f && lane == 0) a.dk[r * nsb + sb] = 0.0f;
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        if ((lane & 1) == 0) a.bs[r * (a.K / 16) + sb * 16 + lane / 2] = (int16_t)sum;
    }
}

struct MMb {
    const char *a;
    int64_t anb1, anb2, anb3;
    int64_t K, N, A2, A3, M, B2, B3;
    Act x;
    float *out;
};

// Integer dot of 32 unsigned 4/5-bit codes (4 words of low values 0..15, 4 of high values 16..31,
// already carrying bit 4) with 32 activation codes.
__device__ __forceinline__ int dot32(const uint32_t *lo, const uint32_t *hi, const int8_t *x) {
    const int4 xa = *(const int4 *)x, xb = *(const int4 *)(x + 16);
    int s = __dp4a((int)lo[0], xa.x, 0);
    s = __dp4a((int)lo[1], xa.y, s);
    s = __dp4a((int)lo[2], xa.z, s);
    s = __dp4a((int)lo[3], xa.w, s);
    s = __dp4a((int)hi[0], xb.x, s);
    s = __dp4a((int)hi[1], xb.y, s);
    s = __dp4a((int)hi[2], xb.z, s);
    return __dp4a((int)hi[3], xb.w, s);
}

constexpr int KQ_ROWS = 8;  // activation rows a warp takes at once (the weight codes stay in registers)

// q4_1 / q5_1: a warp takes one weight row and up to KQ_ROWS activation rows of one batch index;
// lane u owns blocks u, u + 32, ... (the chain of block u % 32) and decodes each block's codes once
// for every activation row.
template <int T, int R>
__global__ void mm_q1_kernel(MMb p) {
    constexpr int UB = T == T_Q4_1 ? 20 : 24;
    const int lane = threadIdx.x & 31;
    const int64_t nu = p.K / 32;
    const int64_t mgroups = (p.M + R - 1) / R;
    const int64_t ntask = p.N * mgroups * p.B2 * p.B3;
    for (int64_t w = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; w < ntask; w += ((int64_t)gridDim.x * blockDim.x) >> 5) {
        const int64_t n = w % p.N;
        int64_t t = w / p.N;
        const int64_t mg = t % mgroups;
        t /= mgroups;
        const int64_t i2 = t % p.B2, i3 = t / p.B2;
        const int64_t a2 = i2 / (p.B2 / p.A2), a3 = i3 / (p.B3 / p.A3);
        const uint8_t *row = (const uint8_t *)(p.a + n * p.anb1 + a2 * p.anb2 + a3 * p.anb3);
        const int m0 = (int)(mg * R);
        const int mr = (int)(p.M - m0 < R ? p.M - m0 : R);
        const int64_t r0 = m0 + p.M * (i2 + p.B2 * i3);
        float acc[R];
#pragma unroll
        for (int k = 0; k < R; k++) acc[k] = 0.0f;
        for (int64_t u = lane; u < nu; u += 32) {
            const uint8_t *blk = row + u * UB;
            const uint8_t *qs = blk + (T == T_Q4_1 ? 4 : 8);
            uint32_t lo[4], hi[4];
            const uint32_t qh = T == T_Q5_1 ? ld32(blk + 4) : 0u;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint32_t v = ld32(qs + 4 * i);
                lo[i] = (v & 0x0f0f0f0fu) | spread4((qh >> (4 * i)) & 15u);
                hi[i] = ((v >> 4) & 0x0f0f0f0fu) | spread4((qh >> (16 + 4 * i)) & 15u);
            }
            const float dw = h2f((uint16_t)ld16(blk)), mw = h2f((uint16_t)ld16(blk + 2));
#pragma unroll
            for (int k = 0; k < R; k++) {
                if (k >= mr) break;
                const int64_t r = r0 + k, bi = r * nu + u;
                const int isum = dot32(lo, hi, p.x.qx + r * p.K + u * 32);
                acc[k] = __fmaf_rn(__fmul_rn(dw, h2f(p.x.dx[bi])), __int2float_rn(isum), acc[k]);
                acc[k] = __fmaf_rn(mw, h2f(p.x.sx[bi]), acc[k]);
            }
        }
#pragma unroll
        for (int k = 0; k < R; k++) {
            if (k >= mr) break;
            const float v = warp_butterfly(acc[k]);
            if (lane == 0) p.out[(r0 + k) * p.N + n] = v;
        }
    }
}

// K-quants, sub-block parallel: a warp takes KQ_WR weight rows and up to KQ_ROWS activation rows of
// one batch index; in step i its four 8-lane groups take super-blocks 4i .. 4i + 3, lane (g, j)
// sub-block j of super-block 4i + g (32 values; for q6_K its two 16-value sub-blocks). The codes
// stay in registers for every activation row. The 8 lanes' integer parts are summed exactly by
// shuffles, and super-block s is folded into the chain of lane s % 32.

// One lane's share of one super-block: its 32 codes (value order; signed bytes for q6_K), its
// sub-block scales (q6_K: two int8 scales; q4_K/q5_K: 6-bit scale and min) and the fp16 d / dmin.
struct KqPart {
    uint32_t c[8];
    int sc0, sc1, mn;
    uint32_t dh, mh;
};

template <int T>
__device__ __forceinline__ void kq_load(KqPart &k, const uint8_t *row, int64_t s, int64_t nu, int sub) {
    constexpr int UB = T == T_Q4_K ? 144 : T == T_Q5_K ? 176 : 210;
    k.sc0 = k.sc1 = k.mn = 0;
    k.dh = k.mh = 0;
    if (s >= nu) {
#pragma unroll
        for (int i = 0; i < 8; i++) k.c[i] = 0;
        return;
    }
    const uint8_t *blk = row + s * UB;
    if constexpr (T == T_Q6_K) {
        const int h = sub / 4, r = 32 * (sub % 4);  // values 32 sub .. 32 sub + 31
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int r4 = r + 4 * i;
            const uint32_t ql = ld32a2(blk + 64 * h + r4 % 64), qh = ld32a2(blk + 128 + 32 * h + r4 % 32);
            k.c[i] = __vsub4(((ql >> (4 * (r4 / 64))) & 0x0f0f0f0fu) | (((qh >> (2 * (r4 / 32))) & 0x03030303u) << 4),
                             0x20202020u);
        }
        k.sc0 = (int8_t)blk[192 + 2 * sub];
        k.sc1 = (int8_t)blk[193 + 2 * sub];
        k.dh = ld16(blk + 208);
    } else {
        const uint4 *qs = (const uint4 *)(blk + (T == T_Q4_K ? 16 : 48) + 32 * (sub / 2));  // 16-byte aligned
        const uint4 q0 = qs[0], q1 = qs[1];
        const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        uint32_t hb[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if constexpr (T == T_Q5_K) {
            const uint4 h0 = ((const uint4 *)(blk + 16))[0], h1 = ((const uint4 *)(blk + 16))[1];
            const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
            for (int i = 0; i < 8; i++) hb[i] = ((hw[i] >> sub) & 0x01010101u) << 4;
        }
#pragma unroll
        for (int i = 0; i < 8; i++) k.c[i] = ((w[i] >> (4 * (sub % 2))) & 0x0f0f0f0fu) | hb[i];
        kq_scale_min(blk + 4, sub, k.sc0, k.mn);
        k.dh = ld16(blk);
        k.mh = ld16(blk + 2);
    }
}

// Folds super-blocks s0 .. s0 + 3 (lane group g holds s0 + g) of KQ_WR weight rows into their
// chains, for every activation row: each activation code slice is loaded once for the KQ_WR rows;
// the 8 lanes' integer parts are summed by shuffles, then super-block s goes into lane s % 32's
// chain.
constexpr int KQ_WR = 2;  // weight rows per warp

template <int T, int R>
__device__ __forceinline__ void kq_fold(const KqPart *k, const MMb &p, int64_t s0, int64_t nu, int lane, int mr,
                                        int64_t r0, float (*acc)[R]) {
    const int sub = lane & 7;
    const int64_t s = s0 + (lane >> 3);
    const bool have = s < nu;
    const int base = (int)(s0 & 31), g2 = lane - base;
    const bool mine = g2 >= 0 && g2 < 4 && s0 + g2 < nu;  // lane owns the chain of super-block s0 + g2
    const int src = (mine ? g2 : 0) * 8;
#pragma unroll
    for (int m = 0; m < R; m++) {
        if (m >= mr) break;  // mr is the same on every lane
        const int64_t r = r0 + m;
        int isc[KQ_WR], imn[KQ_WR];
        float dx = 0.0f;
        int4 xa = make_int4(0, 0, 0, 0), xb = xa;
        int bsum = 0;
        if (have) {
            const int8_t *xu = p.x.qx + r * p.K + s * 256 + 32 * sub;
            xa = *(const int4 *)xu;
            xb = *(const int4 *)(xu + 16);
            dx = p.x.dk[r * nu + s];
            if constexpr (T != T_Q6_K) {
                const int16_t *bs = p.x.bs + (r * nu + s) * 16;
                bsum = (int)bs[2 * sub] + (int)bs[2 * sub + 1];
            }
        }
#pragma unroll
        for (int w = 0; w < KQ_WR; w++) {
            const uint32_t *c = k[w].c;
            int t0 = __dp4a((int)c[0], xa.x, 0);
            t0 = __dp4a((int)c[1], xa.y, t0);
            t0 = __dp4a((int)c[2], xa.z, t0);
            t0 = __dp4a((int)c[3], xa.w, t0);
            int t1 = __dp4a((int)c[4], xb.x, 0);
            t1 = __dp4a((int)c[5], xb.y, t1);
            t1 = __dp4a((int)c[6], xb.z, t1);
            t1 = __dp4a((int)c[7], xb.w, t1);
            isc[w] = T == T_Q6_K ? k[w].sc0 * t0 + k[w].sc1 * t1 : k[w].sc0 * (t0 + t1);
            imn[w] = k[w].mn * bsum;
            isc[w] += __shfl_xor_sync(0xffffffffu, isc[w], 1);
            isc[w] += __shfl_xor_sync(0xffffffffu, isc[w], 2);
            isc[w] += __shfl_xor_sync(0xffffffffu, isc[w], 4);
            if constexpr (T != T_Q6_K) {
                imn[w] += __shfl_xor_sync(0xffffffffu, imn[w], 1);
                imn[w] += __shfl_xor_sync(0xffffffffu, imn[w], 2);
                imn[w] += __shfl_xor_sync(0xffffffffu, imn[w], 4);
            }
        }
        const float vdx = __shfl_sync(0xffffffffu, dx, src);
#pragma unroll
        for (int w = 0; w < KQ_WR; w++) {
            const int visc = __shfl_sync(0xffffffffu, isc[w], src), vimn = __shfl_sync(0xffffffffu, imn[w], src);
            const uint16_t vdh = (uint16_t)__shfl_sync(0xffffffffu, k[w].dh, src);
            const uint16_t vmh = (uint16_t)__shfl_sync(0xffffffffu, k[w].mh, src);
            if (mine) {
                acc[w][m] = __fmaf_rn(__fmul_rn(h2f(vdh), vdx), __int2float_rn(visc), acc[w][m]);
                if constexpr (T != T_Q6_K)
                    acc[w][m] = __fmaf_rn(-__fmul_rn(h2f(vmh), vdx), __int2float_rn(vimn), acc[w][m]);
            }
        }
    }
}

template <int T, int R>
__global__ void mm_kq_kernel(MMb p) {
    constexpr int UB = T == T_Q4_K ? 144 : T == T_Q5_K ? 176 : 210;
    const int lane = threadIdx.x & 31, sub = lane & 7, grp = lane >> 3;
    const int64_t nu = p.K / 256;
    const int64_t npair = (p.N + KQ_WR - 1) / KQ_WR;
    const int64_t mgroups = (p.M + R - 1) / R;
    const int64_t ntask = npair * mgroups * p.B2 * p.B3;
    for (int64_t w = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; w < ntask; w += ((int64_t)gridDim.x * blockDim.x) >> 5) {
        const int64_t n0 = (w % npair) * KQ_WR;
        int64_t t = w / npair;
        const int64_t mg = t % mgroups;
        t /= mgroups;
        const int64_t i2 = t % p.B2, i3 = t / p.B2;
        const int64_t a2 = i2 / (p.B2 / p.A2), a3 = i3 / (p.B3 / p.A3);
        const uint8_t *rows[KQ_WR];
        int64_t ulim[KQ_WR];  // super-blocks to load from each weight row (0 past the last row)
#pragma unroll
        for (int r = 0; r < KQ_WR; r++) {
            const int64_t n = n0 + r < p.N ? n0 + r : n0;
            rows[r] = (const uint8_t *)(p.a + n * p.anb1 + a2 * p.anb2 + a3 * p.anb3);
            ulim[r] = n0 + r < p.N ? nu : 0;
        }
        const int m0 = (int)(mg * R);
        const int mr = (int)(p.M - m0 < R ? p.M - m0 : R);
        const int64_t r0 = m0 + p.M * (i2 + p.B2 * i3);  // activation row index of m0
        float acc[KQ_WR][R];
#pragma unroll
        for (int r = 0; r < KQ_WR; r++)
#pragma unroll
            for (int k = 0; k < R; k++) acc[r][k] = 0.0f;
        for (int64_t s0 = 0; s0 < nu; s0 += 4) {
            KqPart parts[KQ_WR];
#pragma unroll
            for (int r = 0; r < KQ_WR; r++) kq_load<T>(parts[r], rows[r], s0 + grp, ulim[r], sub);
            kq_fold<T, R>(parts, p, s0, nu, lane, mr, r0, acc);
        }
        (void)UB;
#pragma unroll
        for (int r = 0; r < KQ_WR; r++) {
            if (n0 + r >= p.N) break;
#pragma unroll
            for (int k = 0; k < R; k++) {
                if (k >= mr) break;
                const float v = warp_butterfly(acc[r][k]);
                if (lane == 0) p.out[(r0 + k) * p.N + n0 + r] = v;
            }
        }
    }
}

bool k_quant(Type t) { return t == T_Q4_K || t == T_Q5_K || t == T_Q6_K; }

}  // namespace

bool raw_block_type(Type t) { return t == T_Q4_1 || t == T_Q5_1 || k_quant(t); }
bool expands_to_q8_0(Type t) { return t == T_Q5_0 || t == T_IQ4_NL; }

void expand_to_q8_0(Type t, const uint8_t *raw, int64_t nrows, int64_t K, char *dst, cudaStream_t s) {
    if (!expands_to_q8_0(t) || K % 32) throw std::runtime_error("expand_to_q8_0: not a q5_0 / iq4_nl row set");
    expand_q8_0_kernel<<<grid_for(nrows * (K / 32)), 256, 0, s>>>((int)t, raw, nrows, K / 32, dst);
    check("expand_q8_0");
}

size_t mul_mat_block_scratch_bytes(const TD &a, const TD &b) {
    const int64_t rows = b.ne[1] * b.ne[2] * b.ne[3], K = a.ne[0];
    const size_t q = ((size_t)(rows * K) + 255) / 256 * 256;
    if (k_quant(a.type)) return q + ((size_t)(rows * (K / 256)) * 4 + 255) / 256 * 256 + (size_t)(rows * (K / 16)) * 2 + 256;
    return q + 2 * (((size_t)(rows * (K / 32)) * 2 + 255) / 256 * 256) + 256;
}

void mul_mat_block(const TD &a, const TD &b, const TD &out, void *scratch, cudaStream_t s) {
    const int un = k_quant(a.type) ? 256 : 32;
    if (!raw_block_type(a.type) || a.ne[0] % un) throw std::runtime_error("mul_mat_block: unsupported weight");
    MMb p{};
    p.a = a.data;
    p.anb1 = a.nb[1], p.anb2 = a.nb[2], p.anb3 = a.nb[3];
    p.K = a.ne[0], p.N = a.ne[1], p.A2 = a.ne[2], p.A3 = a.ne[3];
    p.M = b.ne[1], p.B2 = b.ne[2], p.B3 = b.ne[3];
    Act &x = p.x;
    x.b = b.data;
    x.K = p.K, x.M = p.M, x.B2 = p.B2, x.B3 = p.B3;
    x.bnb0 = b.nb[0], x.bnb1 = b.nb[1], x.bnb2 = b.nb[2], x.bnb3 = b.nb[3];
    const int64_t rows = p.M * p.B2 * p.B3;
    char *sp = (char *)scratch;
    x.qx = (int8_t *)sp;
    sp += ((size_t)(rows * p.K) + 255) / 256 * 256;
    if (k_quant(a.type)) {
        x.dk = (float *)sp;
        sp += ((size_t)(rows * (p.K / 256)) * 4 + 255) / 256 * 256;
        x.bs = (int16_t *)sp;
        act_q8_K_kernel<<<grid_for(rows * (p.K / 256) * 32), 256, 0, s>>>(x);
    } else {
        x.dx = (uint16_t *)sp;
        sp += ((size_t)(rows * (p.K / 32)) * 2 + 255) / 256 * 256;
        x.sx = (uint16_t *)sp;
        act_q8_1_kernel<<<grid_for(rows * (p.K / 32) * 32), 256, 0, s>>>(x);
    }
    check("act_q8_1 / act_q8_K");
    p.out = (float *)out.data;
    // one activation row (decode): kernels sized for it; more: KQ_ROWS rows per warp
    const int R = p.M == 1 ? 1 : KQ_ROWS;
    const unsigned gk = grid_for(p.N * ((p.M + R - 1) / R) * p.B2 * p.B3 * 32);
    const unsigned gkq = grid_for((p.N + KQ_WR - 1) / KQ_WR * ((p.M + R - 1) / R) * p.B2 * p.B3 * 32);
#define GCB_BLOCKQ_LAUNCH(RR)                                                      \
    switch (a.type) {                                                              \
        case T_Q4_1: mm_q1_kernel<T_Q4_1, RR><<<gk, 256, 0, s>>>(p); break;        \
        case T_Q5_1: mm_q1_kernel<T_Q5_1, RR><<<gk, 256, 0, s>>>(p); break;        \
        case T_Q4_K: mm_kq_kernel<T_Q4_K, RR><<<gkq, 256, 0, s>>>(p); break;       \
        case T_Q5_K: mm_kq_kernel<T_Q5_K, RR><<<gkq, 256, 0, s>>>(p); break;       \
        default: mm_kq_kernel<T_Q6_K, RR><<<gkq, 256, 0, s>>>(p); break;           \
    }
    if (R == 1) {
        GCB_BLOCKQ_LAUNCH(1)
    } else {
        GCB_BLOCKQ_LAUNCH(KQ_ROWS)
    }
#undef GCB_BLOCKQ_LAUNCH
    check("mul_mat_block");
}

}  // namespace k
}  // namespace gcb
