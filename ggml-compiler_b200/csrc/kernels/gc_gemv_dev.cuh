// Device building blocks of the streamed quantized GEMV, shared by the per-op kernel (gc_fused.cu)
// and the per-token decode kernel (gc_mega.cu).
//
// Weights stream as pieces (one 8-row tile x one 128-block segment each, gc_qweight.cuh) through a
// ring of NS shared-memory slots: the producer lane puts piece t in slot t % NS after the slot's
// previous piece was released (empty barrier) and arms full[t % NS] with the byte count; the team of
// 8 consumer warps owning that piece waits on full, computes and releases. A CTA's pieces are
// numbered in the order (phase, local group, segment, piece of the group), which producer and
// consumers both derive from the same geometry.
//
// Arithmetic is the CPU checker's: the activation row -> Q8_0 blocks (d = amax/127 in fp16,
// codes = nearest-even(x * 127/amax)), lane l owns blocks l, l+32, ... of a row (segments are
// multiples of 32 blocks, walked in order), acc = fma(d_w * d_x, isum, acc) with the exact integer
// dot, then the 32-lane butterfly.
#pragma once

#include "../gc_fused.h"
#include "gc_math.cuh"
#include "gc_qweight.cuh"
#include "gc_tma.cuh"

namespace gcb {
namespace k {

constexpr int GEMV_MAXM = 8;

// Geometry of one GEMV over the tiled weights.
struct GemvGeo {
    int64_t nb, nseg, groups;  // blocks per row, segments per row, row groups (tiles / tile pairs)
    int cb, pieces;            // code bytes per block, pieces per (group, segment)
    int64_t half_tiles;        // ROPE_QKV: tiles per half head
};

__host__ __device__ inline GemvGeo gemv_geo(const FusedArgs &a) {
    GemvGeo G{};
    G.nb = a.K / 32;
    G.nseg = qw_nseg(G.nb);
    G.cb = a.qtype == T_Q4_0 ? 16 : 32;
    if (a.map == MAP_SINGLE) {
        G.groups = (a.wrows[0] + QTR - 1) / QTR;
        G.pieces = 1;
    } else if (a.map == MAP_SWIGLU) {
        G.groups = (a.wrows[0] + QTR - 1) / QTR;
        G.pieces = 2;
    } else {
        G.half_tiles = (a.D / 2) / QTR;
        G.groups = (a.H + 2 * a.Hkv) * G.half_tiles;
        G.pieces = 2;
    }
    return G;
}

// Groups of a GEMV handled by CTA `cta` of `nctas` (groups cta, cta + nctas, ...).
__host__ __device__ inline int64_t local_groups(int64_t groups, int64_t cta, int64_t nctas) {
    return cta < groups ? (groups - cta + nctas - 1) / nctas : 0;
}

// Source of piece r (0/1) of group g, segment s; the matrix and the tile of piece r.
__device__ __forceinline__ const char *gemv_piece(const FusedArgs &a, const GemvGeo &G, int64_t g, int r, int64_t s,
                                                  int *mat, int64_t *tile) {
    int m = 0;
    int64_t t;
    if (a.map == MAP_SINGLE) {
        t = g;
    } else if (a.map == MAP_SWIGLU) {
        m = r;
        t = g;
    } else {
        const int64_t head = g / G.half_tiles, p = g % G.half_tiles;
        int64_t h;
        if (head < a.H) {
            m = 0;
            h = head;
        } else if (head < a.H + a.Hkv) {
            m = 1;
            h = head - a.H;
        } else {
            m = 2;
            h = head - a.H - a.Hkv;
        }
        t = h * (a.D / QTR) + p + r * G.half_tiles;
    }
    *mat = m;
    *tile = t;
    return a.wc[m] + qw_piece_off(G.nb, G.cb, t, s);
}

struct Ring {
    uint64_t *full, *empty;
    unsigned char *slots;
    int ns;
    int64_t slot_bytes;
};

// Producer: put this CTA's pieces of one GEMV into the ring, continuing the piece count `t`.
// Returns false if a slot was never released (bounded wait).
__device__ inline bool produce_gemv(const FusedArgs &a, const GemvGeo &G, const Ring &R, int64_t &t, int64_t cta,
                                    int64_t nctas) {
    for (int64_t g = cta; g < G.groups; g += nctas) {
        for (int64_t s = 0; s < G.nseg; s++) {
            const uint32_t pb = (uint32_t)qw_piece_bytes(G.nb, G.cb, s);
            for (int r = 0; r < G.pieces; r++, t++) {
                const int slot = (int)(t % R.ns);
                if (t >= R.ns && !mbar_wait(&R.empty[slot], (uint32_t)(((t / R.ns) - 1) & 1))) return false;
                mbar_expect_tx(&R.full[slot], pb);
                int mat;
                int64_t tile;
                bulk_g2s(R.slots + slot * R.slot_bytes, gemv_piece(a, G, g, r, s, &mat, &tile), pb, &R.full[slot]);
            }
        }
    }
    return true;
}

// Activation row(s) -> Q8_0 blocks in shared memory (sq codes, sdf scales as f32, ss8 8 x code sums),
// with rms_norm * w first for PRO_NORM. Run by the NCT consumer threads (thread ids 0 .. NCT-1);
// `bar` is their named barrier. The sum of squares uses the 256-partial double tree (threads 0..255).
template <int M, int NCT>
__device__ inline void gemv_prologue(const FusedArgs &a, int8_t *sq, float *sdf, int *ss8, double *red, int bar) {
    const int64_t K = a.K, nb = K / 32;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    constexpr int NW = NCT / 32;
#pragma unroll
    for (int m = 0; m < M; m++) {
        const float *x = a.x + m * a.ldx;
        float scale = 1.0f;
        if (a.pro == PRO_NORM) {
            double p = 0.0;
            if (tid < 256)
                for (int64_t i = tid; i < K; i += 256) p = __dadd_rn(p, (double)__fmul_rn(x[i], x[i]));
            if (tid < 256) red[tid] = p;
            named_bar(bar, NCT);
#pragma unroll
            for (int off = 128; off >= 1; off >>= 1) {
                if (tid < off) red[tid] = __dadd_rn(red[tid], red[tid + off]);
                named_bar(bar, NCT);
            }
            const double tot = red[0];
            named_bar(bar, NCT);
            const float mean = __double2float_rn(__ddiv_rn(tot, (double)K));
            scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
        }
        const int sub = lane >> 3, e = (lane & 7) * 4;
        for (int64_t b0 = (int64_t)warp * 4; b0 < nb; b0 += NW * 4) {
            const int64_t b = b0 + sub;
            const bool ok = b < nb;
            float4 v = ok ? *(const float4 *)(x + b * 32 + e) : make_float4(0.f, 0.f, 0.f, 0.f);
            if (a.pro == PRO_NORM && ok) {
                const float4 w = *(const float4 *)(a.norm_w + b * 32 + e);
                v.x = __fmul_rn(__fmul_rn(v.x, scale), w.x);
                v.y = __fmul_rn(__fmul_rn(v.y, scale), w.y);
                v.z = __fmul_rn(__fmul_rn(v.z, scale), w.z);
                v.w = __fmul_rn(__fmul_rn(v.w, scale), w.w);
            }
            float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
            for (int off = 4; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
            const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
            const int q0 = __float2int_rn(__fmul_rn(v.x, id)), q1 = __float2int_rn(__fmul_rn(v.y, id));
            const int q2 = __float2int_rn(__fmul_rn(v.z, id)), q3 = __float2int_rn(__fmul_rn(v.w, id));
            int sum = q0 + q1 + q2 + q3;
#pragma unroll
            for (int off = 4; off >= 1; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
            if (ok) {
                *(uint32_t *)(sq + (size_t)m * K + b * 32 + e) =
                    (uint32_t)(q0 & 255) | ((uint32_t)(q1 & 255) << 8) | ((uint32_t)(q2 & 255) << 16) | ((uint32_t)(q3 & 255) << 24);
                if ((lane & 7) == 0) {
                    sdf[m * nb + b] = h2f(f2h(__fdiv_rn(amax, 127.0f)));
                    ss8[m * nb + b] = 8 * sum;
                }
            }
        }
    }
    named_bar(bar, NCT);
}

// One quantized block of this lane's row against every activation row.
template <int QT, int NR, int M>
__device__ __forceinline__ void gemv_block(float (&acc)[NR][M], int r, const unsigned char *codes, const uint16_t *scl, int j,
                                           int b, const int8_t *sq, const float *sdf, const int *ss8, int64_t K, int64_t nb) {
    const float dw = h2f(scl[j]);
    if (QT == 0) {
        const uint4 w = *(const uint4 *)(codes + j * 16);
#pragma unroll
        for (int m = 0; m < M; m++) {
            const int4 *x4 = (const int4 *)(sq + m * K + b * 32);
            const int4 xa = x4[0], xb = x4[1];
            int v = 0;
            v = __dp4a((int)(w.x & 0x0f0f0f0fu), xa.x, v);
            v = __dp4a((int)((w.x >> 4) & 0x0f0f0f0fu), xb.x, v);
            v = __dp4a((int)(w.y & 0x0f0f0f0fu), xa.y, v);
            v = __dp4a((int)((w.y >> 4) & 0x0f0f0f0fu), xb.y, v);
            v = __dp4a((int)(w.z & 0x0f0f0f0fu), xa.z, v);
            v = __dp4a((int)((w.z >> 4) & 0x0f0f0f0fu), xb.z, v);
            v = __dp4a((int)(w.w & 0x0f0f0f0fu), xa.w, v);
            v = __dp4a((int)((w.w >> 4) & 0x0f0f0f0fu), xb.w, v);
            v -= ss8[m * nb + b];
            acc[r][m] = __fmaf_rn(__fmul_rn(dw, sdf[m * nb + b]), (float)v, acc[r][m]);
        }
    } else {
        const int4 w0 = *(const int4 *)(codes + j * 32), w1 = *(const int4 *)(codes + j * 32 + 16);
#pragma unroll
        for (int m = 0; m < M; m++) {
            const int4 *x4 = (const int4 *)(sq + m * K + b * 32);
            const int4 xa = x4[0], xb = x4[1];
            int v = 0;
            v = __dp4a(w0.x, xa.x, v);
            v = __dp4a(w0.y, xa.y, v);
            v = __dp4a(w0.z, xa.z, v);
            v = __dp4a(w0.w, xa.w, v);
            v = __dp4a(w1.x, xb.x, v);
            v = __dp4a(w1.y, xb.y, v);
            v = __dp4a(w1.z, xb.z, v);
            v = __dp4a(w1.w, xb.w, v);
            acc[r][m] = __fmaf_rn(__fmul_rn(dw, sdf[m * nb + b]), (float)v, acc[r][m]);
        }
    }
}

// Consumer side of one GEMV: this team's groups (every `teams`-th local group, starting at `team`),
// pieces numbered from t0, then the epilogue. `wt` is the warp index within the team (the row of
// the tile it owns). Returns false on a timed-out wait.
template <int QT, int NR, int M>
__device__ inline bool consume_gemv(const FusedArgs &a, const GemvGeo &G, const Ring &R, int64_t t0, int64_t cta,
                                    int64_t nctas, int team, int teams, int wt, const int8_t *sq, const float *sdf,
                                    const int *ss8) {
    constexpr int CB = QT == 0 ? 16 : 32;
    const int lane = threadIdx.x & 31;
    const int64_t K = a.K, nb = G.nb;
    const int64_t per_group = G.nseg * G.pieces;
    int64_t gl = 0;
    for (int64_t g = cta; g < G.groups; g += nctas, gl++) {
        if (gl % teams != team) continue;
        float acc[NR][M];
#pragma unroll
        for (int r = 0; r < NR; r++)
#pragma unroll
            for (int m = 0; m < M; m++) acc[r][m] = 0.0f;
        int64_t t = t0 + gl * per_group;
        for (int64_t s = 0; s < G.nseg; s++) {
            const int sb = (int)qw_seg_blocks(nb, s);
            const int bbase = (int)(s * QSEG);
#pragma unroll
            for (int r = 0; r < NR; r++, t++) {
                const int slot = (int)(t % R.ns);
                int ready = 1;
                if (lane == 0) ready = mbar_wait(&R.full[slot], (uint32_t)((t / R.ns) & 1)) ? 1 : 0;
                if (!__shfl_sync(0xffffffffu, ready, 0)) return false;  // uniform within the warp
                const unsigned char *piece = R.slots + slot * R.slot_bytes;
                const unsigned char *codes = piece + wt * sb * CB;
                const uint16_t *scl = (const uint16_t *)(piece + QTR * sb * CB) + wt * sb;
                if (sb == QSEG) {
#pragma unroll
                    for (int i = 0; i < QSEG / 32; i++)
                        gemv_block<QT, NR, M>(acc, r, codes, scl, lane + 32 * i, bbase + lane + 32 * i, sq, sdf, ss8, K, nb);
                } else {
                    for (int j = lane; j < sb; j += 32) gemv_block<QT, NR, M>(acc, r, codes, scl, j, bbase + j, sq, sdf, ss8, K, nb);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&R.empty[slot]);
            }
        }
        // epilogue for this warp's row(s)
        int mat;
        int64_t tile;
        gemv_piece(a, G, g, 0, 0, &mat, &tile);
        const int64_t row0 = tile * QTR + wt;
#pragma unroll
        for (int m = 0; m < M; m++) {
            float y[NR];
#pragma unroll
            for (int r = 0; r < NR; r++) y[r] = warp_butterfly(acc[r][m]);
            if (lane != 0) continue;
            if (a.map == MAP_SINGLE) {
                if (row0 >= a.wrows[0]) continue;
                float v = y[0];
                if (a.res) v = __fadd_rn(a.res[m * a.ldr + row0], v);
                a.out[m * a.ldo + row0] = v;
            } else if (a.map == MAP_SWIGLU) {
                if (row0 >= a.wrows[0]) continue;
                a.out[m * a.ldo + row0] = __fmul_rn(gc_silu(y[0]), y[NR - 1]);
            } else {
                const int64_t half = a.D / 2, h = row0 / a.D, i = row0 % a.D;
                const int32_t p = a.pos[m];
                float y0 = y[0], y1 = y[NR - 1];
                if (mat < 2) {
                    float c, sn;
                    if (p >= 0 && p < a.npos) {
                        c = a.table[(p * half + i) * 2];
                        sn = a.table[(p * half + i) * 2 + 1];
                    } else {
                        float theta = (float)p;
                        for (int64_t kk = 0; kk < i; kk++) theta = __fmul_rn(theta, a.theta_scale);
                        c = cosf(theta);
                        sn = sinf(theta);
                    }
                    const float x0 = y0, x1 = y1;
                    y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
                    y1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
                }
                if (mat == 0) {
                    float *qo = a.q_out + m * a.ldq + h * a.D;
                    qo[i] = y0;
                    qo[i + half] = y1;
                } else if (p >= 0 && p < a.cache_rows) {
                    char *base = (mat == 1 ? a.kcache : a.vcache) + p * a.cache_nb1 + h * a.cache_nb2;
                    ((__half *)base)[i] = __float2half_rn(y0);
                    ((__half *)base)[i + half] = __float2half_rn(y1);
                } else if (a.err) {
                    atomicExch(a.err, 1);
                }
            }
        }
    }
    return true;
}

__host__ __device__ inline size_t gemv_act_bytes(int M, int64_t K) {
    return ((size_t)M * (size_t)K + (size_t)M * (size_t)(K / 32) * 8 + 127) / 128 * 128;
}

}  // namespace k
}  // namespace gcb
