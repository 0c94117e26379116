// Device building blocks of the streamed quantized GEMV, shared by the per-op kernel (gc_fused.cu)
// and the per-token decode kernel (gc_mega.cu).
//
// Weights stream as pieces (one 8-row tile x one 128-block segment each, gc_qweight.cuh) through a
// ring of NS (a power of two) shared-memory slots: the producer lane puts piece t in slot t % NS
// after the slot's previous piece was released (empty barrier) and arms full[t % NS] with the byte
// count; the team of 8 consumer warps owning that piece waits on full, computes and releases. A
// CTA's local row groups are taken in chunks (gemv_chunk); its pieces are numbered in the order
// (phase, chunk, segment, local group of the chunk, piece of the group), which producer and
// consumers both derive from the same geometry. Counters and geometry are 32-bit: no 64-bit
// division on the streaming path.
//
// Arithmetic is the CPU checker's: the activation row -> Q8_0 blocks (d = amax/127 in fp16,
// codes = nearest-even(x * 127/amax)), lane l owns blocks l, l+32, ... of a row (segments are
// multiples of 32 blocks, walked in order), acc = fma(d_w * d_x, isum, acc) with the exact integer
// dot, then the 32-lane butterfly. Only the fma chain and the butterfly are ordered; the block
// products they consume may be computed in any order, which is what lets a lane load a piece's
// blocks ahead of the arithmetic.
#pragma once

#include "../gc_fused.h"
#include "gc_math.cuh"
#include "gc_qweight.cuh"
#include "gc_tma.cuh"

namespace gcb {
namespace k {

constexpr int GEMV_MAXM = 8;

// Shared-memory staging of M activation rows of K values: int8 codes [M][K], f32 block scales
// [M][K / 32], int 8 x code sums [M][K / 32], rounded up to 128 bytes.
__host__ __device__ inline size_t gemv_act_bytes(int M, int64_t K) {
    return ((size_t)M * (size_t)K + (size_t)M * (size_t)(K / 32) * 8 + 127) / 128 * 128;
}

// Geometry of one GEMV over the tiled weights. With a.nshard > 1 the groups are this shard's: a
// contiguous run of tiles (MAP_SINGLE, MAP_SWIGLU) or this shard's query and K/V heads (MAP_ROPE_QKV);
// gemv_piece maps them back to the global tiles, so every row keeps its single-shard arithmetic.
struct GemvGeo {
    int nb, nseg, groups;  // blocks per row, segments per row, row groups (tiles / tile pairs)
    int cb, pieces;        // code bytes per block, pieces per (group, segment)
    int half_tiles;        // ROPE_QKV: tiles per half head
    int gbase;             // SINGLE / SWIGLU: first tile of the shard
    int hq, hkv, q0, kv0;  // ROPE_QKV: query / K/V heads of the shard, first of each
};

// First tile of shard `r` of `n` over `tiles` tiles (the host planner splits exchanges the same way).
__host__ __device__ inline int shard_tile(int tiles, int r, int n) { return (int)((int64_t)tiles * r / n); }

__host__ __device__ inline GemvGeo gemv_geo(const FusedArgs &a) {
    GemvGeo G{};
    G.nb = (int)(a.K / 32);
    G.nseg = (int)qw_nseg(G.nb);
    G.cb = a.qtype == T_Q4_0 ? 16 : 32;
    if (a.map == MAP_SINGLE || a.map == MAP_SWIGLU) {
        const int tiles = (int)((a.wrows[0] + QTR - 1) / QTR);
        G.gbase = shard_tile(tiles, a.shard, a.nshard);
        G.groups = shard_tile(tiles, a.shard + 1, a.nshard) - G.gbase;
        G.pieces = a.map == MAP_SINGLE ? 1 : 2;
    } else {
        G.half_tiles = (int)((a.D / 2) / QTR);
        G.hq = (int)(a.H / a.nshard);
        G.hkv = (int)(a.Hkv / a.nshard);
        G.q0 = a.shard * G.hq;
        G.kv0 = a.shard * G.hkv;
        G.groups = (G.hq + 2 * G.hkv) * G.half_tiles;
        G.pieces = 2;
    }
    return G;
}

// Groups of a GEMV handled by CTA `cta` of `nctas` (groups cta, cta + nctas, ...).
__host__ __device__ inline int local_groups(int groups, int cta, int nctas) {
    return cta < groups ? (groups - cta + nctas - 1) / nctas : 0;
}

// Local row groups per chunk: segment-major walks (so a lane's activation registers serve the
// chunk's `cg` groups per team) need one activation row; with more rows each group is its own chunk.
__host__ __device__ inline int gemv_chunk(int M, int teams, int cg) { return M == 1 ? cg * teams : 1; }

// Source of piece r (0/1) of group g, segment s; the matrix and the tile of piece r.
__device__ __forceinline__ const char *gemv_piece(const FusedArgs &a, const GemvGeo &G, int g, int r, int s, int *mat,
                                                  int *tile) {
    int m = 0, t;
    if (a.map == MAP_SINGLE) {
        t = g + G.gbase;
    } else if (a.map == MAP_SWIGLU) {
        m = r;
        t = g + G.gbase;
    } else {
        const int head = g / G.half_tiles, p = g - head * G.half_tiles;
        int h;
        if (head < G.hq) {
            m = 0;
            h = G.q0 + head;
        } else if (head < G.hq + G.hkv) {
            m = 1;
            h = G.kv0 + head - G.hq;
        } else {
            m = 2;
            h = G.kv0 + head - G.hq - G.hkv;
        }
        t = h * (2 * G.half_tiles) + p + r * G.half_tiles;
    }
    *mat = m;
    *tile = t;
    return a.wc[m] + qw_piece_off(G.nb, G.cb, t, s);
}

// Piece t lives in slot t mod ns; its fill is phase floor(t / ns) of that slot's barriers. The
// quotient comes from a multiply-high by magic = ceil(2^32 / ns), exact for t < 2^32 / ns (a CTA
// streams far fewer pieces in one launch), so any slot count fits the shared-memory budget.
struct Ring {
    uint64_t *full, *empty;
    unsigned char *slots;
    uint32_t ns, magic;
    int slot_bytes;
    __device__ __forceinline__ uint32_t round(uint32_t t) const { return __umulhi(t, magic); }
    __device__ __forceinline__ int slot(uint32_t t) const { return (int)(t - round(t) * ns); }
    __device__ __forceinline__ uint32_t parity(uint32_t t) const { return round(t) & 1u; }
    __device__ __forceinline__ unsigned char *data(uint32_t t) const { return slots + (size_t)slot(t) * slot_bytes; }
};

__host__ inline uint32_t ring_magic(uint32_t ns) { return (uint32_t)((((uint64_t)1 << 32) + ns - 1) / ns); }

// Producer: put this CTA's pieces of one GEMV into the ring, continuing the piece count `t`.
// Returns false if a slot was never released (bounded wait).
__device__ inline bool produce_gemv(const FusedArgs &a, const GemvGeo &G, const Ring &R, uint32_t &t, int cta, int nctas,
                                    int chunk, uint64_t *hold = nullptr) {
    const int L = local_groups(G.groups, cta, nctas);
    const uint64_t policy = a.stream_evict_first ? l2_policy_evict_first() : 0;
    for (int c0 = 0; c0 < L; c0 += chunk) {
        const int c1 = c0 + chunk < L ? c0 + chunk : L;
        for (int s = 0; s < G.nseg; s++) {
            const uint32_t pb = (uint32_t)qw_piece_bytes(G.nb, G.cb, s);
            for (int gl = c0; gl < c1; gl++)
                for (int r = 0; r < G.pieces; r++, t++) {
                    const int slot = R.slot(t);
                    if (hold && t == (uint32_t)a.hold_pieces) mbar_wait(hold, 0);  // a late prologue only delays
                    if (t >= R.ns && !mbar_wait(&R.empty[slot], R.parity(t) ^ 1u)) return false;
                    mbar_expect_tx(&R.full[slot], pb);
                    int mat, tile;
                    const char *src = gemv_piece(a, G, cta + gl * nctas, r, s, &mat, &tile);
                    if (a.stream_evict_first) bulk_g2s_hint(R.data(t), src, pb, &R.full[slot], policy);
                    else bulk_g2s(R.data(t), src, pb, &R.full[slot]);
                }
        }
    }
    return true;
}

// This CTA's share of the L2 prefetch ranges (FusedArgs::pf): an even split over the launch's CTAs,
// in requests of at most 32 KiB.
__device__ inline void prefetch_next(const FusedArgs &a, int cta, int nctas) {
#pragma unroll
    for (int r = 0; r < 3; r++) {
        const int64_t n = a.pf_bytes[r];
        if (n <= 0) continue;
        const int64_t per = ((n + nctas - 1) / nctas + 255) & ~(int64_t)255;
        const int64_t b0 = (int64_t)cta * per, b1 = b0 + per < n ? b0 + per : n;
        for (int64_t o = b0; o < b1; o += 32768) l2_prefetch(a.pf[r] + o, (uint32_t)(b1 - o < 32768 ? b1 - o : 32768));
    }
}

// Drain after a failed wait: the copies still in flight into the ring land before the CTA exits.
__device__ inline void drain_ring(const Ring &R, uint32_t t) {
    const uint32_t ns = R.ns;
    for (uint32_t u = t > ns ? t - ns : 0; u < t; u++) mbar_wait(&R.full[R.slot(u)], R.parity(u), 100000000ull);
}

// Activation row(s) -> Q8_0 blocks in shared memory (sq codes, sdf scales as f32, ss8 8 x code sums),
// with rms_norm * w first for PRO_NORM. Run by the NCT consumer threads (thread ids 0 .. NCT-1);
// `bar` is their named barrier. The sum of squares uses the 256-partial double tree (threads 0..255).
// Loads are issued in batches ahead of the arithmetic that consumes them.
constexpr int GEMV_UB = 4;  // 4-block groups in flight per warp in the quantization pass

// The norm weights of the quantization pass's first round (PRO_NORM): a weight, written by no
// kernel of the step, so consumers may load it before griddepcontrol.wait and overlap the latency
// with the previous kernel's tail. `w` then goes to gemv_prologue.
template <int NCT>
__device__ __forceinline__ void gemv_norm_prefetch(const FusedArgs &a, float4 (&w)[GEMV_UB]) {
    const int nb = (int)(a.K / 32), warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int NW = NCT / 32;
    const int sub = lane >> 3, e = (lane & 7) * 4;
#pragma unroll
    for (int u = 0; u < GEMV_UB; u++) {
        const int b = warp * 4 + u * NW * 4 + sub;
        w[u] = (a.pro == PRO_NORM && b < nb) ? *(const float4 *)(a.norm_w + b * 32 + e) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

template <int M, int NCT>
__device__ inline void gemv_prologue(const FusedArgs &a, int8_t *sq, float *sdf, int *ss8, double *red, int bar,
                                     const float4 *wpre = nullptr) {
    const int K = (int)a.K, nb = K / 32;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    constexpr int NW = NCT / 32;
    constexpr int U = 16;  // loads in flight per thread in the sum of squares
    constexpr int UB = GEMV_UB;
    const int sub = lane >> 3, e = (lane & 7) * 4;
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    constexpr int STRIDE = NW * 4 * UB;  // blocks of one quantization round (UB 4-block groups per warp)
#pragma unroll
    for (int m = 0; m < M; m++) {
        const float *x = a.x + m * a.ldx;
        // a round's loads: the activation values and, for PRO_NORM, the norm weights
        auto load = [&](int b0, float4 (&v)[UB], float4 (&w)[UB]) {
#pragma unroll
            for (int u = 0; u < UB; u++) {
                const int b = b0 + u * NW * 4 + sub;
                v[u] = b < nb ? __ldcg((const float4 *)(x + b * 32 + e)) : zero;
                w[u] = (wpre && m == 0 && b0 == warp * 4) ? wpre[u]  // first round, loaded before the wait
                                                        : (a.pro == PRO_NORM && b < nb) ? *(const float4 *)(a.norm_w + b * 32 + e) : zero;
            }
        };
        // the first quantization round's loads go out before the norm's sum of squares, so both
        // passes wait for L2 once
        float4 v[UB], w[UB], vn[UB], wn[UB];
        load(warp * 4, v, w);
        float scale = 1.0f;
        if (a.pro == PRO_NORM) {
            if (tid < 256) {
                double p = 0.0;
                for (int i0 = tid; i0 < K; i0 += 256 * U) {
                    float vv[U];
#pragma unroll
                    for (int u = 0; u < U; u++) vv[u] = i0 + 256 * u < K ? __ldcg(x + i0 + 256 * u) : 0.0f;
#pragma unroll
                    for (int u = 0; u < U; u++)
                        if (i0 + 256 * u < K) p = __dadd_rn(p, (double)__fmul_rn(vv[u], vv[u]));
                }
                red[tid] = p;
            } else if constexpr (NCT > 256) {
                // threads the sum does not use pull the norm weights toward L1 for the pass below
                for (int i = (tid - 256) * 32; i < K; i += (NCT - 256) * 32)
                    asm volatile("prefetch.global.L1 [%0];" ::"l"(a.norm_w + i));
            }
            named_bar(bar, NCT);
            // the tree red[t] += red[t + off], off = 128 .. 1: three levels through shared memory,
            // the last five in warp 0 with shuffles (lane t adds lane t + off: the same pairs)
#pragma unroll
            for (int off = 128; off >= 32; off >>= 1) {
                if (tid < off) red[tid] = __dadd_rn(red[tid], red[tid + off]);
                named_bar(bar, NCT);
            }
            if (tid < 32) {
                double vd = red[tid];
#pragma unroll
                for (int off = 16; off >= 1; off >>= 1) vd = __dadd_rn(vd, __shfl_down_sync(0xffffffffu, vd, off));
                if (tid == 0) red[0] = vd;
            }
            named_bar(bar, NCT);
            const double tot = red[0];
            named_bar(bar, NCT);
            const float mean = __double2float_rn(__ddiv_rn(tot, (double)K));
            scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
        }
        for (int b0 = warp * 4; b0 < nb; b0 += STRIDE) {
            if (b0 + STRIDE < nb) load(b0 + STRIDE, vn, wn);  // the next round's loads first
#pragma unroll
            for (int u = 0; u < UB; u++) {
                const int b = b0 + u * NW * 4 + sub;
                float4 t = v[u];
                if (a.pro == PRO_NORM) {
                    t.x = __fmul_rn(__fmul_rn(t.x, scale), w[u].x);
                    t.y = __fmul_rn(__fmul_rn(t.y, scale), w[u].y);
                    t.z = __fmul_rn(__fmul_rn(t.z, scale), w[u].z);
                    t.w = __fmul_rn(__fmul_rn(t.w, scale), w[u].w);
                }
                float amax = fmaxf(fmaxf(fabsf(t.x), fabsf(t.y)), fmaxf(fabsf(t.z), fabsf(t.w)));
#pragma unroll
                for (int off = 4; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
                const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
                const int q0 = __float2int_rn(__fmul_rn(t.x, id)), q1 = __float2int_rn(__fmul_rn(t.y, id));
                const int q2 = __float2int_rn(__fmul_rn(t.z, id)), q3 = __float2int_rn(__fmul_rn(t.w, id));
                int sum = q0 + q1 + q2 + q3;
#pragma unroll
                for (int off = 4; off >= 1; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
                if (b < nb) {
                    *(uint32_t *)(sq + m * K + b * 32 + e) = (uint32_t)(q0 & 255) | ((uint32_t)(q1 & 255) << 8) |
                                                             ((uint32_t)(q2 & 255) << 16) | ((uint32_t)(q3 & 255) << 24);
                    if ((lane & 7) == 0) {
                        sdf[m * nb + b] = h2f(f2h(__fdiv_rn(amax, 127.0f)));
                        ss8[m * nb + b] = 8 * sum;
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < UB; u++) {
                v[u] = vn[u];
                w[u] = wn[u];
            }
        }
    }
    named_bar(bar, NCT);
}

// PRO_Q8: the M rows' staged blocks (a.xq, gemv_act_bytes(M, K) bytes) copied into shared memory by
// the NCT consumer threads.
template <int NCT>
__device__ inline void gemv_stage_q8(const FusedArgs &a, int8_t *sq, int bar, int M = 1) {
    const int n = (int)(gemv_act_bytes(M, a.K) / 16);
    const int4 *src = (const int4 *)a.xq;
    int4 *dst = (int4 *)sq;
    for (int i = threadIdx.x; i < n; i += NCT) dst[i] = __ldcg(src + i);
    named_bar(bar, NCT);
}

// One warp: the Q8_0 block of 32 consecutive f32 values at x (written by other CTAs: read through
// L2) into the staging layout at (codes, d, s8), with the prologue's rule: d = amax / 127 in fp16,
// codes = nearest-even(x * 127 / amax), s8 = 8 x the code sum.
__device__ inline void quantize_block_warp(const float *x, int8_t *codes, float *d, int *s8) {
    const int lane = threadIdx.x & 31;
    const float v = __ldcg(x + lane);
    const float amax = warp_max(fabsf(v));
    const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
    const int q = __float2int_rn(__fmul_rn(v, id));
    int sum = q;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    codes[lane] = (int8_t)q;
    if (lane == 0) {
        *d = h2f(f2h(__fdiv_rn(amax, 127.0f)));
        *s8 = 8 * sum;
    }
}

// After the CTA's consumers stored their rows (one activation row): what the launch emits for the
// next GEMV (FusedArgs::act_mode). `red` is the prologue's shared scratch, free by now.
template <int NCT>
__device__ inline void gemv_emit_act8(const FusedArgs &a, const GemvGeo &G, double *red, int bar) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    named_bar(bar, NCT);  // every consumer warp's rows are stored
    const int64_t N = a.wrows[0];
    int8_t *codes = (int8_t *)a.act_out;
    float *d = (float *)(a.act_out + N);
    int *s8 = (int *)(d + N / 32);
    if (a.act_mode == ACT8_NORM) {
        int *flag = (int *)red;
        if (threadIdx.x == 0) {
            __threadfence();
            const bool last = atomicAdd(a.act_cnt, 1) == (int)gridDim.x - 1;
            if (last) {
                *a.act_cnt = 0;
                __threadfence();
            }
            *flag = last ? 1 : 0;
        }
        named_bar(bar, NCT);
        const int last = *flag;
        named_bar(bar, NCT);  // `red` is the norm's scratch next
        if (!last) return;
        FusedArgs na = a;
        na.x = a.out;
        na.ldx = a.ldo;
        na.K = N;
        na.M = 1;
        na.pro = PRO_NORM;
        na.norm_w = a.act_norm_w;
        na.eps = a.act_eps;
        gemv_prologue<1, NCT>(na, codes, d, s8, red, bar);
    } else {
        // each 32-row block is quantized by the CTA that stores its last 8-row tile
        const int L = local_groups(G.groups, blockIdx.x, gridDim.x);
        for (int gl = warp; gl < L; gl += NCT / 32) {
            const int blk = (G.gbase + (int)blockIdx.x + gl * (int)gridDim.x) / (32 / QTR);
            int done = 0;
            if (lane == 0) {
                __threadfence();
                done = atomicAdd(a.act_cnt + blk, 1) == 32 / QTR - 1;
                if (done) {
                    a.act_cnt[blk] = 0;
                    __threadfence();
                }
            }
            if (__shfl_sync(0xffffffffu, done, 0))
                quantize_block_warp(a.out + (int64_t)blk * 32, codes + (int64_t)blk * 32, d + blk, s8 + blk);
        }
    }
}

// Epilogue operands of row `row0` (loaded by lane 0 before the row's pieces arrive): the residual
// (SINGLE) or the rotation's cos / sin (ROPE_QKV, q and k rows).
template <int M>
__device__ __forceinline__ void gemv_epi_load(const FusedArgs &a, int mat, int row0, float (&e0)[M], float (&e1)[M]) {
#pragma unroll
    for (int m = 0; m < M; m++) e0[m] = e1[m] = 0.0f;
    if (a.map == MAP_SINGLE) {
        if (a.res && row0 < a.wrows[0])
#pragma unroll
            for (int m = 0; m < M; m++) e0[m] = a.res[m * a.ldr + row0];
    } else if (a.map == MAP_ROPE_QKV && mat < 2) {
        const int D = (int)a.D, half = D / 2, i = row0 % D;
#pragma unroll
        for (int m = 0; m < M; m++) {
            const int32_t p = a.pos[m];
            if (p >= 0 && p < a.npos) {
                e0[m] = a.table[((int64_t)p * half + i) * 2];
                e1[m] = a.table[((int64_t)p * half + i) * 2 + 1];
            }
        }
    }
}

// Lane 0: row `row0`'s results y[piece][m] (already reduced over the warp) -> outputs.
template <int NR, int M>
__device__ __forceinline__ void gemv_epi_store(const FusedArgs &a, int mat, int row0, const float (&y)[NR][M],
                                               const float (&e0)[M], const float (&e1)[M]) {
#pragma unroll
    for (int m = 0; m < M; m++) {
        if (a.map == MAP_SINGLE) {
            if (row0 >= a.wrows[0]) continue;
            float v = y[0][m];
            if (a.res) v = __fadd_rn(e0[m], v);
            a.out[m * a.ldo + row0] = v;
        } else if (a.map == MAP_SWIGLU) {
            if (row0 >= a.wrows[0]) continue;
            a.out[m * a.ldo + row0] = __fmul_rn(gc_silu(y[0][m]), y[NR - 1][m]);
        } else {
            const int D = (int)a.D, half = D / 2, h = row0 / D, i = row0 - h * D;
            const int32_t p = a.pos[m];
            float y0 = y[0][m], y1 = y[NR - 1][m];
            if (mat < 2) {
                float c, sn;
                if (p >= 0 && p < a.npos) {
                    c = e0[m];
                    sn = e1[m];
                } else {
                    float theta = (float)p;
                    for (int kk = 0; kk < i; kk++) theta = __fmul_rn(theta, a.theta_scale);
                    c = cosf(theta);
                    sn = sinf(theta);
                }
                const float x0 = y0, x1 = y1;
                y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
                y1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
            }
            if (mat == 0) {
                float *qo = a.q_out + m * a.ldq + (int64_t)h * D;
                qo[i] = y0;
                qo[i + half] = y1;
            } else if (p >= 0 && p < a.cache_rows) {
                char *base = (mat == 1 ? a.kcache : a.vcache) + m * a.cache_nb3 + p * a.cache_nb1 + h * a.cache_nb2;
                ((__half *)base)[i] = __float2half_rn(y0);
                ((__half *)base)[i + half] = __float2half_rn(y1);
            } else if (a.err) {
                atomicExch(a.err, 1);
            }
        }
    }
}

// Waits (lane 0, bounded) for piece t to land; the outcome is shared with the warp.
__device__ __forceinline__ bool gemv_wait_piece(const Ring &R, uint32_t t) {
    int ready = 1;
    if ((threadIdx.x & 31) == 0) ready = mbar_wait(&R.full[R.slot(t)], R.parity(t)) ? 1 : 0;
    return __shfl_sync(0xffffffffu, ready, 0) != 0;
}

// ---------------------------------------------------------------- one activation row

constexpr int GEMV_NI = QSEG / 32;  // blocks of a lane in one segment

// a: four unsigned bytes, b: four signed bytes; c + their dot product.
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Conversions kept off the XU pipe (f16 -> f32 and int -> float there ran at a quarter of the FMA
// pipe's rate and held up the block loop), with the same results:
// - the block scale product d_w * d_x as one fma.rn.f32.f16 of the two f16 values with a -0 addend:
//   the product of two f16 values is exact in f32, so this equals __fmul_rn of their f32 forms
//   (the -0 keeps a zero product's sign);
// - the integer dot as a float through the 1.5 * 2^23 bias: for |v| < 2^22 the bits 0x4B400000 + v
//   are the float 12582912 + v, and subtracting 12582912 leaves v exactly.
__device__ __forceinline__ float mul_f16(uint32_t a, uint32_t b) {
    float d;
    asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(d) : "h"((unsigned short)a), "h"((unsigned short)b), "f"(-0.0f));
    return d;
}
__device__ __forceinline__ float i2f_exact(int v) { return __fsub_rn(__int_as_float(v + 0x4B400000), 12582912.0f); }

// This lane's blocks (lane + 32 i) of one segment of the activation row, from shared memory; the
// block scales as their f16 bits (the staging layout holds f16 values as f32, so this is exact).
struct Act1 {
    int4 lo[GEMV_NI], hi[GEMV_NI];
    uint32_t dh[GEMV_NI];
    int s8[GEMV_NI];
};

__device__ __forceinline__ void act1_load(Act1 &x, const int8_t *sq, const float *sdf, const int *ss8, int bbase, int sb,
                                          int lane) {
#pragma unroll
    for (int i = 0; i < GEMV_NI; i++) {
        const int j = lane + 32 * i;
        if (j < sb) {
            const int4 *x4 = (const int4 *)(sq + (bbase + j) * 32);
            x.lo[i] = x4[0];
            x.hi[i] = x4[1];
            x.dh[i] = __half_as_ushort(__float2half_rn(sdf[bbase + j]));
            x.s8[i] = ss8[bbase + j];
        }
    }
}

// acc += this lane's blocks of one row of a piece, against the activation registers: every load of
// the row first, then the products in block order. FULL: a whole segment (sb == QSEG), so every
// lane has all GEMV_NI blocks and no bound is tested; the integer dots of the blocks are then
// independent straight-line code, and only the fma chain is ordered.
template <int QT, bool FULL>
__device__ __forceinline__ void piece_row1(float &acc, const unsigned char *codes, const uint16_t *scl, const Act1 &x,
                                           int sb, int lane) {
    constexpr int CB = QT == 0 ? 16 : 32;
    int4 w0[GEMV_NI], w1[GEMV_NI];
    uint16_t sw[GEMV_NI];
#pragma unroll
    for (int i = 0; i < GEMV_NI; i++) {
        const int j = lane + 32 * i;
        if (FULL || j < sb) {
            w0[i] = *(const int4 *)(codes + j * CB);
            if (QT == 1) w1[i] = *(const int4 *)(codes + j * CB + 16);
            sw[i] = scl[j];
        }
    }
#pragma unroll
    for (int i = 0; i < GEMV_NI; i++) {
        if (!FULL && lane + 32 * i >= sb) break;
        int v = 0;
        if (QT == 0) {
            // low nibbles as they are; high nibbles masked in place (16 x their value), so that dot
            // product is exactly 16 x the high-nibble dot and is shifted back once (exact: integer)
            const uint32_t *w = (const uint32_t *)&w0[i];
            int lo = -x.s8[i], hi = 0;  // the 8 x sum(x) offset of Q4_0's (q - 8) folded into the start
            lo = __dp4a((int)(w[0] & 0x0f0f0f0fu), x.lo[i].x, lo);
            hi = dp4a_us(w[0] & 0xf0f0f0f0u, x.hi[i].x, hi);
            lo = __dp4a((int)(w[1] & 0x0f0f0f0fu), x.lo[i].y, lo);
            hi = dp4a_us(w[1] & 0xf0f0f0f0u, x.hi[i].y, hi);
            lo = __dp4a((int)(w[2] & 0x0f0f0f0fu), x.lo[i].z, lo);
            hi = dp4a_us(w[2] & 0xf0f0f0f0u, x.hi[i].z, hi);
            lo = __dp4a((int)(w[3] & 0x0f0f0f0fu), x.lo[i].w, lo);
            hi = dp4a_us(w[3] & 0xf0f0f0f0u, x.hi[i].w, hi);
            v = lo + (hi >> 4);
        } else {
            v = __dp4a(w0[i].x, x.lo[i].x, v);
            v = __dp4a(w0[i].y, x.lo[i].y, v);
            v = __dp4a(w0[i].z, x.lo[i].z, v);
            v = __dp4a(w0[i].w, x.lo[i].w, v);
            v = __dp4a(w1[i].x, x.hi[i].x, v);
            v = __dp4a(w1[i].y, x.hi[i].y, v);
            v = __dp4a(w1[i].z, x.hi[i].z, v);
            v = __dp4a(w1[i].w, x.hi[i].w, v);
        }
        acc = __fmaf_rn(mul_f16(sw[i], x.dh[i]), i2f_exact(v), acc);
    }
}

// Consumer side of one GEMV with one activation row: this team's groups (every `teams`-th local
// group, starting at `team`), chunk by chunk and segment-major inside a chunk, pieces numbered from
// t0; the butterflies and epilogues of a chunk's groups run together at its end. `wt` is the warp's
// row within the tile. False on a timed-out wait.
template <int QT, int NR, int CG>
__device__ inline bool consume_gemv1(const FusedArgs &a, const GemvGeo &G, const Ring &R, uint32_t t0, int cta, int nctas,
                                     int team, int teams, int wt, const int8_t *sq, const float *sdf, const int *ss8) {
    constexpr int CB = QT == 0 ? 16 : 32;
    const int lane = threadIdx.x & 31;
    const int L = local_groups(G.groups, cta, nctas), chunk = gemv_chunk(1, teams, CG);
    const int per_group = G.nseg * G.pieces;
    Act1 x;
    int loaded = -1;  // segment whose activation is in x
    for (int c0 = 0; c0 < L; c0 += chunk) {
        const int c1 = c0 + chunk < L ? c0 + chunk : L, n = c1 - c0;
        int mat[CG], row0[CG];
        float acc[CG][NR], e0[CG][1], e1[CG][1];
#pragma unroll
        for (int j = 0; j < CG; j++) {
            const int q = team + j * teams;
            mat[j] = row0[j] = 0;
#pragma unroll
            for (int r = 0; r < NR; r++) acc[j][r] = 0.0f;
            e0[j][0] = e1[j][0] = 0.0f;
            if (q < n) {
                int tile;
                gemv_piece(a, G, cta + (c0 + q) * nctas, 0, 0, &mat[j], &tile);
                row0[j] = tile * QTR + wt;
                if (lane == 0) gemv_epi_load<1>(a, mat[j], row0[j], e0[j], e1[j]);
            }
        }
        const uint32_t tb = t0 + (uint32_t)(c0 * per_group);
        for (int s = 0; s < G.nseg; s++) {
            const int sb = (int)qw_seg_blocks(G.nb, s);
            if (s != loaded) {
                act1_load(x, sq, sdf, ss8, s * QSEG, sb, lane);
                loaded = s;
            }
#pragma unroll
            for (int j = 0; j < CG; j++) {
                const int q = team + j * teams;
                if (q >= n) break;
#pragma unroll
                for (int r = 0; r < NR; r++) {
                    const uint32_t t = tb + (uint32_t)((s * n + q) * G.pieces + r);
                    if (!gemv_wait_piece(R, t)) return false;
                    const unsigned char *piece = R.data(t);
                    if (sb == QSEG)
                        piece_row1<QT, true>(acc[j][r], piece + wt * QSEG * CB, (const uint16_t *)(piece + QTR * QSEG * CB) + wt * QSEG,
                                             x, QSEG, lane);
                    else
                        piece_row1<QT, false>(acc[j][r], piece + wt * sb * CB, (const uint16_t *)(piece + QTR * sb * CB) + wt * sb,
                                              x, sb, lane);
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&R.empty[R.slot(t)]);
                }
            }
        }
        float y[CG][NR][1];
#pragma unroll
        for (int j = 0; j < CG; j++)
#pragma unroll
            for (int r = 0; r < NR; r++) y[j][r][0] = acc[j][r];
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1)  // the butterflies of every group at once
#pragma unroll
            for (int j = 0; j < CG; j++)
#pragma unroll
                for (int r = 0; r < NR; r++) y[j][r][0] = __fadd_rn(y[j][r][0], __shfl_xor_sync(0xffffffffu, y[j][r][0], off));
        if (lane == 0)
#pragma unroll
            for (int j = 0; j < CG; j++)
                if (team + j * teams < n) gemv_epi_store<NR, 1>(a, mat[j], row0[j], y[j], e0[j], e1[j]);
    }
    return true;
}

// ---------------------------------------------------------------- several activation rows

// Several activation rows: one quantized block of RPW tile rows (row rr at codes + rr * cstride,
// its scales at scl + rr * sstride) against every activation row; each activation block is loaded
// from shared memory once for the RPW weight rows. Integer dots are exact, so their partial sums
// may be grouped in any order; the float fma per (row, activation row) is the one-row order.
template <int QT, int NR, int M, int RPW>
__device__ __forceinline__ void gemv_blockR(float (&acc)[NR][RPW][M], int r, const unsigned char *codes, int cstride,
                                            const uint16_t *scl, int sstride, int j, int b, const int8_t *sq,
                                            const float *sdf, const int *ss8, int K, int nb) {
    float dw[RPW];
#pragma unroll
    for (int rr = 0; rr < RPW; rr++) dw[rr] = h2f(scl[rr * sstride + j]);
    if (QT == 0) {
        uint32_t lo[RPW][4], hi[RPW][4];
#pragma unroll
        for (int rr = 0; rr < RPW; rr++) {
            const uint4 w = *(const uint4 *)(codes + rr * cstride + j * 16);
            const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int q = 0; q < 4; q++) {
                lo[rr][q] = wv[q] & 0x0f0f0f0fu;
                hi[rr][q] = (wv[q] >> 4) & 0x0f0f0f0fu;
            }
        }
#pragma unroll
        for (int m = 0; m < M; m++) {
            const int4 *x4 = (const int4 *)(sq + m * K + b * 32);
            const int4 xa = x4[0], xb = x4[1];
            const int xl[4] = {xa.x, xa.y, xa.z, xa.w}, xh[4] = {xb.x, xb.y, xb.z, xb.w};
            const float dx = sdf[m * nb + b];
            const int s8 = ss8[m * nb + b];
#pragma unroll
            for (int rr = 0; rr < RPW; rr++) {
                const int v = (__dp4a((int)lo[rr][0], xl[0], __dp4a((int)hi[rr][0], xh[0], 0)) +
                               __dp4a((int)lo[rr][1], xl[1], __dp4a((int)hi[rr][1], xh[1], 0))) +
                              (__dp4a((int)lo[rr][2], xl[2], __dp4a((int)hi[rr][2], xh[2], 0)) +
                               __dp4a((int)lo[rr][3], xl[3], __dp4a((int)hi[rr][3], xh[3], -s8)));
                acc[r][rr][m] = __fmaf_rn(__fmul_rn(dw[rr], dx), i2f_exact(v), acc[r][rr][m]);
            }
        }
    } else {
        int w[RPW][8];
#pragma unroll
        for (int rr = 0; rr < RPW; rr++) {
            const int4 a = *(const int4 *)(codes + rr * cstride + j * 32), c = *(const int4 *)(codes + rr * cstride + j * 32 + 16);
            w[rr][0] = a.x, w[rr][1] = a.y, w[rr][2] = a.z, w[rr][3] = a.w;
            w[rr][4] = c.x, w[rr][5] = c.y, w[rr][6] = c.z, w[rr][7] = c.w;
        }
#pragma unroll
        for (int m = 0; m < M; m++) {
            const int4 *x4 = (const int4 *)(sq + m * K + b * 32);
            const int4 xa = x4[0], xb = x4[1];
            const int xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
            const float dx = sdf[m * nb + b];
#pragma unroll
            for (int rr = 0; rr < RPW; rr++) {
                const int v = (__dp4a(w[rr][0], xv[0], __dp4a(w[rr][1], xv[1], 0)) + __dp4a(w[rr][2], xv[2], __dp4a(w[rr][3], xv[3], 0))) +
                              (__dp4a(w[rr][4], xv[4], __dp4a(w[rr][5], xv[5], 0)) + __dp4a(w[rr][6], xv[6], __dp4a(w[rr][7], xv[7], 0)));
                acc[r][rr][m] = __fmaf_rn(__fmul_rn(dw[rr], dx), i2f_exact(v), acc[r][rr][m]);
            }
        }
    }
}

// Consumer side of one GEMV. One activation row: consume_gemv1. Several: the CTA's row groups are
// taken in chunks of `teams` groups, segment-major inside a chunk (the producer's order for a
// chunk of that size), team `team` owning group `team` of each chunk; a team is 8 / RPW warps, warp
// `wt` owning tile rows RPW wt .. RPW wt + RPW - 1, so each activation block is read from shared
// memory once for RPW weight rows. Each row keeps the one-row arithmetic: lane l, blocks l, l + 32,
// ... in order, then the butterfly. False on a timed-out wait.
template <int QT, int NR, int M, int CG, int RPW = 1>
__device__ inline bool consume_gemv(const FusedArgs &a, const GemvGeo &G, const Ring &R, uint32_t t0, int cta, int nctas,
                                    int team, int teams, int wt, const int8_t *sq, const float *sdf, const int *ss8) {
    if constexpr (M == 1) {
        return consume_gemv1<QT, NR, CG>(a, G, R, t0, cta, nctas, team, teams, wt, sq, sdf, ss8);
    } else {
        constexpr int CB = QT == 0 ? 16 : 32;
        const int lane = threadIdx.x & 31;
        const int K = (int)a.K, nb = G.nb;
        const int per_group = G.nseg * G.pieces;
        const int L = local_groups(G.groups, cta, nctas);
        for (int c0 = 0; c0 < L; c0 += teams) {
            const int n = c0 + teams < L ? teams : L - c0;
            if (team >= n) break;
            int mat, tile;
            gemv_piece(a, G, cta + (c0 + team) * nctas, 0, 0, &mat, &tile);
            const int row0 = tile * QTR + RPW * wt;
            float e0[RPW][M], e1[RPW][M];
            if (lane == 0)
#pragma unroll
                for (int rr = 0; rr < RPW; rr++) gemv_epi_load<M>(a, mat, row0 + rr, e0[rr], e1[rr]);
            float acc[NR][RPW][M];
#pragma unroll
            for (int r = 0; r < NR; r++)
#pragma unroll
                for (int rr = 0; rr < RPW; rr++)
#pragma unroll
                    for (int m = 0; m < M; m++) acc[r][rr][m] = 0.0f;
            const uint32_t tb = t0 + (uint32_t)(c0 * per_group);
            for (int s = 0; s < G.nseg; s++) {
                const int sb = (int)qw_seg_blocks(nb, s);
                const int bbase = s * QSEG;
#pragma unroll
                for (int r = 0; r < NR; r++) {
                    const uint32_t t = tb + (uint32_t)((s * n + team) * G.pieces + r);
                    if (!gemv_wait_piece(R, t)) return false;
                    const unsigned char *piece = R.data(t);
                    const unsigned char *codes = piece + RPW * wt * sb * CB;
                    const uint16_t *scl = (const uint16_t *)(piece + QTR * sb * CB) + RPW * wt * sb;
                    if (sb == QSEG) {
#pragma unroll
                        for (int i = 0; i < QSEG / 32; i++)
                            gemv_blockR<QT, NR, M, RPW>(acc, r, codes, QSEG * CB, scl, QSEG, lane + 32 * i, bbase + lane + 32 * i,
                                                        sq, sdf, ss8, K, nb);
                    } else {
                        for (int j = lane; j < sb; j += 32)
                            gemv_blockR<QT, NR, M, RPW>(acc, r, codes, sb * CB, scl, sb, j, bbase + j, sq, sdf, ss8, K, nb);
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&R.empty[R.slot(t)]);
                }
            }
#pragma unroll
            for (int rr = 0; rr < RPW; rr++) {
                float y[NR][M];
#pragma unroll
                for (int m = 0; m < M; m++)
#pragma unroll
                    for (int r = 0; r < NR; r++) y[r][m] = warp_butterfly(acc[r][rr][m]);
                if (lane == 0) gemv_epi_store<NR, M>(a, mat, row0 + rr, y, e0[rr], e1[rr]);
            }
        }
        return true;
    }
}

// Ring slots for a shared-memory budget: as many as fit, at most `maxns`.
__host__ inline int ring_slots(size_t budget, size_t head, size_t slot_bytes, int maxns) {
    int n = budget > head ? (int)((budget - head) / slot_bytes) : 0;
    return n < maxns ? n : maxns;
}

}  // namespace k
}  // namespace gcb
