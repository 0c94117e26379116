// Decode-time quantized GEMV on B200: persistent CTAs streaming weight tiles with bulk copies
// (cp.async.bulk) into a shared-memory ring, with the neighbouring nodes folded in.
//
// Weights are in the tiled layout of gc_qweight.cuh: a (tile of 8 rows, 128-block segment) piece is
// one contiguous range. A CTA owns a set of row groups ("groups": one tile, or a pair of tiles for the
// paired maps) and walks them segment by segment. Warp 8 is the producer: one lane issues a bulk
// copy per piece into ring slot s and arms full[s] with the byte count. Warps 0-7 are consumers:
// each owns one row (or row pair) of the group, waits on full[s], accumulates its blocks from shared
// memory and arrives on empty[s], which the producer waits on before refilling the slot.
//
//   prologue  ACT:  the input row(s) f32 -> Q8_0 blocks (ggml's activation conversion)
//             NORM: rms_norm(x) * w first (the rms_norm + mul nodes), then Q8_0
//   map       SINGLE: out[m, n]                               (o_proj, down, lm_head, plain mul_mat)
//             ROPE_QKV: rows i and i + D/2 of a head of [Wq; Wk; Wv] per warp, NEOX rope on q and k,
//                       q to a buffer, k and v cast to f16 into the KV cache at `pos` (set_rows)
//             SWIGLU: row i of Wgate and of Wup per warp, out = silu(g) * u
//   epilogue  optional residual: out = res + y (the add node)
//
// Arithmetic is op for op the unfused nodes' in the CPU checker's order: lane l owns blocks l, l+32,
// l+64, ... of a row (segments are whole multiples of 32 blocks, walked in order), per block
// acc = fma(d_w * d_x, isum, acc) with the exact integer dot, then the 32-lane butterfly.
//
// PDL: the producer never reads anything an earlier kernel writes, so it starts streaming at once;
// the consumers execute griddepcontrol.wait before reading the activation. Nothing is written before
// that wait. Every mbarrier wait is bounded in time; a timeout sets the error word (2) and the CTA
// drains its copies in flight (again bounded) and exits.
#include <stdexcept>
#include <string>

#include "../gc_fused.h"
#include "gc_math.cuh"
#include "gc_qweight.cuh"
#include "gc_tma.cuh"

namespace gcb {
namespace k {

namespace {

constexpr int NCW = 8;                  // consumer warps
constexpr int NTHREADS = (NCW + 1) * 32;
constexpr int MAXM = 8;
constexpr int MAXNS = 8;

struct Geo {
    int64_t nb, nseg, groups;
    int cb, pieces;       // pieces per stage (1 or 2)
    int64_t stage_bytes;  // ring slot size
    int ns;               // ring slots
    int64_t half_tiles;   // ROPE: tiles per half head
};

// Source of piece `r` (0 or 1) of group `g`, segment `s`.
__device__ __forceinline__ const char *piece_src(const FusedArgs &a, const Geo &G, int64_t g, int r, int64_t s, int *mat,
                                                 int64_t *tile) {
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

// 256-way double tree over the consumer threads (named barrier 1).
__device__ __forceinline__ double tree256_consumers(double p, double *sh) {
    const int t = threadIdx.x;
    sh[t] = p;
    named_bar(1, NCW * 32);
#pragma unroll
    for (int off = 128; off >= 1; off >>= 1) {
        if (t < off) sh[t] = __dadd_rn(sh[t], sh[t + off]);
        named_bar(1, NCW * 32);
    }
    const double r = sh[0];
    named_bar(1, NCW * 32);
    return r;
}

__host__ __device__ __forceinline__ size_t act_head_bytes(int M, int64_t K, int64_t nb) {
    return (((size_t)(2 * MAXNS) * 8 + 256 * 8 + (size_t)M * K + (size_t)M * nb * 8 + 127) / 128) * 128;
}

// One quantized block of this lane's row against every activation row: exact integer dot, then
// acc = fma(d_w * d_x, isum, acc).
template <int QT, int NR, int M>
__device__ __forceinline__ void block_step(float (&acc)[NR][M], int r, const unsigned char *codes, const uint16_t *scl,
                                           int j, int bbase, const int8_t *sq, const float *sdf, const int *ss8,
                                           int64_t K, int64_t nb) {
    const int b = bbase + j;
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

template <int QT, int NR, int M>
__global__ void __launch_bounds__(NTHREADS, 2) gemv_tma_kernel(FusedArgs a, Geo G) {
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t *full = (uint64_t *)smem;
    uint64_t *empty = full + MAXNS;
    double *red = (double *)(empty + MAXNS);           // [256]
    int8_t *sq = (int8_t *)(red + 256);                 // [M][K] activation codes
    const int64_t K = a.K, nb = G.nb;
    float *sdf = (float *)(sq + (size_t)M * K);         // [M][nb] block scales (fp16 values as f32)
    int *ss8 = (int *)(sdf + (size_t)M * nb);           // [M][nb] 8 x block code sums (Q4_0 offset)
    unsigned char *ring = smem + act_head_bytes(M, K, nb);
    constexpr int CB = QT == 0 ? 16 : 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < G.ns; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NCW);
        }
        mbar_fence_init();
    }
    __syncthreads();
    pdl_trigger();

    if (warp == NCW) {  // ---------------- producer
        if (lane != 0) return;
        int64_t t = 0;
        bool ok = true;
        for (int64_t g = blockIdx.x; g < G.groups && ok; g += gridDim.x) {
            for (int64_t s = 0; s < G.nseg; s++, t++) {
                const int slot = (int)(t % G.ns);
                if (t >= G.ns && !mbar_wait(&empty[slot], (uint32_t)(((t / G.ns) - 1) & 1))) {
                    ok = false;
                    break;
                }
                const uint32_t pb = (uint32_t)qw_piece_bytes(nb, CB, s);
                mbar_expect_tx(&full[slot], pb * G.pieces);
                for (int r = 0; r < G.pieces; r++) {
                    int mat;
                    int64_t tile;
                    const char *src = piece_src(a, G, g, r, s, &mat, &tile);
                    bulk_g2s(ring + slot * G.stage_bytes + r * (int64_t)pb, src, pb, &full[slot]);
                }
            }
        }
        if (!ok) {  // a consumer stopped: record it, then let the copies already issued land
            if (a.err) atomicExch(a.err, 2);
            for (int64_t u = t - G.ns; u < t; u++)
                if (u >= 0) mbar_wait(&full[u % G.ns], (uint32_t)((u / G.ns) & 1), 100000000ull);
        }
        return;
    }

    // ---------------- consumers: activation prologue (after the producing kernel is done)
    pdl_wait();
    for (int m = 0; m < M; m++) {
        const float *x = a.x + m * a.ldx;
        float scale = 1.0f;
        if (a.pro == PRO_NORM) {  // the sum of squares in the 256-partial order
            double p = 0.0;
            for (int64_t i = threadIdx.x; i < K; i += NCW * 32) p = __dadd_rn(p, (double)__fmul_rn(x[i], x[i]));
            const double tot = tree256_consumers(p, red);
            const float mean = __double2float_rn(__ddiv_rn(tot, (double)K));
            scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
        }
        // 4 blocks per warp step: 8 lanes per block, 4 values per lane
        const int sub = lane >> 3, e = (lane & 7) * 4;
        for (int64_t b0 = (int64_t)warp * 4; b0 < nb; b0 += NCW * 4) {
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
    named_bar(1, NCW * 32);

    int64_t t = 0;
    for (int64_t g = blockIdx.x; g < G.groups; g += gridDim.x) {
        float acc[NR][M];
#pragma unroll
        for (int r = 0; r < NR; r++)
#pragma unroll
            for (int m = 0; m < M; m++) acc[r][m] = 0.0f;
        for (int64_t s = 0; s < G.nseg; s++, t++) {
            const int slot = (int)(t % G.ns);
            if (!mbar_wait(&full[slot], (uint32_t)((t / G.ns) & 1))) {
                if (a.err) atomicExch(a.err, 2);
                return;
            }
            const int sb = (int)qw_seg_blocks(nb, s);
            const int pb = QTR * sb * (CB + 2);
            const int bbase = (int)(s * QSEG);
#pragma unroll
            for (int r = 0; r < NR; r++) {
                const unsigned char *piece = ring + slot * G.stage_bytes + r * pb;
                const unsigned char *codes = piece + warp * sb * CB;
                const uint16_t *scl = (const uint16_t *)(piece + QTR * sb * CB) + warp * sb;
                if (sb == QSEG) {
#pragma unroll
                    for (int i = 0; i < QSEG / 32; i++)
                        block_step<QT, NR, M>(acc, r, codes, scl, lane + 32 * i, bbase, sq, sdf, ss8, K, nb);
                } else {
                    for (int j = lane; j < sb; j += 32) block_step<QT, NR, M>(acc, r, codes, scl, j, bbase, sq, sdf, ss8, K, nb);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
        // epilogue for this warp's row(s)
        int mat;
        int64_t tile;
        piece_src(a, G, g, 0, 0, &mat, &tile);
        const int64_t row0 = tile * QTR + warp;  // row of piece 0 in matrix `mat`
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
                const int64_t half = a.D / 2, h = row0 / a.D, i = row0 % a.D;  // i < half: piece 1 is row i + half
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
}

int g_num_sms = 0;
size_t g_smem_budget = 0;

template <int QT, int NR, int M>
void launch_t(const FusedArgs &a, const Geo &G0, cudaStream_t s, bool pdl) {
    auto kern = gemv_tma_kernel<QT, NR, M>;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        attr = true;
    }
    Geo G = G0;
    const size_t head = act_head_bytes(M, a.K, G.nb);
    const size_t budget = g_smem_budget ? g_smem_budget : 110 * 1024;
    int ns = (int)((budget > head ? budget - head : 0) / (size_t)G.stage_bytes);
    ns = ns < 2 ? 2 : (ns > MAXNS ? MAXNS : ns);
    G.ns = ns;
    const size_t smem = head + (size_t)ns * (size_t)G.stage_bytes;
    const int per_sm = smem <= 113 * 1024 ? 2 : 1;
    cudaLaunchConfig_t cfg = {};
    const int64_t cap = (int64_t)g_num_sms * per_sm;
    const int64_t ctas = G.groups < cap ? G.groups : cap;
    cfg.gridDim = dim3((unsigned)(ctas < 1 ? 1 : ctas));
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a, G);
    if (e != cudaSuccess) throw std::runtime_error(std::string("CUDA launch of gemv_tma failed: ") + cudaGetErrorString(e));
}

template <int QT, int NR>
void launch_m(const FusedArgs &a, const Geo &G, cudaStream_t s, bool pdl) {
    switch (a.M) {
        case 1: launch_t<QT, NR, 1>(a, G, s, pdl); break;
        case 2: launch_t<QT, NR, 2>(a, G, s, pdl); break;
        case 3: launch_t<QT, NR, 3>(a, G, s, pdl); break;
        case 4: launch_t<QT, NR, 4>(a, G, s, pdl); break;
        case 5: launch_t<QT, NR, 5>(a, G, s, pdl); break;
        case 6: launch_t<QT, NR, 6>(a, G, s, pdl); break;
        case 7: launch_t<QT, NR, 7>(a, G, s, pdl); break;
        case 8: launch_t<QT, NR, 8>(a, G, s, pdl); break;
        default: throw std::runtime_error("gemv_tma: 1 to 8 activation rows");
    }
}

}  // namespace

bool fused_gemv_supported(int64_t K, int64_t M, int map) {
    (void)map;
    if (K % 32 || M < 1 || M > MAXM) return false;
    return (size_t)M * K + (size_t)M * (K / 32) * 8 <= 64 * 1024;
}

void fused_gemv(const FusedArgs &a, cudaStream_t s, bool pdl) {
    if (!g_num_sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (const char *b = std::getenv("GCB_GEMV_SMEM_KB")) g_smem_budget = (size_t)std::atoi(b) * 1024;
    }
    Geo G{};
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
        if ((a.D / 2) % QTR) throw std::runtime_error("gemv_tma: head size must be a multiple of 16");
        G.half_tiles = (a.D / 2) / QTR;
        G.groups = (a.H + 2 * a.Hkv) * G.half_tiles;
        G.pieces = 2;
    }
    G.stage_bytes = (int64_t)G.pieces * qw_piece_bytes(G.nb, G.cb, 0);
    const bool q4 = a.qtype == T_Q4_0;
    if (G.pieces == 1) {
        if (q4) launch_m<0, 1>(a, G, s, pdl);
        else launch_m<1, 1>(a, G, s, pdl);
    } else {
        if (q4) launch_m<0, 2>(a, G, s, pdl);
        else launch_m<1, 2>(a, G, s, pdl);
    }
}

}  // namespace k
}  // namespace gcb
