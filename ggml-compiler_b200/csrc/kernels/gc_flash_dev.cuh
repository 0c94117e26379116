// Device parts of split-KV flash attention shared by the split kernel (gc_flash.cu) and the decode
// kernel's attention phases (gc_mega.cu): one 64-key chunk's partial for the query heads of one K/V
// head, and the in-order merge of a head's chunk partials.
//
// The arithmetic is the CPU checker's, in its order: the query rounded to f16; a score is the head
// dot in the lane-split order (lane l owns elements [l*D/32, (l+1)*D/32)), then the 32-lane
// butterfly, times scale, plus the mask; per chunk the max m, p_j = exp(s_j - m), l = sum of p_j and
// o = sum of p_j v_j in key order; chunks merged in order with weights exp(m_c - M). Only those
// sums are ordered: the loads feeding them are issued ahead.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

#include "gc_math.cuh"

namespace gcb {
namespace k {

constexpr int FL_CH = 64;  // keys per chunk (the order's chunk size)

struct FlashChunk {
    const char *q;        // query row of the group's first head
    int64_t qnb0, qnbh;   // bytes between a head's elements, between heads
    const char *mask;     // mask row of the group's first head at this chunk's first key, or null
    int64_t mne2, mnbh;   // mask heads (broadcast when 1) and bytes between them
    int hbase;            // global index of the group's first head (for the mask broadcast)
    float scale;
    int D, n, G;          // head size, keys in this chunk, heads in the group
    float *part;          // partial (m, l, o[D]) of the group's first head
    int64_t pstride;      // floats between the partials of consecutive heads
};

// Stages the group's query rows (rounded to f16) and this chunk's mask values into shared memory:
// qs [G][D], ms [G][FL_CH] (0 where there is no mask). Threads tid = 0 .. nthreads-1; the caller
// synchronises before flash_chunk reads them. Issued while the chunk's K/V copies are in flight.
__device__ inline void flash_stage(const FlashChunk &c, float *qs, float *ms, int tid, int nthreads) {
    for (int i = tid; i < c.G * c.D; i += nthreads) {
        const int g = i / c.D, e = i - g * c.D;
        qs[i] = __half2float(__float2half_rn(*(const float *)(c.q + g * c.qnbh + e * c.qnb0)));
    }
    for (int i = tid; i < c.G * FL_CH; i += nthreads) {
        const int g = i / FL_CH, j = i - g * FL_CH;
        float v = 0.0f;
        if (c.mask && j < c.n)
            v = __half2float(((const __half *)(c.mask + (int64_t)((c.hbase + g) % c.mne2 - c.hbase % c.mne2) * c.mnbh))[j]);
        ms[i] = v;
    }
}

// f16 operands straight into f32 arithmetic on the FMA pipe (no f16 -> f32 conversions, which run on
// the narrower XU pipe and bounded the chunk's time). fma.rn.f32.f16 forms the exact product of
// the two halves and adds c with one rounding: the same result as converting both halves to f32
// (exact) and one __fmaf_rn.
// acc = fma(q.lo, k.lo, acc), then fma(q.hi, k.hi, acc): two consecutive elements of a row each.
__device__ __forceinline__ float fma2_f16(uint32_t q2, uint32_t k2, float acc) {
    asm("{\n\t.reg .f16 ql, qh, kl, kh;\n\tmov.b32 {ql, qh}, %1;\n\tmov.b32 {kl, kh}, %2;\n\t"
        "fma.rn.f32.f16 %0, ql, kl, %0;\n\tfma.rn.f32.f16 %0, qh, kh, %0;\n\t}"
        : "+f"(acc)
        : "r"(q2), "r"(k2));
    return acc;
}

// An f16 value as f32, exactly, on the FMA pipe: h x 1 + (-0) (the -0 addend keeps the sign of a
// zero; every other value is the product itself).
__device__ __forceinline__ float f16_to_f32_fma(uint16_t h) {
    float d;
    asm("{\n\t.reg .f16 one;\n\tmov.b16 one, 0x3C00;\n\tfma.rn.f32.f16 %0, %1, one, %2;\n\t}"
        : "=f"(d)
        : "h"(h), "f"(-0.0f));
    return d;
}

// The lane's D/32 consecutive key elements (f16 in shared memory) as floats.
template <int CPL>
__device__ __forceinline__ void load_krow(const __half *kr, float (&kv)[CPL]) {
    if constexpr (CPL == 2) {
        const float2 f = __half22float2(*(const __half2 *)kr);
        kv[0] = f.x;
        kv[1] = f.y;
    } else if constexpr (CPL == 4) {
        const uint2 u = *(const uint2 *)kr;
        const float2 a = __half22float2(*(const __half2 *)&u.x), b = __half22float2(*(const __half2 *)&u.y);
        kv[0] = a.x;
        kv[1] = a.y;
        kv[2] = b.x;
        kv[3] = b.y;
    } else {
#pragma unroll
        for (int e = 0; e < CPL; e++) kv[e] = __half2float(kr[e]);
    }
}

// Scores of head-slot pass g0 against the chunk's K rows (Ks: [n][D] halves in shared memory), then
// each active warp's copy of the chunk's probabilities (ps). The query rows and mask values were
// staged by flash_stage (qs, ms). `nslots` head slots of WPH warps each (warps 0 .. nslots*WPH-1
// call this); sc: [nslots][FL_CH] scores, ps: [warps][FL_CH]. `bar` synchronises those warps; Ks is
// no longer read once this returns. D (head size) is a multiple of 32.
template <int WPH, int D, class Bar>
__device__ inline void flash_scores(const FlashChunk &c, const __half *Ks, const float *qs, const float *ms, float *sc,
                                    float *ps, int g0, int nslots, Bar bar) {
    constexpr int CPL = D / 32;  // elements of a lane in a dot
    const int n = c.n;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hw = warp / WPH, quarter = warp % WPH;
    const float ninf = -__int_as_float(0x7f800000);
    const int g = g0 + hw;
    const bool active = g < c.G;
    const int gg = active ? g : 0;
    float *sh = sc + hw * FL_CH;
    // the lane's query elements: as f16 pairs when a lane owns an even count (qs holds values already
    // rounded to f16, so the conversion back is exact), else as floats
    constexpr bool PAIRS = CPL % 2 == 0;
    constexpr int NQ2 = PAIRS ? CPL / 2 : 1;
    uint32_t q2[NQ2];
    float qv[CPL];
#pragma unroll
    for (int e = 0; e < CPL; e++) qv[e] = qs[gg * D + lane * CPL + e];
#pragma unroll
    for (int e = 0; e < NQ2; e++)
        q2[e] = PAIRS ? (uint32_t)__half_as_ushort(__float2half_rn(qv[2 * e])) |
                            ((uint32_t)__half_as_ushort(__float2half_rn(qv[2 * e + 1])) << 16)
                      : 0u;
    const float *mrow = ms + gg * FL_CH;
    // this warp's CH/WPH keys, 8 at a time
    for (int k0 = quarter * (FL_CH / WPH); k0 < (quarter + 1) * (FL_CH / WPH); k0 += 8) {
        float p[8];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int j = k0 + u;
            float acc = 0.0f;
            if (j < n) {
                if constexpr (PAIRS) {
                    const uint32_t *kr = (const uint32_t *)(Ks + j * D + lane * CPL);  // 4-byte aligned
#pragma unroll
                    for (int e = 0; e < CPL / 2; e++) acc = fma2_f16(q2[e], kr[e], acc);  // elements in order
                } else {
                    float kv[CPL];
                    load_krow<CPL>(Ks + j * D + lane * CPL, kv);
#pragma unroll
                    for (int e = 0; e < CPL; e++) acc = __fmaf_rn(qv[e], kv[e], acc);
                }
            }
            p[u] = acc;
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
            for (int u = 0; u < 8; u++) p[u] = __fadd_rn(p[u], __shfl_xor_sync(0xffffffffu, p[u], off));
        if (lane < 8 && active) {
            const int j = k0 + lane;
            float pu = p[0];
#pragma unroll
            for (int u = 1; u < 8; u++)
                if (lane == u) pu = p[u];
            float s = ninf;
            if (j < n) {
                s = __fmul_rn(pu, c.scale);
                s = __fadd_rn(s, mrow[j]);
            }
            sh[j] = s;
        }
    }
    bar();
    // chunk max and weights (every warp of the head computes the same values)
    const float s0 = sh[lane], s1 = sh[lane + 32];
    const float m = warp_max(fmaxf(s0, s1));
    if (active && m != ninf) {
        float *pw = ps + warp * FL_CH;
        pw[lane] = lane < n ? gc_expf(__fsub_rn(s0, m)) : 0.0f;
        pw[lane + 32] = lane + 32 < n ? gc_expf(__fsub_rn(s1, m)) : 0.0f;
    }
    __syncwarp();
}

// The chunk partial (m, l, o) of head-slot pass g0 from its scores (sc) and this warp's
// probabilities (ps) against the chunk's V rows (Vs: [n][D] halves in shared memory). Per warp: no
// barrier inside.
template <int WPH, int D>
__device__ inline void flash_values(const FlashChunk &c, const __half *Vs, const float *sc, const float *ps, int g0) {
    constexpr int OE = D / 32 / WPH > 0 ? D / 32 / WPH : 1;  // output elements per lane
    const int n = c.n;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hw = warp / WPH, quarter = warp % WPH;
    const float ninf = -__int_as_float(0x7f800000);
    const int g = g0 + hw;
    if (g >= c.G) return;
    const float *sh = sc + hw * FL_CH;
    const float m = warp_max(fmaxf(sh[lane], sh[lane + 32]));
    float *dst = c.part + g * c.pstride;
    if (m == ninf) {
        if (quarter == 0 && lane == 0) {
            dst[0] = ninf;
            dst[1] = 0.0f;
        }
        for (int d = quarter * 32 + lane; d < D; d += WPH * 32) dst[2 + d] = 0.0f;
        return;
    }
    const float *pw = ps + warp * FL_CH;
    float l = 0.0f, o[OE];
#pragma unroll
    for (int e = 0; e < OE; e++) o[e] = 0.0f;
    const __half *vcol = Vs + quarter * 32 + lane;
    // keys in order, four probabilities per (broadcast) load; p = 0 past the chunk's end
    for (int j0 = 0; j0 < n; j0 += 4) {
        const float4 p4 = *(const float4 *)(pw + j0);
        const float pj[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
        for (int u = 0; u < 4; u++) {
            if (j0 + u >= n) break;
            l = __fadd_rn(l, pj[u]);
            const __half *vr = vcol + (j0 + u) * D;
#pragma unroll
            for (int e = 0; e < OE; e++)
                if (D >= WPH * 32 || quarter * 32 < D)
                    o[e] = __fmaf_rn(pj[u], f16_to_f32_fma(__half_as_ushort(vr[e * WPH * 32])), o[e]);
        }
    }
    if (quarter == 0 && lane == 0) {
        dst[0] = m;
        dst[1] = l;
    }
#pragma unroll
    for (int e = 0; e < OE; e++)
        if (D >= WPH * 32 || quarter * 32 < D) dst[2 + quarter * 32 + lane + e * WPH * 32] = o[e];
}

// Both halves with K and V resident together (Ks, Vs), every head of the group.
template <int WPH, int D, class Bar>
__device__ inline void flash_chunk(const FlashChunk &c, const __half *Ks, const __half *Vs, const float *qs,
                                   const float *ms, float *sc, float *ps, int nslots, Bar bar) {
    for (int g0 = 0; g0 < c.G; g0 += nslots) {
        flash_scores<WPH, D>(c, Ks, qs, ms, sc, ps, g0, nslots, bar);
        flash_values<WPH, D>(c, Vs, sc, ps, g0);
        bar();
    }
}

// Synchronises every thread of the CTA (a flash_chunk barrier for kernels that run it with all warps).
struct SyncCta {
    __device__ void operator()() const { __syncthreads(); }
};

// One warp: merge head partials pp[c * (D + 2)], c < nch, in chunk order into orow[D]. The
// partials were written by other CTAs: they are read from L2 (ld.global.cg), all of a batch of
// chunks at once.
// LOCAL: the partials are in this CTA's shared memory (plain loads) rather than global memory
// written by other CTAs (L2 loads).
template <int D, bool LOCAL = false, int BATCH = 4>  // BATCH: chunks fetched at once
__device__ inline void flash_merge(const float *pp, int nch, float *orow, int8_t *qcodes = nullptr, float *qd = nullptr,
                                   int *qs8 = nullptr) {
    auto ld = [](const float *p) { return LOCAL ? *p : __ldcg(p); };
    constexpr int MAXD = D;
    const int lane = threadIdx.x & 31, cpl = D / 32;
    const float ninf = -__int_as_float(0x7f800000);
    float M = ninf, L = 0.0f, O[MAXD / 32];
#pragma unroll
    for (int e = 0; e < MAXD / 32; e++) O[e] = 0.0f;
    // the overall max first (one load per lane per 32 chunks), unless one batch holds every chunk
    if (nch > BATCH) {
        for (int c0 = 0; c0 < nch; c0 += 32)
            if (c0 + lane < nch) M = fmaxf(M, ld(pp + (int64_t)(c0 + lane) * (D + 2)));
        M = warp_max(M);
    }
    for (int c0 = 0; c0 < nch; c0 += BATCH) {
        float bm[BATCH], bl[BATCH], bo[BATCH][MAXD / 32];
#pragma unroll
        for (int u = 0; u < BATCH; u++) {
            const bool ok = c0 + u < nch;
            const float *pc = pp + (int64_t)(c0 + u) * (D + 2);
            bm[u] = ok ? ld(pc) : ninf;
            bl[u] = ok ? ld(pc + 1) : 0.0f;
#pragma unroll
            for (int e = 0; e < MAXD / 32; e++) bo[u][e] = (ok && e < cpl) ? ld(pc + 2 + lane * cpl + e) : 0.0f;
        }
        if (nch <= BATCH)
#pragma unroll
            for (int u = 0; u < BATCH; u++) M = fmaxf(M, bm[u]);
#pragma unroll
        for (int u = 0; u < BATCH; u++) {
            if (bm[u] == ninf) continue;
            const float wgt = gc_expf(__fsub_rn(bm[u], M));
            L = __fmaf_rn(wgt, bl[u], L);
#pragma unroll
            for (int e = 0; e < MAXD / 32; e++)
                if (e < cpl) O[e] = __fmaf_rn(wgt, bo[u][e], O[e]);
        }
    }
    const float inv = L == 0.0f ? 0.0f : __fdiv_rn(1.0f, L);
#pragma unroll
    for (int e = 0; e < MAXD / 32; e++)
        if (e < cpl) orow[lane * cpl + e] = __fmul_rn(O[e], inv);
    if (qcodes) {
        // the row's Q8_0 blocks for the GEMV that reads it (the GEMV prologue's rule: d = amax / 127
        // in fp16, codes = nearest-even(v * 127 / amax), 8 x the code sum); a block of 32 values is
        // 32 / cpl consecutive lanes
        constexpr int LPB = 32 / (MAXD / 32);
        float amax = 0.0f;
#pragma unroll
        for (int e = 0; e < MAXD / 32; e++) amax = fmaxf(amax, fabsf(__fmul_rn(O[e], inv)));
#pragma unroll
        for (int off = LPB / 2; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
        const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
        int sum = 0;
#pragma unroll
        for (int e = 0; e < MAXD / 32; e++) {
            const int q = __float2int_rn(__fmul_rn(__fmul_rn(O[e], inv), id));
            qcodes[lane * cpl + e] = (int8_t)q;
            sum += q;
        }
#pragma unroll
        for (int off = LPB / 2; off >= 1; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
        if (lane % LPB == 0) {
            qd[lane / LPB] = h2f(f2h(__fdiv_rn(amax, 127.0f)));
            qs8[lane / LPB] = 8 * sum;
        }
    }
}

}  // namespace k
}  // namespace gcb
