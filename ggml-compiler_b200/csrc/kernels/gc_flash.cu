// Split-KV flash attention over the f16 KV cache (decode and short prefills).
//
// Same result, bit for bit, as the generic flash_attn kernel and the CPU checker: the query rounded
// to f16; scores as head dots in the lane-split order (lane l owns elements [l*D/32, (l+1)*D/32),
// then the 32-lane butterfly), times scale, plus the mask; keys in chunks of 64 with the chunk max m,
// p_j = exp(s_j - m), l = sum p_j and o = sum p_j v_j in key order; chunks merged in order with
// weights exp(m_c - M).
//
// One CTA per (chunk, K/V head, batch, query row): the chunk's K and V rows (contiguous in the
// cache) land in shared memory with one bulk copy each. For each query head of the GQA group four
// warps work together: each scores 16 keys (8 keys in flight per lane), the four share the scores
// through shared memory, and each then accumulates a quarter of the head's elements over all 64 keys.
// The CTA writes its chunk partial (m, l, o[D]) to scratch; the last CTA to finish for a
// (query row, K/V head) merges every chunk in chunk order (an atomic arrival counter, reset by that
// CTA), so no second kernel is needed. Waits are bounded; a timeout sets the error word.
#include <stdexcept>
#include <string>

#include "../gc_kernels.h"
#include "gc_math.cuh"
#include "gc_tma.cuh"

namespace gcb {
namespace k {

namespace {

constexpr int CH = 64;     // keys per chunk (the order's chunk size)
constexpr int MAXD = 256;  // head sizes up to 256 here (D % 32 == 0); others use the generic kernel
constexpr int WPH = 4;     // warps per query head
constexpr int MAXG = 4;    // query heads per CTA (larger GQA groups loop)

struct SplitArgs {
    const char *q;
    int64_t D, Sq, H, B, qnb0, qnb1, qnb2, qnb3;
    const char *k;
    int64_t nkv, Hkv, knb1, knb2, knb3;
    const char *v;
    int64_t vnb1, vnb2, vnb3;
    const char *mask;
    int64_t mne2, mne3, mnb1, mnb2, mnb3;
    float scale;
    float *part;     // [B][Sq][H][nch][D + 2]
    float *out;      // [D, H, Sq, B] rows of this launch
    int *counters;   // [B][Sq][Hkv], zero between launches
    int *err;
    int64_t nch;
};

__global__ void __launch_bounds__(MAXG * WPH * 32) flash_split_kernel(SplitArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int D = (int)a.D, c = D / 32;
    __shared__ uint64_t bar;
    __shared__ int last;
    __half *Ks = (__half *)smem;                  // [CH][D]
    __half *Vs = Ks + CH * D;                     // [CH][D]
    float *sc = (float *)(Vs + CH * D);           // [MAXG][CH] scores

    const int64_t ch = blockIdx.x;
    const int64_t hk = blockIdx.y % a.Hkv, b = blockIdx.y / a.Hkv;
    const int64_t iq = blockIdx.z;
    const int64_t j0 = ch * CH;
    const int n = (int)min((int64_t)CH, a.nkv - j0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t G = a.H / a.Hkv;
    const int hw = warp / WPH, quarter = warp % WPH;  // head slot in the CTA, warp within the head
    const float ninf = -__int_as_float(0x7f800000);

    pdl_wait();  // the KV cache row of this step was written by the previous kernel
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        mbar_fence_init();
    }
    __syncthreads();
    const bool rows_contig = a.knb1 == 2 * a.D && a.vnb1 == 2 * a.D;
    if (rows_contig) {
        if (threadIdx.x == 0) {
            const uint32_t bytes = (uint32_t)(n * D * 2);
            mbar_expect_tx(&bar, 2 * bytes);
            bulk_g2s(Ks, a.k + hk * a.knb2 + b * a.knb3 + j0 * a.knb1, bytes, &bar);
            bulk_g2s(Vs, a.v + hk * a.vnb2 + b * a.vnb3 + j0 * a.vnb1, bytes, &bar);
        }
        if (!mbar_wait(&bar, 0)) {
            if (a.err) atomicExch(a.err, 2);
            return;
        }
    } else {
        for (int t = threadIdx.x; t < n * D / 2; t += blockDim.x) {
            const int r = t / (D / 2), w = t % (D / 2);
            ((uint32_t *)(Ks + r * D))[w] = ((const uint32_t *)(a.k + hk * a.knb2 + b * a.knb3 + (j0 + r) * a.knb1))[w];
            ((uint32_t *)(Vs + r * D))[w] = ((const uint32_t *)(a.v + hk * a.vnb2 + b * a.vnb3 + (j0 + r) * a.vnb1))[w];
        }
        __syncthreads();
    }

    for (int64_t g0 = 0; g0 < G; g0 += MAXG) {
        const int64_t g = g0 + hw;
        const bool active = g < G;
        const int64_t h = hk * G + (active ? g : 0);
        float *sh = sc + hw * CH;
        // query slice of this lane (f16-rounded), lane-split ownership
        float qv[MAXD / 32];
        const char *qrow = a.q + iq * a.qnb1 + h * a.qnb2 + b * a.qnb3;
#pragma unroll
        for (int e = 0; e < MAXD / 32; e++)
            qv[e] = e < c ? __half2float(__float2half_rn(*(const float *)(qrow + (lane * c + e) * a.qnb0))) : 0.0f;
        const __half *mrow = a.mask ? (const __half *)(a.mask + iq * a.mnb1 + (h % a.mne2) * a.mnb2 + (b % a.mne3) * a.mnb3)
                                    : nullptr;
        // scores: this warp's 16 keys, 8 at a time
        for (int k0 = quarter * (CH / WPH); k0 < (quarter + 1) * (CH / WPH); k0 += 8) {
            float p[8];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int j = k0 + u;
                float acc = 0.0f;
                if (j < n) {
                    const __half *kr = Ks + j * D + lane * c;
#pragma unroll
                    for (int e = 0; e < MAXD / 32; e++)
                        if (e < c) acc = __fmaf_rn(qv[e], __half2float(kr[e]), acc);
                }
                p[u] = acc;
            }
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
                for (int u = 0; u < 8; u++) p[u] = __fadd_rn(p[u], __shfl_xor_sync(0xffffffffu, p[u], off));
            if (lane < 8 && active) {
                const int j = k0 + lane;
                float s = ninf;
                float pu = p[0];
#pragma unroll
                for (int u = 1; u < 8; u++)
                    if (lane == u) pu = p[u];
                if (j < n) {
                    s = __fmul_rn(pu, a.scale);
                    s = __fadd_rn(s, mrow ? __half2float(mrow[j0 + j]) : 0.0f);
                }
                sh[j] = s;
            }
        }
        __syncthreads();
        // chunk max, weights, sum (every warp of the head computes the same values)
        const float s0 = sh[lane], s1 = sh[lane + 32];
        const float m = warp_max(fmaxf(s0, s1));
        float *dst = a.part + ((((b * a.Sq + iq) * a.H + h) * a.nch + ch) * (a.D + 2));
        if (active) {
            if (m == ninf) {
                if (quarter == 0 && lane == 0) {
                    dst[0] = ninf;
                    dst[1] = 0.0f;
                }
                for (int d = quarter * 32 + lane; d < D; d += WPH * 32) dst[2 + d] = 0.0f;
            } else {
                const float p0 = lane < n ? gc_expf(__fsub_rn(s0, m)) : 0.0f;
                const float p1 = lane + 32 < n ? gc_expf(__fsub_rn(s1, m)) : 0.0f;
                float l = 0.0f;
                float o[MAXD / 32 / WPH > 0 ? MAXD / 32 / WPH : 1];
                const int per = (D + WPH * 32 - 1) / (WPH * 32);  // elements per lane in this quarter
#pragma unroll
                for (int e = 0; e < (MAXD / 32 / WPH > 0 ? MAXD / 32 / WPH : 1); e++) o[e] = 0.0f;
                for (int j = 0; j < n; j++) {
                    const float pj = __shfl_sync(0xffffffffu, j < 32 ? p0 : p1, j & 31);
                    l = __fadd_rn(l, pj);
                    const __half *vr = Vs + j * D;
#pragma unroll
                    for (int e = 0; e < (MAXD / 32 / WPH > 0 ? MAXD / 32 / WPH : 1); e++) {
                        const int d = quarter * 32 + lane + e * WPH * 32;
                        if (e < per && d < D) o[e] = __fmaf_rn(pj, __half2float(vr[d]), o[e]);
                    }
                }
                if (quarter == 0 && lane == 0) {
                    dst[0] = m;
                    dst[1] = l;
                }
#pragma unroll
                for (int e = 0; e < (MAXD / 32 / WPH > 0 ? MAXD / 32 / WPH : 1); e++) {
                    const int d = quarter * 32 + lane + e * WPH * 32;
                    if (e < per && d < D) dst[2 + d] = o[e];
                }
            }
        }
        __syncthreads();
    }

    // last CTA of this (batch, query row, K/V head) merges every chunk of its heads
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        int *cnt = a.counters + (b * a.Sq + iq) * a.Hkv + hk;
        last = atomicAdd(cnt, 1) == (int)a.nch - 1;
        if (last) *cnt = 0;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int64_t g = warp; g < G; g += blockDim.x / 32) {
        const int64_t h = hk * G + g;
        const float *pp = a.part + (((b * a.Sq + iq) * a.H + h) * a.nch) * (a.D + 2);
        // the overall max: one load per lane per 32 chunks
        float M = ninf;
        for (int64_t c0 = 0; c0 < a.nch; c0 += 32)
            if (c0 + lane < a.nch) M = fmaxf(M, __ldcg(pp + (c0 + lane) * (a.D + 2)));
        M = warp_max(M);
        // chunks merged in order, their partials fetched 8 chunks at a time
        constexpr int BATCH = 8;
        float L = 0.0f, O[MAXD / 32];
#pragma unroll
        for (int e = 0; e < MAXD / 32; e++) O[e] = 0.0f;
        for (int64_t c0 = 0; c0 < a.nch; c0 += BATCH) {
            float bm[BATCH], bl[BATCH], bo[BATCH][MAXD / 32];
#pragma unroll
            for (int u = 0; u < BATCH; u++) {
                const bool ok = c0 + u < a.nch;
                const float *pc = pp + (c0 + u) * (a.D + 2);
                bm[u] = ok ? __ldcg(pc) : ninf;
                bl[u] = ok ? __ldcg(pc + 1) : 0.0f;
#pragma unroll
                for (int e = 0; e < MAXD / 32; e++) bo[u][e] = (ok && e < c) ? __ldcg(pc + 2 + lane * c + e) : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < BATCH; u++) {
                if (bm[u] == ninf) continue;
                const float wgt = gc_expf(__fsub_rn(bm[u], M));
                L = __fmaf_rn(wgt, bl[u], L);
#pragma unroll
                for (int e = 0; e < MAXD / 32; e++)
                    if (e < c) O[e] = __fmaf_rn(wgt, bo[u][e], O[e]);
            }
        }
        const float inv = L == 0.0f ? 0.0f : __fdiv_rn(1.0f, L);
        float *orow = a.out + a.D * (h + a.H * (iq + a.Sq * b));
#pragma unroll
        for (int e = 0; e < MAXD / 32; e++)
            if (e < c) orow[lane * c + e] = __fmul_rn(O[e], inv);
    }
}

constexpr size_t kMaxPartBytes = 64u << 20;  // scratch for chunk partials per row group

}  // namespace

bool flash_split_ok(const TD &q) { return q.ne[0] <= MAXD && q.ne[0] % 32 == 0; }

size_t flash_split_scratch_bytes(const TD &q, const TD &kk) {
    const int64_t nch = (kk.ne[1] + CH - 1) / CH;
    const size_t per_row = (size_t)(q.ne[2] * q.ne[3] * nch * (q.ne[0] + 2)) * 4;  // one query row, all heads
    const int64_t rows_per = std::max<int64_t>(1, (int64_t)(kMaxPartBytes / per_row));
    return per_row * (size_t)std::min<int64_t>(rows_per, q.ne[1]);
}

size_t flash_split_counters(const TD &q, const TD &kk) {
    const size_t per_row = (size_t)(q.ne[2] * q.ne[3] * ((kk.ne[1] + CH - 1) / CH) * (q.ne[0] + 2)) * 4;
    const int64_t rows_per = std::max<int64_t>(1, (int64_t)(kMaxPartBytes / per_row));
    return (size_t)(q.ne[3] * std::min<int64_t>(rows_per, q.ne[1]) * kk.ne[2]);
}

void flash_attn_split(const TD &q, const TD &kk, const TD &v, const TD *mask, const TD &out, float scale, void *scratch,
                      int *counters, int *err, cudaStream_t s) {
    SplitArgs a{};
    a.q = q.data;
    a.D = q.ne[0];
    a.H = q.ne[2];
    a.B = q.ne[3];
    a.qnb0 = q.nb[0];
    a.qnb1 = q.nb[1];
    a.qnb2 = q.nb[2];
    a.qnb3 = q.nb[3];
    a.k = kk.data;
    a.nkv = kk.ne[1];
    a.Hkv = kk.ne[2];
    a.knb1 = kk.nb[1];
    a.knb2 = kk.nb[2];
    a.knb3 = kk.nb[3];
    a.v = v.data;
    a.vnb1 = v.nb[1];
    a.vnb2 = v.nb[2];
    a.vnb3 = v.nb[3];
    a.mne2 = a.mne3 = 1;
    if (mask) {
        a.mne2 = mask->ne[2];
        a.mne3 = mask->ne[3];
        a.mnb1 = mask->nb[1];
        a.mnb2 = mask->nb[2];
        a.mnb3 = mask->nb[3];
    }
    a.scale = scale;
    a.nch = (a.nkv + CH - 1) / CH;
    a.part = (float *)scratch;
    a.counters = counters;
    a.err = err;
    const int64_t G = a.H / a.Hkv;
    const int hslots = (int)std::min<int64_t>(G, MAXG);
    const int threads = hslots * WPH * 32;
    const size_t smem = (size_t)CH * a.D * 2 * 2 + (size_t)MAXG * CH * 4;
    static bool attr_set = false;
    if (!attr_set) {
        cudaFuncSetAttribute(flash_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        attr_set = true;
    }
    const int64_t Sq = q.ne[1];
    const size_t per_row = (size_t)(a.H * a.B * a.nch * (a.D + 2)) * 4;
    const int64_t rows_per = std::max<int64_t>(1, (int64_t)(kMaxPartBytes / per_row));
    if (a.B != 1 && rows_per < Sq) throw std::runtime_error("flash_split: batched prefill needs one row group");
    for (int64_t q0 = 0; q0 < Sq; q0 += rows_per) {
        const int64_t nq = std::min(rows_per, Sq - q0);
        SplitArgs g = a;
        g.q = a.q + q0 * a.qnb1;
        g.mask = mask ? mask->data + q0 * a.mnb1 : nullptr;
        g.Sq = nq;
        g.out = (float *)out.data + q0 * a.D * a.H;  // out [D, H, Sq, B]: rows q0.. (one batch)
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)a.nch, (unsigned)(a.Hkv * a.B), (unsigned)nq);
        cfg.blockDim = dim3(threads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = s;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        const cudaError_t e = cudaLaunchKernelEx(&cfg, flash_split_kernel, g);
        if (e != cudaSuccess) throw std::runtime_error(std::string("CUDA launch of flash_split failed: ") + cudaGetErrorString(e));
    }
}

}  // namespace k
}  // namespace gcb
