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
#include <cooperative_groups.h>

#include <cstdio>
#include <cstdlib>
#include <map>
#include <mutex>
#include <stdexcept>
#include <string>
#include <utility>

#include "../gc_fused.h"
#include "../gc_kernels.h"
#include "gc_flash_dev.cuh"
#include "gc_math.cuh"
#include "gc_tma.cuh"

namespace gcb {
namespace k {

namespace {

constexpr int CH = FL_CH;  // keys per chunk (the order's chunk size)
constexpr int MAXD_ALL = 256;  // head sizes up to 256 here (D % 32 == 0); others use the generic kernel
constexpr int WPH = 4;     // warps per query head
constexpr int MAXG = 4;    // query heads per CTA (larger GQA groups loop)
constexpr int RQ = 16;     // query rows per CTA (prefill): the chunk's K/V rows are staged once for all

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
    float *out;      // [D, oH, Sq, B] rows of this launch (heads 0..H-1 of each row)
    int64_t oH;      // heads per output row: H, or more when this launch writes a slice of the heads
    int *counters;   // [B][Sq][Hkv], zero between launches
    int *err;
    int64_t nch;
    uint64_t *trace;  // [CTA][8] %globaltimer stamps, or null: start, staged, past the wait, K/V landed,
                      // done, chunk computed, past the arrival counter (the cluster kernel: past the
                      // cluster barrier), and done again in the cluster kernel only
    char *act_out;    // one query row: its Q8_0 blocks in the GEMV staging layout (K = H x D), or null
    const int32_t *kv_pos;  // cluster kernel: [B] positions the previous kernel writes (early K/V copies)
    int64_t cpc;            // multi-chunk kernel: consecutive chunks per CTA
    size_t merge_smem;      // multi-chunk kernel: dynamic shared memory the merging CTA may stage partials in
};

template <int MAXD>
__global__ void __launch_bounds__(MAXG * WPH * 32, 2) flash_split_kernel(SplitArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int D = (int)a.D;
    __shared__ uint64_t bar;
    __shared__ int last;
    __half *Ks = (__half *)smem;                  // [CH][D]
    __half *Vs = Ks + CH * D;                     // [CH][D]
    float *sc = (float *)(Vs + CH * D);           // [MAXG][CH] scores
    float *ps = sc + MAXG * CH;                   // [warps][CH] probabilities
    const int64_t Gq = a.H / a.Hkv;
    float *qs = ps + MAXG * WPH * CH;             // [G][D] query rows
    float *ms = qs + Gq * D;                      // [G][CH] mask values

    const int64_t ch = blockIdx.x;
    const int64_t hk = blockIdx.y % a.Hkv, b = blockIdx.y / a.Hkv;
    const int64_t iq0 = blockIdx.z * (int64_t)RQ, iq1 = min(iq0 + RQ, a.Sq);
    const int64_t j0 = ch * CH;
    const int n = (int)min((int64_t)CH, a.nkv - j0);
    const int warp = threadIdx.x >> 5;
    const int64_t G = a.H / a.Hkv;
    const float ninf = -__int_as_float(0x7f800000);

    const int64_t cta_id = blockIdx.x + (int64_t)gridDim.x * (blockIdx.y + (int64_t)gridDim.y * blockIdx.z);
    uint64_t *stamps = a.trace && threadIdx.x == 0 ? a.trace + cta_id * 8 : nullptr;
    if (stamps) stamps[0] = global_ns();
    pdl_trigger();  // the next GEMV may start streaming its weights now; it waits for this grid to finish before reading
    pdl_wait();     // the KV cache row of this step was written by the previous kernel
    if (stamps) stamps[2] = global_ns();
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
    } else {
        for (int t = threadIdx.x; t < n * D / 2; t += blockDim.x) {
            const int r = t / (D / 2), w = t % (D / 2);
            ((uint32_t *)(Ks + r * D))[w] = ((const uint32_t *)(a.k + hk * a.knb2 + b * a.knb3 + (j0 + r) * a.knb1))[w];
            ((uint32_t *)(Vs + r * D))[w] = ((const uint32_t *)(a.v + hk * a.vnb2 + b * a.vnb3 + (j0 + r) * a.vnb1))[w];
        }
    }
    // The chunk's K/V rows stay in shared memory for every query row of this CTA; each row's
    // partials are exactly the one-row kernel's (same chunk, same order).
    for (int64_t iq = iq0; iq < iq1; iq++) {
        FlashChunk fc;
        fc.q = a.q + iq * a.qnb1 + (hk * G) * a.qnb2 + b * a.qnb3;
        fc.qnb0 = a.qnb0;
        fc.qnbh = a.qnb2;
        fc.mask = a.mask ? a.mask + iq * a.mnb1 + ((hk * G) % a.mne2) * a.mnb2 + (b % a.mne3) * a.mnb3 + j0 * 2 : nullptr;
        fc.mne2 = a.mne2;
        fc.mnbh = a.mnb2;
        fc.hbase = (int)(hk * G);
        fc.scale = a.scale;
        fc.D = D;
        fc.n = n;
        fc.G = (int)G;
        fc.part = a.part + ((((b * a.Sq + iq) * a.H + hk * G) * a.nch + ch) * (a.D + 2));
        fc.pstride = a.nch * (a.D + 2);
        flash_stage(fc, qs, ms, threadIdx.x, blockDim.x);  // the first row: while the copies are in flight
        if (stamps && iq == iq0) stamps[1] = global_ns();
        // a chunk whose keys the mask hides from every head of this row contributes nothing: its
        // partial is (m = -inf, l = 0), which the merge skips, without the arithmetic
        int live = !fc.mask;
        for (int i = threadIdx.x; !live && i < (int)G * CH; i += blockDim.x) live = (i % CH) < n && ms[i] != ninf;
        live = __syncthreads_or(live);
        if (iq == iq0 && rows_contig && !__syncthreads_and(mbar_wait(&bar, 0))) {  // every thread leaves together
            // the error word, and NaN in the output rows of this CTA's heads (this chunk's partials
            // never arrive, so nothing else writes them): a caller that cannot read the error word
            // (the allocation-free entry point) still sees the failure
            for (int64_t r = iq0; r < iq1; r++)
                for (int64_t i = threadIdx.x; i < G * a.D; i += blockDim.x)
                    a.out[a.D * (hk * G + i / a.D + a.oH * (r + a.Sq * b)) + i % a.D] = __int_as_float(0x7fc00000);
            if (threadIdx.x == 0 && a.err) atomicExch(a.err, 2);
            return;
        }
        if (stamps && iq == iq0) stamps[3] = global_ns();
        if (live) {
            const int nslots = (int)(blockDim.x / 32) / WPH;
            flash_chunk<WPH, MAXD>(fc, Ks, Vs, qs, ms, sc, ps, nslots, SyncCta());  // MAXD is the head size
        } else if (threadIdx.x < G) {
            fc.part[threadIdx.x * fc.pstride] = ninf;
            fc.part[threadIdx.x * fc.pstride + 1] = 0.0f;
        }

        // the last CTA of this (batch, query row, K/V head) merges every chunk of its heads
        if (stamps && iq == iq0) stamps[5] = global_ns();
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence();  // this CTA's partials (ordered before by the barrier) are visible first
            int *cnt = a.counters + (b * a.Sq + iq) * a.Hkv + hk;
            last = atomicAdd(cnt, 1) == (int)a.nch - 1;
            if (last) {
                *cnt = 0;
                __threadfence();
            }
        }
        __syncthreads();
        if (stamps && iq == iq0) stamps[6] = global_ns();
        if (last)
            for (int64_t g = warp; g < G; g += blockDim.x / 32) {
                const int64_t h = hk * G + g;
                const int64_t K = a.H * a.D;
                int8_t *qc = a.act_out ? (int8_t *)a.act_out + h * a.D : nullptr;
                float *qd = a.act_out ? (float *)(a.act_out + K) + h * a.D / 32 : nullptr;
                int *qs = a.act_out ? (int *)((float *)(a.act_out + K) + K / 32) + h * a.D / 32 : nullptr;
                flash_merge<MAXD>(a.part + (((b * a.Sq + iq) * a.H + h) * a.nch) * (a.D + 2), (int)a.nch,
                                  a.out + a.D * (h + a.oH * (iq + a.Sq * b)), qc, qd, qs);
            }
        __syncthreads();  // qs / ms / sc / ps and `last` are reused by the next row
    }
    if (stamps) stamps[4] = global_ns();
}

// One query row per batch (decode; K/V rows contiguous) over many CTAs' worth of chunks: each CTA
// takes a.cpc consecutive chunks of one (K/V head, batch), the next chunk's K/V copy in flight
// (double buffer) while the current one is computed, each chunk's partial exactly the split
// kernel's; the last CTA of a (batch, K/V head) merges every chunk in chunk order. Used when the
// cluster kernel would need more CTAs than fit at once (batched decode), so each CTA's fixed costs
// (copy latency, barriers, the arrival counter) are paid once per a.cpc chunks.
template <int MAXD>
__global__ void __launch_bounds__(MAXG * WPH * 32, 2) flash_multi_kernel(SplitArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int D = (int)a.D;
    __shared__ uint64_t bar[2];
    __shared__ int last;
    __half *Kb[2], *Vb[2];
    Kb[0] = (__half *)smem;
    Vb[0] = Kb[0] + CH * D;
    Kb[1] = Vb[0] + CH * D;
    Vb[1] = Kb[1] + CH * D;
    float *sc = (float *)(Vb[1] + CH * D);
    float *ps = sc + MAXG * CH;
    const int64_t G = a.H / a.Hkv;
    float *qs = ps + MAXG * WPH * CH;
    float *ms = qs + G * D;
    const int64_t hk = blockIdx.y % a.Hkv, b = blockIdx.y / a.Hkv;
    const int64_t c0 = blockIdx.x * a.cpc, c1 = min(a.nch, c0 + a.cpc);
    const int warp = threadIdx.x >> 5;
    const float ninf = -__int_as_float(0x7f800000);
    const int64_t cta_id = blockIdx.x + (int64_t)gridDim.x * blockIdx.y;
    uint64_t *stamps = a.trace && threadIdx.x == 0 ? a.trace + cta_id * 8 : nullptr;
    if (stamps) stamps[0] = global_ns();
    pdl_trigger();
    pdl_wait();
    if (stamps) stamps[2] = global_ns();
    auto issue = [&](int64_t c, int buf) {
        const int64_t j0 = c * CH;
        const uint32_t bytes = (uint32_t)(min((int64_t)CH, a.nkv - j0) * D * 2);
        mbar_expect_tx(&bar[buf], 2 * bytes);
        bulk_g2s(Kb[buf], a.k + hk * a.knb2 + b * a.knb3 + j0 * a.knb1, bytes, &bar[buf]);
        bulk_g2s(Vb[buf], a.v + hk * a.vnb2 + b * a.vnb3 + j0 * a.vnb1, bytes, &bar[buf]);
    };
    if (threadIdx.x == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        mbar_fence_init();
        if (c0 < c1) issue(c0, 0);
    }
    __syncthreads();
    for (int64_t c = c0; c < c1; c++) {
        const int ci = (int)(c - c0), buf = ci & 1;
        // the other buffer was last read by chunk c - 1, whose iteration ended in a barrier
        if (threadIdx.x == 0 && c + 1 < c1) issue(c + 1, buf ^ 1);
        const int64_t j0 = c * CH;
        const int n = (int)min((int64_t)CH, a.nkv - j0);
        FlashChunk fc;
        fc.q = a.q + (hk * G) * a.qnb2 + b * a.qnb3;
        fc.qnb0 = a.qnb0;
        fc.qnbh = a.qnb2;
        fc.mask = a.mask ? a.mask + ((hk * G) % a.mne2) * a.mnb2 + (b % a.mne3) * a.mnb3 + j0 * 2 : nullptr;
        fc.mne2 = a.mne2;
        fc.mnbh = a.mnb2;
        fc.hbase = (int)(hk * G);
        fc.scale = a.scale;
        fc.D = D;
        fc.n = n;
        fc.G = (int)G;
        fc.part = a.part + (((b * a.H + hk * G) * a.nch + c) * (a.D + 2));
        fc.pstride = a.nch * (a.D + 2);
        flash_stage(fc, qs, ms, threadIdx.x, blockDim.x);
        int live = !fc.mask;
        for (int i = threadIdx.x; !live && i < (int)G * CH; i += blockDim.x) live = (i % CH) < n && ms[i] != ninf;
        live = __syncthreads_or(live);
        const bool landed = __syncthreads_and(mbar_wait(&bar[buf], (uint32_t)((ci >> 1) & 1)));
        if (!landed) {  // a NaN partial: the merged rows come out NaN; the error word says why
            if (threadIdx.x < G) {
                fc.part[threadIdx.x * fc.pstride] = __int_as_float(0x7fc00000);
                fc.part[threadIdx.x * fc.pstride + 1] = 0.0f;
            }
            if (threadIdx.x == 0 && a.err) atomicExch(a.err, 2);
        } else if (live) {
            const int nslots = (int)(blockDim.x / 32) / WPH;
            flash_chunk<WPH, MAXD>(fc, Kb[buf], Vb[buf], qs, ms, sc, ps, nslots, SyncCta());
        } else if (threadIdx.x < G) {
            fc.part[threadIdx.x * fc.pstride] = ninf;
            fc.part[threadIdx.x * fc.pstride + 1] = 0.0f;
        }
        __syncthreads();  // buffers, qs / ms / sc / ps free for the next chunk
    }
    if (stamps) stamps[5] = global_ns();
    if (threadIdx.x == 0) {
        __threadfence();  // this CTA's partials (ordered before by the barrier) are visible first
        int *cnt = a.counters + b * a.Hkv + hk;
        last = atomicAdd(cnt, 1) == (int)gridDim.x - 1;
        if (last) {
            *cnt = 0;
            __threadfence();
        }
    }
    __syncthreads();
    if (stamps) stamps[6] = global_ns();
    if (last) {
        // every chunk partial of this (batch, K/V head) into shared memory at once (all warps, many
        // loads in flight), then the in-order merge from there: same arithmetic, no per-batch L2
        // round trips in the merging warps
        const int64_t plen = G * a.nch * (a.D + 2);
        const float *pg = a.part + ((b * a.H + hk * G) * a.nch) * (a.D + 2);
        const bool staged = (size_t)plen * 4 <= a.merge_smem;
        float *pl = (float *)smem;
        if (staged) {
            for (int64_t i = threadIdx.x; i < plen; i += blockDim.x) pl[i] = __ldcg(pg + i);
            __syncthreads();
        }
        for (int64_t g = warp; g < G; g += blockDim.x / 32) {
            const int64_t h = hk * G + g;
            const int64_t K = a.H * a.D;
            int8_t *qc = a.act_out ? (int8_t *)a.act_out + h * a.D : nullptr;
            float *qd = a.act_out ? (float *)(a.act_out + K) + h * a.D / 32 : nullptr;
            int *qs8 = a.act_out ? (int *)((float *)(a.act_out + K) + K / 32) + h * a.D / 32 : nullptr;
            float *orow = a.out + a.D * (h + a.oH * b);
            if (staged)
                flash_merge<MAXD, true>(pl + g * a.nch * (a.D + 2), (int)a.nch, orow, qc, qd, qs8);
            else
                flash_merge<MAXD>(pg + g * a.nch * (a.D + 2), (int)a.nch, orow, qc, qd, qs8);
        }
    }
    if (stamps) stamps[4] = global_ns();
}

// One query row of decode (Sq == 1, K/V rows contiguous, at most FL_CLUSTER_MAX chunks): one thread
// block cluster per (K/V head, batch), one CTA per 64-key chunk. Each CTA computes its chunk
// partials exactly as the split kernel does, but writes them into the shared memory of the
// cluster's rank-0 CTA (distributed shared memory); after a cluster barrier rank 0 merges them in
// chunk order from its own shared memory. No global scratch, counters or fences: the cross-CTA
// merge costs one cluster barrier. A chunk whose K/V copy timed out writes a NaN partial (the
// merged rows come out NaN) and sets the error word; every CTA still reaches both barriers.
constexpr int FL_CLUSTER_MAX = 16;

template <int MAXD>
__global__ void __launch_bounds__(MAXG * WPH * 32, 2) flash_cluster_kernel(SplitArgs a) {
    namespace cg = cooperative_groups;
    extern __shared__ __align__(128) unsigned char smem[];
    const cg::cluster_group cluster = cg::this_cluster();
    const int D = (int)a.D;
    __shared__ uint64_t bar;
    __half *Ks = (__half *)smem;
    __half *Vs = Ks + CH * D;
    float *sc = (float *)(Vs + CH * D);
    float *ps = sc + MAXG * CH;
    const int64_t G = a.H / a.Hkv;
    float *qs = ps + MAXG * WPH * CH;
    float *ms = qs + G * D;
    float *parts = ms + G * CH;  // rank 0: [G][nch][D + 2] partials of every chunk
    const int64_t ch = blockIdx.x;
    const int64_t hk = blockIdx.y % a.Hkv, b = blockIdx.y / a.Hkv;
    const int64_t j0 = ch * CH;
    const int n = (int)min((int64_t)CH, a.nkv - j0);
    const int warp = threadIdx.x >> 5;
    const float ninf = -__int_as_float(0x7f800000);
    const int64_t cta_id = blockIdx.x + (int64_t)gridDim.x * blockIdx.y;
    uint64_t *stamps = a.trace && threadIdx.x == 0 ? a.trace + cta_id * 8 : nullptr;
    if (stamps) stamps[0] = global_ns();
    pdl_trigger();
    const bool early = a.kv_pos != nullptr;
    auto copy_kv = [&] {
        mbar_init(&bar, 1);
        mbar_fence_init();
        const uint32_t bytes = (uint32_t)(n * D * 2);
        mbar_expect_tx(&bar, 2 * bytes);
        bulk_g2s(Ks, a.k + hk * a.knb2 + b * a.knb3 + j0 * a.knb1, bytes, &bar);
        bulk_g2s(Vs, a.v + hk * a.vnb2 + b * a.vnb3 + j0 * a.vnb1, bytes, &bar);
    };
    if (early && threadIdx.x == 0) copy_kv();  // rows of earlier steps: complete before this launch
    pdl_wait();
    if (stamps) stamps[2] = global_ns();
    if (!early && threadIdx.x == 0) copy_kv();
    cluster.sync();  // every CTA of the cluster has started: its shared memory may be written
    FlashChunk fc;
    fc.q = a.q + (hk * G) * a.qnb2 + b * a.qnb3;
    fc.qnb0 = a.qnb0;
    fc.qnbh = a.qnb2;
    fc.mask = a.mask ? a.mask + ((hk * G) % a.mne2) * a.mnb2 + (b % a.mne3) * a.mnb3 + j0 * 2 : nullptr;
    fc.mne2 = a.mne2;
    fc.mnbh = a.mnb2;
    fc.hbase = (int)(hk * G);
    fc.scale = a.scale;
    fc.D = D;
    fc.n = n;
    fc.G = (int)G;
    fc.part = cluster.map_shared_rank(parts, 0) + ch * (a.D + 2);
    fc.pstride = a.nch * (a.D + 2);
    flash_stage(fc, qs, ms, threadIdx.x, blockDim.x);
    if (stamps) stamps[1] = global_ns();
    int live = !fc.mask;
    for (int i = threadIdx.x; !live && i < (int)G * CH; i += blockDim.x) live = (i % CH) < n && ms[i] != ninf;
    live = __syncthreads_or(live);
    const bool landed = __syncthreads_and(mbar_wait(&bar, 0));
    if (early && landed) {
        // the row the previous kernel wrote may have been copied before it was written: read it
        // again (from L2: that kernel has completed)
        const int64_t p = (int64_t)a.kv_pos[b] - j0;
        if (p >= 0 && p < n) {
            const int w = D / 2;  // 32-bit words per row
            for (int i = threadIdx.x; i < 2 * w; i += blockDim.x) {
                const bool isv = i >= w;
                const int c = isv ? i - w : i;
                const char *src = isv ? a.v + hk * a.vnb2 + b * a.vnb3 + (j0 + p) * a.vnb1
                                      : a.k + hk * a.knb2 + b * a.knb3 + (j0 + p) * a.knb1;
                ((uint32_t *)((isv ? Vs : Ks) + p * D))[c] = __ldcg((const unsigned int *)src + c);
            }
        }
        __syncthreads();
    }
    if (stamps) stamps[3] = global_ns();
    if (!landed) {
        if (threadIdx.x < G) {
            fc.part[threadIdx.x * fc.pstride] = __int_as_float(0x7fc00000);
            fc.part[threadIdx.x * fc.pstride + 1] = 0.0f;
        }
        if (threadIdx.x == 0 && a.err) atomicExch(a.err, 2);
    } else if (live) {
        const int nslots = (int)(blockDim.x / 32) / WPH;
        flash_chunk<WPH, MAXD>(fc, Ks, Vs, qs, ms, sc, ps, nslots, SyncCta());
    } else if (threadIdx.x < G) {
        fc.part[threadIdx.x * fc.pstride] = ninf;
        fc.part[threadIdx.x * fc.pstride + 1] = 0.0f;
    }
    if (stamps) stamps[5] = global_ns();
    cluster.sync();  // every partial is in rank 0's shared memory
    if (stamps) stamps[6] = global_ns();
    if (cluster.block_rank() == 0)
        for (int64_t g = warp; g < G; g += blockDim.x / 32) {
            const int64_t h = hk * G + g;
            const int64_t K = a.H * a.D;
            int8_t *qc = a.act_out ? (int8_t *)a.act_out + h * a.D : nullptr;
            float *qd = a.act_out ? (float *)(a.act_out + K) + h * a.D / 32 : nullptr;
            int *qs8 = a.act_out ? (int *)((float *)(a.act_out + K) + K / 32) + h * a.D / 32 : nullptr;
            flash_merge<MAXD, true>(parts + g * a.nch * (a.D + 2), (int)a.nch, a.out + a.D * (h + a.oH * b * a.Sq), qc, qd,
                                    qs8);
        }
    if (stamps) stamps[4] = stamps[7] = global_ns();  // [7]: set only by the cluster kernel
}

constexpr size_t kMaxPartBytes = 256u << 20;  // scratch for chunk partials per row group

bool flash_cluster_enabled() {
    static const bool on = [] {
        const char *e = std::getenv("GCB_ATTN_CLUSTER");
        return !e || std::atoi(e) != 0;
    }();
    return on;
}

// Whether clusters of `size` CTAs of this kernel with this shared memory can be resident (asked
// once per kernel, size and shared-memory size; sizes above 8 need the non-portable attribute).
bool flash_cluster_fits(void (*kern)(SplitArgs), cudaLaunchConfig_t cfg, size_t smem, int size) {
    static std::mutex mu;
    static std::map<std::pair<void *, std::pair<size_t, int>>, bool> known;
    std::lock_guard<std::mutex> lk(mu);
    const auto key = std::make_pair((void *)kern, std::make_pair(smem, size));
    auto it = known.find(key);
    if (it != known.end()) return it->second;
    // the kernel's limit, not this size: one instantiation serves configurations of several sizes.
    // The limit is the device's opt-in maximum less the kernel's static shared memory (asking for
    // the whole 227 KiB fails, and the cluster kernel then never ran).
    cudaFuncAttributes fa{};
    int dev = 0, optin = 0;
    bool ok = cudaFuncGetAttributes(&fa, kern) == cudaSuccess && cudaGetDevice(&dev) == cudaSuccess &&
              cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) == cudaSuccess;
    const size_t maxdyn = ok && (size_t)optin > fa.sharedSizeBytes ? (size_t)optin - fa.sharedSizeBytes : 0;
    ok = ok && smem <= maxdyn;
    if (ok) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)maxdyn);
        if (e == cudaSuccess && size > 8) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess)
            std::fprintf(stderr, "ggml_compiler_b200: cluster attention (%d CTAs) unavailable: %s\n", size, cudaGetErrorString(e));
        ok = e == cudaSuccess;
    }
    // the occupancy query takes the cluster shape alone (with the launch's programmatic-serialization
    // attribute in the list it fails, which read as "does not fit")
    cudaLaunchAttribute ca[1];
    ca[0].id = cudaLaunchAttributeClusterDimension;
    ca[0].val.clusterDim.x = (unsigned)size;
    ca[0].val.clusterDim.y = 1;
    ca[0].val.clusterDim.z = 1;
    cfg.attrs = ca;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (ok) {
        const cudaError_t e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
        if (e != cudaSuccess)  // not a "does not fit" answer: say why the split kernel runs instead
            std::fprintf(stderr, "ggml_compiler_b200: cluster attention (%d CTAs) unavailable: %s\n", size, cudaGetErrorString(e));
        ok = e == cudaSuccess && clusters >= 1;
    }
    cudaGetLastError();
    known[key] = ok;
    return ok;
}

// The cluster kernel for one decode row, if it applies and clusters of a.nch CTAs fit: launched
// (launch) or only checked, which caches the occupancy answer outside any stream capture.
bool cluster_decode(const SplitArgs &a, size_t smem, int threads, cudaStream_t s, bool launch) {
    const bool rows_contig = a.knb1 == 2 * a.D && a.vnb1 == 2 * a.D &&
                             (((uintptr_t)a.k | (uintptr_t)a.v | (uintptr_t)a.knb2 | (uintptr_t)a.vnb2) % 16) == 0;
    if (a.nch < 2 || a.nch > FL_CLUSTER_MAX || !rows_contig || !flash_cluster_enabled()) return false;
    // more CTAs than two per SM (batched decode): the multi-chunk kernel pays each CTA's fixed costs
    // once per several chunks instead
    if (a.nch * a.Hkv * a.B > 2 * (int64_t)num_sms()) return false;
    void (*ck)(SplitArgs) = nullptr;
    switch (a.D) {
        case 32: ck = flash_cluster_kernel<32>; break;
        case 64: ck = flash_cluster_kernel<64>; break;
        case 96: ck = flash_cluster_kernel<96>; break;
        case 128: ck = flash_cluster_kernel<128>; break;
        case 160: ck = flash_cluster_kernel<160>; break;
        case 192: ck = flash_cluster_kernel<192>; break;
        case 224: ck = flash_cluster_kernel<224>; break;
        case 256: ck = flash_cluster_kernel<256>; break;
        default: return false;
    }
    const int64_t G = a.H / a.Hkv;
    const size_t csmem = smem + (size_t)G * a.nch * (a.D + 2) * 4;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)a.nch, (unsigned)(a.Hkv * a.B), 1);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = csmem;
    cfg.stream = s;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    at[1].id = cudaLaunchAttributeClusterDimension;
    at[1].val.clusterDim.x = (unsigned)a.nch;
    at[1].val.clusterDim.y = 1;
    at[1].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 2;
    if (!flash_cluster_fits(ck, cfg, csmem, (int)a.nch)) return false;
    if (!launch) return true;
    SplitArgs g = a;
    g.Sq = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, ck, g);
    if (e != cudaSuccess) throw std::runtime_error(std::string("CUDA launch of flash_cluster failed: ") + cudaGetErrorString(e));
    return true;
}

}  // namespace

bool flash_split_ok(const TD &q) { return q.ne[0] <= MAXD_ALL && q.ne[0] % 32 == 0; }

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

size_t flash_split_ctas(const TD &q, const TD &kk) {
    return (size_t)((kk.ne[1] + CH - 1) / CH) * (size_t)(kk.ne[2] * q.ne[3]) * (size_t)((q.ne[1] + RQ - 1) / RQ);
}

bool flash_split_prepare(const TD &q, const TD &kk, const TD &v, const TD &out) {
    if (q.ne[1] != 1 || flash_prefill_ok(q, kk, v, out) || !flash_split_ok(q)) return false;
    SplitArgs a{};
    a.D = q.ne[0];
    a.H = q.ne[2];
    a.B = q.ne[3];
    a.k = kk.data;
    a.v = v.data;
    a.nkv = kk.ne[1];
    a.Hkv = kk.ne[2];
    a.knb1 = kk.nb[1];
    a.knb2 = kk.nb[2];
    a.vnb1 = v.nb[1];
    a.vnb2 = v.nb[2];
    a.nch = (a.nkv + CH - 1) / CH;
    const int64_t G = a.H / a.Hkv;
    const int threads = (int)std::min<int64_t>(G, MAXG) * WPH * 32;
    const size_t smem = (size_t)CH * a.D * 2 * 2 + (size_t)MAXG * CH * 4 + (size_t)MAXG * WPH * CH * 4 +
                        (size_t)G * (a.D + CH) * 4;
    return cluster_decode(a, smem, threads, nullptr, false);
}

void flash_attn_split(const TD &q, const TD &kk, const TD &v, const TD *mask, const TD &out, float scale, void *scratch,
                      int *counters, int *err, cudaStream_t s, uint64_t *trace, char *act_out, const int32_t *kv_pos,
                      bool prefill_tc) {
    if (flash_prefill_ok(q, kk, v, out)) {
        if (prefill_tc) flash_prefill_tc(q, kk, v, mask, out, scale, s);
        else flash_prefill(q, kk, v, mask, out, scale, err, s);
        return;
    }
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
    a.oH = out.nb[2] / (4 * a.D);
    if (out.nb[0] != 4 || out.nb[1] != 4 * a.D || out.nb[2] % (4 * a.D) || a.oH < a.H || out.nb[3] != out.nb[2] * q.ne[1])
        throw std::runtime_error("flash_split: output rows must be [D, heads] blocks of f32 with contiguous heads");
    a.nch = (a.nkv + CH - 1) / CH;
    a.part = (float *)scratch;
    a.counters = counters;
    a.err = err;
    a.trace = trace;
    a.act_out = q.ne[1] == 1 && q.ne[3] == 1 ? act_out : nullptr;
    const int64_t G = a.H / a.Hkv;
    const int hslots = (int)std::min<int64_t>(G, MAXG);
    const int threads = hslots * WPH * 32;
    const size_t smem = (size_t)CH * a.D * 2 * 2 + (size_t)MAXG * CH * 4 + (size_t)MAXG * WPH * CH * 4 +
                        (size_t)G * (a.D + CH) * 4;
    void (*kern)(SplitArgs) = nullptr;  // one instantiation per head size
    switch (a.D) {
        case 32: kern = flash_split_kernel<32>; break;
        case 64: kern = flash_split_kernel<64>; break;
        case 96: kern = flash_split_kernel<96>; break;
        case 128: kern = flash_split_kernel<128>; break;
        case 160: kern = flash_split_kernel<160>; break;
        case 192: kern = flash_split_kernel<192>; break;
        case 224: kern = flash_split_kernel<224>; break;
        case 256: kern = flash_split_kernel<256>; break;
        default: throw std::runtime_error("flash_split: head size must be a multiple of 32 up to 256");
    }
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    const int64_t Sq = q.ne[1];
    if (Sq == 1) {
        SplitArgs c = a;
        c.mask = mask ? mask->data : nullptr;
        c.out = (float *)out.data;
        c.kv_pos = kv_pos;
        if (cluster_decode(c, smem, threads, s, true)) return;
        const bool rows_contig = a.knb1 == 2 * a.D && a.vnb1 == 2 * a.D &&
                                 (((uintptr_t)a.k | (uintptr_t)a.v | (uintptr_t)a.knb2 | (uintptr_t)a.vnb2 |
                                   (uintptr_t)a.knb3 | (uintptr_t)a.vnb3) % 16) == 0;
        const int64_t pairs = a.Hkv * a.B, wave = 4 * (int64_t)num_sms();  // two waves of two CTAs per SM
        if (rows_contig && a.nch >= 2 && (size_t)(a.H * a.B * a.nch * (a.D + 2)) * 4 <= kMaxPartBytes) {
            void (*mk)(SplitArgs) = nullptr;
            switch (a.D) {
                case 32: mk = flash_multi_kernel<32>; break;
                case 64: mk = flash_multi_kernel<64>; break;
                case 96: mk = flash_multi_kernel<96>; break;
                case 128: mk = flash_multi_kernel<128>; break;
                case 160: mk = flash_multi_kernel<160>; break;
                case 192: mk = flash_multi_kernel<192>; break;
                case 224: mk = flash_multi_kernel<224>; break;
                case 256: mk = flash_multi_kernel<256>; break;
                default: break;
            }
            if (mk) {
                SplitArgs g = c;
                g.Sq = 1;
                const size_t msmem = smem + (size_t)CH * a.D * 2 * 2;  // the second K/V buffer
                cudaFuncSetAttribute(mk, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
                g.merge_smem = msmem;
                // chunks per CTA: the fewest chunk-times over the waves the grid needs, given how many
                // CTAs are resident at once (fewer chunks per CTA on ties); without an occupancy
                // answer, two waves of two CTAs per SM
                int per_sm = 0;
                if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, mk, threads, msmem) != cudaSuccess) {
                    (void)cudaGetLastError();
                    per_sm = 0;
                }
                if (per_sm > 0) {
                    const int64_t slots = (int64_t)per_sm * num_sms();
                    int64_t best = -1, best_cost = 0;
                    for (int64_t cpc = 1; cpc <= a.nch; cpc++) {
                        const int64_t ncta = (a.nch + cpc - 1) / cpc * pairs;
                        const int64_t cost = (ncta + slots - 1) / slots * cpc;
                        if (best < 0 || cost < best_cost) best = cpc, best_cost = cost;
                    }
                    g.cpc = best;
                } else {
                    g.cpc = std::max<int64_t>(1, (a.nch * pairs + wave - 1) / wave);
                }
                cudaLaunchConfig_t cfg = {};
                cfg.gridDim = dim3((unsigned)((a.nch + g.cpc - 1) / g.cpc), (unsigned)pairs, 1);
                cfg.blockDim = dim3(threads);
                cfg.dynamicSmemBytes = msmem;
                cfg.stream = s;
                cudaLaunchAttribute at[1];
                at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
                at[0].val.programmaticStreamSerializationAllowed = 1;
                cfg.attrs = at;
                cfg.numAttrs = 1;
                const cudaError_t e = cudaLaunchKernelEx(&cfg, mk, g);
                if (e != cudaSuccess) throw std::runtime_error(std::string("CUDA launch of flash_multi failed: ") + cudaGetErrorString(e));
                return;
            }
        }
    }
    const size_t per_row = (size_t)(a.H * a.B * a.nch * (a.D + 2)) * 4;
    const int64_t rows_per = std::max<int64_t>(1, (int64_t)(kMaxPartBytes / per_row));
    if (a.B != 1 && rows_per < Sq) throw std::runtime_error("flash_split: batched prefill needs one row group");
    for (int64_t q0 = 0; q0 < Sq; q0 += rows_per) {
        const int64_t nq = std::min(rows_per, Sq - q0);
        SplitArgs g = a;
        g.q = a.q + q0 * a.qnb1;
        g.mask = mask ? mask->data + q0 * a.mnb1 : nullptr;
        g.Sq = nq;
        g.out = (float *)out.data + q0 * a.D * a.oH;  // out [D, oH, Sq, B]: rows q0.. (one batch)
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)a.nch, (unsigned)(a.Hkv * a.B), (unsigned)((nq + RQ - 1) / RQ));
        cfg.blockDim = dim3(threads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = s;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, g);
        if (e != cudaSuccess) throw std::runtime_error(std::string("CUDA launch of flash_split failed: ") + cudaGetErrorString(e));
    }
}

}  // namespace k
}  // namespace gcb
