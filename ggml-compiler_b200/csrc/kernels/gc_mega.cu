// The decode step as one persistent kernel: a cooperative launch (two CTAs per SM) runs a list of
// phases, the fused GEMV groups and the attention of every layer, separated by grid barriers.
//
// Per CTA, warp 8 is the producer: one lane streams the weight pieces of every GEMV phase, in phase
// order, into the shared-memory ring (gc_gemv_dev.cuh). Weights never depend on activations, so the
// stream runs ahead through barriers and attention phases, limited only by free ring slots. Warps
// 0-7 are the consumers: for a GEMV phase one tile row each, with the activation row in registers
// (the same consumer as the per-op kernel, gc_fused.cu); for an attention phase they work on
// (query row, K/V head, 64-key chunk) items as the split-KV flash kernel does (gc_flash_dev.cuh),
// two warps per query head. An item stages the chunk's K rows, then its V rows, in the buffer that
// holds the quantized activation during GEMV phases, so a CTA needs ~100 KB of shared memory and
// two fit an SM.
//
// Every phase computes exactly what the per-op kernels compute (same prologue, same block order,
// same epilogues, same attention chunking and merge), so results are bit-identical to them and to the
// CPU checker.
//
// Grid barrier: each CTA's consumers finish a phase, one thread fences and increments a global
// counter, then waits (bounded in time) until it reaches (phase) x (CTAs). The counter is zeroed by a
// memset before each launch. On a timeout the CTA records the error word (3), stops its consumers
// and lets the producer drain its copies in flight.
#include <stdexcept>
#include <string>

#include "../gc_kernels.h"
#include "gc_flash_dev.cuh"
#include "gc_gemv_dev.cuh"

namespace gcb {
namespace k {

int num_sms();

namespace {

constexpr int TEAMS = 1;
constexpr int CG = 1;                         // row groups per team in a GEMV chunk (gc_gemv_dev.cuh)
constexpr int NCW = 8 * TEAMS;                // consumer warps
constexpr int NCT = NCW * 32;                 // consumer threads
constexpr int NTHREADS = NCT + 32;            // + producer warp
constexpr int MAXNS = 8;
constexpr int CH = FL_CH;                     // attention chunk (keys)
constexpr int MAXD = 128;  // decode kernel head sizes (larger heads use the per-op kernels)
constexpr int WPH = 2;                        // warps per query head
constexpr int MAXG = NCW / WPH;               // query heads per attention item pass
constexpr int MAXGQ = MAXG;                   // query heads per K/V head (one pass)
constexpr size_t SMEM_LIMIT = 112 * 1024;     // dynamic shared memory of a CTA: two per SM

__device__ __forceinline__ int ld_acquire(const int *p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// All consumer threads of all CTAs: the previous phase's writes are visible after this.
// The KV-cache rows a phase writes with plain stores are read by the next phase's bulk copies, so
// both sides also fence between the generic and the async proxy.
__device__ inline bool grid_sync(int *ctr, int target, int *s_abort) {
    fence_proxy_async_global();
    named_bar(2, NCT);
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(ctr, 1);
        const uint64_t t0 = global_ns();
        while (ld_acquire(ctr) < target) {
            if (global_ns() - t0 > 2000000000ull) {
                *s_abort = 1;
                break;
            }
        }
        __threadfence();
        fence_proxy_async_global();
    }
    named_bar(2, NCT);
    return *s_abort == 0;
}

// Named barrier of the consumer warps (the flash_chunk barrier of attention phases).
struct SyncConsumers {
    __device__ void operator()() const { named_bar(3, NCT); }
};

// One attention item: chunk `ch` of K/V head `hk` for query row `iq` (split-KV flash attention,
// gc_flash_dev.cuh): the chunk's K rows, then its V rows, pass through the staging buffer KV; the
// last item of a (query row, K/V head) merges its heads' chunks.
__device__ inline bool attn_item(const MegaAttn &at, int iq, int hk, int ch, __half *KV, float *sc, float *ps, float *qs,
                                 float *ms, uint64_t *abar, uint32_t &aphase, int *s_last) {
    const int D = (int)at.D;
    const int j0 = ch * CH;
    const int n = (int)min((int64_t)CH, at.nkv - j0);
    const int warp = threadIdx.x >> 5;
    const int G = (int)(at.H / at.Hkv);
    const int nch = (int)((at.nkv + CH - 1) / CH);
    const uint32_t bytes = (uint32_t)(n * D * 2);

    FlashChunk fc;
    fc.q = (const char *)(at.q + iq * at.ldq + (int64_t)hk * G * D);
    fc.qnb0 = 4;
    fc.qnbh = 4 * (int64_t)D;
    fc.mask = at.mask ? (const char *)(at.mask + iq * at.mask_ld + j0) : nullptr;
    fc.mne2 = 1;
    fc.mnbh = 0;
    fc.hbase = hk * G;
    fc.scale = at.scale;
    fc.D = D;
    fc.n = n;
    fc.G = G;
    fc.part = at.part + (((int64_t)iq * at.H + (int64_t)hk * G) * nch + ch) * (D + 2);
    fc.pstride = (int64_t)nch * (D + 2);
    if (threadIdx.x == 0) {  // the buffer's earlier plain reads are ordered before the copy's writes
        fence_proxy_async_shared();
        mbar_expect_tx(abar, bytes);
        bulk_g2s(KV, at.k + hk * at.knb2 + (int64_t)j0 * at.knb1, bytes, abar);
    }
    flash_stage(fc, qs, ms, threadIdx.x, NCT);  // while the copy is in flight
    named_bar(3, NCT);
    if (threadIdx.x == 0) *s_last = mbar_wait(abar, aphase & 1) ? 1 : 0;  // one bounded wait, its outcome shared
    aphase++;
    named_bar(3, NCT);
    if (!*s_last) return false;  // uniform: every consumer thread leaves here
    if (D == 128) flash_scores<WPH, 128>(fc, KV, qs, ms, sc, ps, 0, MAXG, SyncConsumers());
    else flash_scores<WPH, 64>(fc, KV, qs, ms, sc, ps, 0, MAXG, SyncConsumers());
    // every consumer passed the barrier inside flash_scores: K is no longer read
    if (threadIdx.x == 0) {
        fence_proxy_async_shared();
        mbar_expect_tx(abar, bytes);
        bulk_g2s(KV, at.v + hk * at.vnb2 + (int64_t)j0 * at.vnb1, bytes, abar);
        *s_last = mbar_wait(abar, aphase & 1) ? 1 : 0;
    }
    aphase++;
    named_bar(3, NCT);
    if (!*s_last) return false;
    if (D == 128) flash_values<WPH, 128>(fc, KV, sc, ps, 0);
    else flash_values<WPH, 64>(fc, KV, sc, ps, 0);

    // the last item of this (query row, K/V head) merges its heads' chunks in chunk order
    named_bar(3, NCT);
    if (threadIdx.x == 0) {
        __threadfence();
        int *cnt = at.counters + iq * at.Hkv + hk;
        *s_last = atomicAdd(cnt, 1) == nch - 1;
        if (*s_last) {
            *cnt = 0;
            __threadfence();
        }
    }
    named_bar(3, NCT);
    if (!*s_last) return true;
    for (int g = warp; g < G; g += NCW) {
        const int64_t h = (int64_t)hk * G + g;
        if (D == 128) flash_merge<128, 4>(at.part + ((iq * at.H + h) * nch) * (D + 2), nch, at.out + at.D * (h + at.H * iq));
        else flash_merge<64, 4>(at.part + ((iq * at.H + h) * nch) * (D + 2), nch, at.out + at.D * (h + at.H * iq));
    }
    return true;
}

template <int QT, int M>
__global__ void __launch_bounds__(NTHREADS, 2) mega_kernel(const MegaPhase *phases, int nph, int log2ns, int slot_bytes,
                                                           size_t act_bytes, int attn_d, int *gbar, int *err,
                                                           uint64_t *trace) {
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t *full = (uint64_t *)smem;
    uint64_t *empty = full + MAXNS;
    uint64_t *abar = empty + MAXNS;
    double *red = (double *)(abar + 2);  // [256]
    int8_t *sq = (int8_t *)(red + 256);  // the activation (GEMV phases) or a K/V chunk (attention)
    float *sc = (float *)((unsigned char *)sq + act_bytes);
    float *ps = sc + MAXG * CH;       // [NCW][CH] attention probabilities
    float *qs = ps + NCW * CH;        // [MAXGQ][MAXD] query rows
    float *ms = qs + MAXGQ * MAXD;    // [MAXGQ][CH] mask values
    unsigned char *slots = (unsigned char *)(ms + MAXGQ * CH);
    __shared__ int s_abort, s_last;
    const Ring R{full, empty, slots, log2ns, slot_bytes};
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t cta = blockIdx.x, nctas = gridDim.x;

    if (threadIdx.x == 0) {
        for (int s = 0; s < (1 << log2ns); s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 8);  // the 8 warps of the team that owns the piece
        }
        mbar_init(abar, 1);
        mbar_fence_init();
        s_abort = 0;
    }
    __syncthreads();

    if (warp == NCW) {  // ---------------- producer: every GEMV phase's pieces, in order
        if (lane != 0) return;
        uint32_t t = 0;
        for (int p = 0; p < nph; p++) {
            if (phases[p].type != 0) continue;
            const FusedArgs &a = phases[p].g;
            if (!produce_gemv(a, gemv_geo(a), R, t, (int)cta, (int)nctas, gemv_chunk(1, TEAMS, CG))) {
                if (err) atomicExch(err, 3);
                drain_ring(R, t);
                return;
            }
            if (trace) trace[(cta * nph + p) * 4 + 3] = global_ns();
        }
        return;
    }

    // ---------------- consumers: every warp runs the same barrier sequence, even after an abort
    uint32_t t = 0;
    uint32_t aphase = 0;
    const int team = warp / 8, wt = warp % 8;
    __shared__ __align__(16) MegaPhase sph;  // the current phase's arguments (cheap to re-read)
    for (int p = 0; p < nph; p++) {
        if (p > 0) grid_sync(gbar, p * (int)nctas, &s_abort);
        for (int i = threadIdx.x; i < (int)(sizeof(MegaPhase) / 4); i += NCT)
            ((int *)&sph)[i] = __ldg((const int *)&phases[p] + i);
        named_bar(1, NCT);
        const bool skip = s_abort != 0;  // read after a named barrier: the same in every warp
        const MegaPhase &ph = sph;
        uint64_t *stamp = trace && threadIdx.x == 0 ? trace + (cta * nph + p) * 4 : nullptr;
        if (stamp) stamp[0] = global_ns();
        if (ph.type == 0) {
            const FusedArgs &a = ph.g;
            const GemvGeo G = gemv_geo(a);
            if (!skip) {
                float *sdf = (float *)(sq + (size_t)M * a.K);
                int *ss8 = (int *)(sdf + (size_t)M * G.nb);
                gemv_prologue<M, NCT>(a, sq, sdf, ss8, red, 1);
                if (stamp) stamp[1] = global_ns();
                bool ok;
                if (G.pieces == 2)
                    ok = consume_gemv<QT, 2, M, CG>(a, G, R, t, (int)cta, (int)nctas, team, TEAMS, wt, sq, sdf, ss8);
                else
                    ok = consume_gemv<QT, 1, M, CG>(a, G, R, t, (int)cta, (int)nctas, team, TEAMS, wt, sq, sdf, ss8);
                if (!ok) s_abort = 1;
            }
            t += (uint32_t)(local_groups(G.groups, (int)cta, (int)nctas) * G.nseg * G.pieces);
            named_bar(1, NCT);  // both teams done with the activation buffer
            if (stamp) stamp[2] = global_ns();
        } else {
            if (stamp) stamp[1] = global_ns();
            const MegaAttn &at = ph.at;
            const int64_t nch = (at.nkv + CH - 1) / CH;
            const int64_t items = at.M * at.Hkv * nch;
            bool ok = !skip;
            for (int64_t i = cta; i < items && ok; i += nctas) {
                const int64_t ch = i % nch, hk = (i / nch) % at.Hkv, iq = i / (nch * at.Hkv);
                ok = attn_item(at, (int)iq, (int)hk, (int)ch, (__half *)sq, sc, ps, qs, ms, abar, aphase, &s_last);
                named_bar(3, NCT);  // the K/V staging area is free again
            }
            if (!ok && !skip && threadIdx.x == 0) s_abort = 1;
            named_bar(3, NCT);
            if (stamp) stamp[2] = global_ns();
        }
    }
    if (s_abort && err && threadIdx.x == 0) atomicExch(err, 3);
}

// The activation buffer, also the K/V staging buffer of attention items.
size_t work_bytes(int64_t kmax, int attn_d) {
    const size_t act = gemv_act_bytes(1, kmax), kv = (size_t)CH * attn_d * 2;
    return ((act > kv ? act : kv) + 127) / 128 * 128;
}

size_t head_bytes(int64_t kmax, int attn_d) {
    return (size_t)(2 * MAXNS + 2) * 8 + 256 * 8 + work_bytes(kmax, attn_d) + (size_t)(MAXG + NCW) * CH * 4 +
           (size_t)MAXGQ * (MAXD + CH) * 4;
}

// Two CTAs of the kernel fit an SM with `smem` bytes each (a cooperative launch needs every CTA resident).
template <int QT>
bool resident(size_t smem) {
    auto kern = mega_kernel<QT, 1>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_LIMIT) != cudaSuccess) return false;
    int n = 0;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, NTHREADS, smem) == cudaSuccess && n >= 2;
}

template <int QT, int M>
void launch(const MegaPhase *phases, int nph, int64_t kmax, int attn_d, int64_t slot_bytes, int *gbar, int *err,
            uint64_t *trace, cudaStream_t s) {
    auto kern = mega_kernel<QT, M>;
    static bool attr = false;
    if (!attr) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_LIMIT);
        if (e != cudaSuccess) throw std::runtime_error(std::string("decode kernel: ") + cudaGetErrorString(e));
        attr = true;
    }
    const size_t act = work_bytes(kmax, attn_d);
    const size_t head = head_bytes(kmax, attn_d);
    const int log2ns = ring_log2(SMEM_LIMIT, head, (size_t)slot_bytes, MAXNS);
    if ((1 << log2ns) < 2) throw std::runtime_error("decode kernel: shared memory too small for the weight ring");
    const size_t smem = head + ((size_t)1 << log2ns) * (size_t)slot_bytes;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(2 * num_sms()));
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, phases, nph, log2ns, (int)slot_bytes, act, attn_d, gbar, err, trace);
    if (e != cudaSuccess) throw std::runtime_error(std::string("CUDA launch of the decode kernel failed: ") + cudaGetErrorString(e));
}

}  // namespace

bool mega_supported(int qtype, int M, int64_t kmax, int attn_d) {
    if (M != 1 || (qtype != T_Q4_0 && qtype != T_Q8_0) || (attn_d != 0 && attn_d != 64 && attn_d != 128)) return false;
    const int64_t slot = (int64_t)QTR * QSEG * ((qtype == T_Q4_0 ? 16 : 32) + 2);
    const size_t head = head_bytes(kmax, attn_d);
    const int log2ns = ring_log2(SMEM_LIMIT, head, (size_t)slot, MAXNS);
    if (head + ((size_t)1 << log2ns) * (size_t)slot > SMEM_LIMIT || (1 << log2ns) < 2) return false;
    const size_t smem = head + ((size_t)1 << log2ns) * (size_t)slot;
    return qtype == T_Q4_0 ? resident<0>(smem) : resident<1>(smem);
}

int mega_ctas() { return 2 * num_sms(); }

void mega_step(const MegaPhase *phases_dev, int nph, int qtype, int M, int64_t kmax, int attn_d, int *gbar, int *err,
               uint64_t *trace, cudaStream_t s) {
    cudaError_t e = cudaMemsetAsync(gbar, 0, sizeof(int), s);
    if (e != cudaSuccess) throw std::runtime_error(std::string("memset of the decode barrier failed: ") + cudaGetErrorString(e));
    const int64_t slot = (int64_t)QTR * QSEG * ((qtype == T_Q4_0 ? 16 : 32) + 2);
    if (M != 1) throw std::runtime_error("decode kernel: one token row");
    if (qtype == T_Q4_0) launch<0, 1>(phases_dev, nph, kmax, attn_d, slot, gbar, err, trace, s);
    else launch<1, 1>(phases_dev, nph, kmax, attn_d, slot, gbar, err, trace, s);
}

}  // namespace k
}  // namespace gcb
