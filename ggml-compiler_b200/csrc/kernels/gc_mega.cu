// The decode step as one persistent kernel: a cooperative launch (one CTA per SM) runs a list of
// phases, the fused GEMV groups and the attention of every layer, separated by grid barriers.
//
// Per CTA, warp 8 is the producer: one lane streams the weight pieces of every GEMV phase, in phase
// order, into the shared-memory ring (gc_gemv_dev.cuh). Weights never depend on activations, so the
// stream runs ahead through barriers and attention phases, limited only by free ring slots. Warps
// 0-7 are the consumers: for a GEMV phase one tile row each, with the activation row in registers;
// for an attention phase they work on (query row, K/V head, 64-key chunk) items as the split-KV
// flash kernel does (gc_flash.cu), two warps per query head.
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
#include "gc_gemv_dev.cuh"

namespace gcb {
namespace k {

int num_sms();

namespace {

constexpr int TEAMS = 1;
constexpr int CG = 2;                         // row groups per team in a GEMV chunk (gc_gemv_dev.cuh)
constexpr int NCW = 8 * TEAMS;                // consumer warps
constexpr int NCT = NCW * 32;                 // consumer threads
constexpr int NTHREADS = NCT + 32;            // + producer warp
constexpr int MAXNS = 32;
constexpr int CH = 64;                        // attention chunk (keys)
constexpr int MAXD = 128;  // decode kernel head sizes (larger heads use the per-op kernels)
constexpr int WPH = 2;                        // warps per query head
constexpr int MAXG = NCW / WPH;               // query heads per attention item pass
constexpr size_t SMEM_LIMIT = 226 * 1024;     // dynamic shared memory (the opt-in 227 KB less the static part)

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

// One attention item: chunk `ch` of K/V head `hk` for query row `iq` (split-KV flash attention).
__device__ inline bool attn_item(const MegaAttn &at, int64_t iq, int64_t hk, int64_t ch, __half *Ks, __half *Vs,
                                 float *sc, uint64_t *abar, uint32_t parity, int *s_last) {
    const int D = (int)at.D, c = D / 32;
    const int64_t j0 = ch * CH;
    const int n = (int)min((int64_t)CH, at.nkv - j0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t G = at.H / at.Hkv;
    const int hw = warp / WPH, quarter = warp % WPH;
    const float ninf = -__int_as_float(0x7f800000);
    const int64_t nch = (at.nkv + CH - 1) / CH;

    if (threadIdx.x == 0) {
        const uint32_t bytes = (uint32_t)(n * D * 2);
        mbar_expect_tx(abar, 2 * bytes);
        bulk_g2s(Ks, at.k + hk * at.knb2 + j0 * at.knb1, bytes, abar);
        bulk_g2s(Vs, at.v + hk * at.vnb2 + j0 * at.vnb1, bytes, abar);
        *s_last = mbar_wait(abar, parity) ? 1 : 0;  // one bounded wait, its outcome shared
    }
    named_bar(3, NCT);
    if (!*s_last) return false;  // uniform: every consumer thread leaves here

    for (int64_t g0 = 0; g0 < G; g0 += MAXG) {
        const int64_t g = g0 + hw;
        const bool active = g < G;
        const int64_t h = hk * G + (active ? g : 0);
        float *sh = sc + hw * CH;
        float qv[MAXD / 32];
        const float *qrow = at.q + iq * at.ldq + h * at.D;
#pragma unroll
        for (int e = 0; e < MAXD / 32; e++) qv[e] = e < c ? __half2float(__float2half_rn(qrow[lane * c + e])) : 0.0f;
        const __half *mrow = at.mask ? at.mask + iq * at.mask_ld : nullptr;
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
                float pu = p[0];
#pragma unroll
                for (int u = 1; u < 8; u++)
                    if (lane == u) pu = p[u];
                float s = ninf;
                if (j < n) {
                    s = __fmul_rn(pu, at.scale);
                    s = __fadd_rn(s, mrow ? __half2float(mrow[j0 + j]) : 0.0f);
                }
                sh[j] = s;
            }
        }
        named_bar(3, NCT);
        const float s0 = sh[lane], s1 = sh[lane + 32];
        const float m = warp_max(fmaxf(s0, s1));
        float *dst = at.part + (((iq * at.H + h) * nch + ch) * (at.D + 2));
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
                constexpr int OE = MAXD / 32 / WPH;
                float o[OE];
#pragma unroll
                for (int e = 0; e < OE; e++) o[e] = 0.0f;
                for (int j = 0; j < n; j++) {
                    const float pj = __shfl_sync(0xffffffffu, j < 32 ? p0 : p1, j & 31);
                    l = __fadd_rn(l, pj);
                    const __half *vr = Vs + j * D;
#pragma unroll
                    for (int e = 0; e < OE; e++) {
                        const int d = quarter * 32 + lane + e * WPH * 32;
                        if (d < D) o[e] = __fmaf_rn(pj, __half2float(vr[d]), o[e]);
                    }
                }
                if (quarter == 0 && lane == 0) {
                    dst[0] = m;
                    dst[1] = l;
                }
#pragma unroll
                for (int e = 0; e < OE; e++) {
                    const int d = quarter * 32 + lane + e * WPH * 32;
                    if (d < D) dst[2 + d] = o[e];
                }
            }
        }
        named_bar(3, NCT);
    }

    // the last item of this (query row, K/V head) merges its heads' chunks in chunk order
    __threadfence();
    named_bar(3, NCT);
    if (threadIdx.x == 0) {
        int *cnt = at.counters + iq * at.Hkv + hk;
        *s_last = atomicAdd(cnt, 1) == (int)nch - 1;
        if (*s_last) *cnt = 0;
    }
    named_bar(3, NCT);
    if (!*s_last) return true;
    __threadfence();
    for (int64_t g = warp; g < G; g += NCW) {
        const int64_t h = hk * G + g;
        const float *pp = at.part + ((iq * at.H + h) * nch) * (at.D + 2);
        float M = ninf;
        for (int64_t c0 = 0; c0 < nch; c0 += 32)
            if (c0 + lane < nch) M = fmaxf(M, __ldcg(pp + (c0 + lane) * (at.D + 2)));
        M = warp_max(M);
        constexpr int BATCH = 8;
        float L = 0.0f, O[MAXD / 32];
#pragma unroll
        for (int e = 0; e < MAXD / 32; e++) O[e] = 0.0f;
        for (int64_t c0 = 0; c0 < nch; c0 += BATCH) {
            float bm[BATCH], bl[BATCH], bo[BATCH][MAXD / 32];
#pragma unroll
            for (int u = 0; u < BATCH; u++) {
                const bool ok = c0 + u < nch;
                const float *pc = pp + (c0 + u) * (at.D + 2);
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
        float *orow = at.out + at.D * (h + at.H * iq);
#pragma unroll
        for (int e = 0; e < MAXD / 32; e++)
            if (e < c) orow[lane * c + e] = __fmul_rn(O[e], inv);
    }
    return true;
}

template <int QT, int M>
// 9 warps: 3 share a scheduler partition, so at most 168 registers a thread keep one CTA per SM.
__global__ void __maxnreg__(168) mega_kernel(const MegaPhase *phases, int nph, int log2ns, int slot_bytes,
                                                           size_t act_bytes, int attn_d, int *gbar, int *err,
                                                           uint64_t *trace) {
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t *full = (uint64_t *)smem;
    uint64_t *empty = full + MAXNS;
    uint64_t *abar = empty + MAXNS;
    double *red = (double *)(abar + 2);  // [256]
    int8_t *sq = (int8_t *)(red + 256);
    __half *Ks = (__half *)((unsigned char *)sq + act_bytes);
    __half *Vs = Ks + CH * attn_d;
    float *sc = (float *)(Vs + CH * attn_d);
    unsigned char *slots = (unsigned char *)(sc + MAXG * CH);
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
    for (int p = 0; p < nph; p++) {
        if (p > 0) grid_sync(gbar, p * (int)nctas, &s_abort);
        const bool skip = s_abort != 0;  // read after a named barrier: the same in every warp
        const MegaPhase &ph = phases[p];
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
                ok = attn_item(at, iq, hk, ch, Ks, Vs, sc, abar, aphase & 1, &s_last);
                aphase++;
                named_bar(3, NCT);  // the K/V staging area is free again
            }
            if (!ok && !skip && threadIdx.x == 0) s_abort = 1;
            named_bar(3, NCT);
            if (stamp) stamp[2] = global_ns();
        }
    }
    if (s_abort && err && threadIdx.x == 0) atomicExch(err, 3);
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
    const size_t act = gemv_act_bytes(M, kmax);
    const size_t head = (size_t)(2 * MAXNS + 2) * 8 + 256 * 8 + act + (size_t)CH * attn_d * 4 + (size_t)MAXG * CH * 4;
    const int log2ns = ring_log2(SMEM_LIMIT, head, (size_t)slot_bytes, MAXNS);
    if ((1 << log2ns) < 4) throw std::runtime_error("decode kernel: shared memory too small for the weight ring");
    const size_t smem = head + ((size_t)1 << log2ns) * (size_t)slot_bytes;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)num_sms());
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

// One CTA of the kernel fits an SM with `smem` bytes (a cooperative launch needs every CTA resident).
template <int QT>
bool resident(size_t smem) {
    auto kern = mega_kernel<QT, 1>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_LIMIT) != cudaSuccess) return false;
    int n = 0;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, NTHREADS, smem) == cudaSuccess && n >= 1;
}

bool mega_supported(int qtype, int M, int64_t kmax, int attn_d) {
    if (M != 1 || (qtype != T_Q4_0 && qtype != T_Q8_0) || attn_d > MAXD || attn_d % 32) return false;
    const int64_t slot = (int64_t)QTR * QSEG * ((qtype == T_Q4_0 ? 16 : 32) + 2);
    const size_t head = (size_t)(2 * MAXNS + 2) * 8 + 256 * 8 + gemv_act_bytes(M, kmax) + (size_t)CH * attn_d * 4 +
                        (size_t)MAXG * CH * 4;
    const int log2ns = ring_log2(SMEM_LIMIT, head, (size_t)slot, MAXNS);
    if ((1 << log2ns) < 4) return false;
    const size_t smem = head + ((size_t)1 << log2ns) * (size_t)slot;
    return qtype == T_Q4_0 ? resident<0>(smem) : resident<1>(smem);
}

int mega_ctas() { return num_sms(); }

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
