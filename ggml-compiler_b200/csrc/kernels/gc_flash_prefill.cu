// Flash attention for prefill calls (many query rows), bit-identical to the split-KV kernel and the
// CPU checker: same 64-key chunks, same per-chunk arithmetic, same in-order merge (gc_flash_dev.cuh
// states the order). What changes is only how the work is laid out:
//
// - One CTA owns 64 (query row, head) pairs of one K/V head (64 / G rows x the G query heads of the
//   group) over every chunk, so each chunk's K/V rows are read once per 64 pairs and the merge
//   happens in the CTA (no partials in global memory, no second kernel phase).
// - Scores: a thread computes 2 pairs x 4 keys. A head dot is the checker's 32 lane chains of D/32
//   fmas combined by the 32-lane butterfly; the butterfly's value equals pairwise summation of the
//   chains taken in bit-reversed lane order (level k adds lanes l and l ^ (16 >> k)), which a
//   thread evaluates with a five-level stack. K is staged transposed (element-major, as floats) so
//   that a thread's four keys are one 16-byte load.
// - Values: a thread owns 4 output elements of D/32 pairs and runs the checker's fma chain over
//   the chunk's keys in order; l is the in-order sum of the probabilities.
// - Merge: the checker needs the overall maximum M before it weights any chunk, so pass 1 computes
//   every chunk's maximum m_c (scores only) and pass 2 computes chunk partials and folds them in
//   chunk order, L = fma(w_c, l_c, L), O = fma(w_c, o_c, O) with w_c = exp(m_c - M). A chunk whose
//   weight is exactly 0 for every pair of the CTA (the causal mask's hidden keys, -65504 in the
//   reference's programs) changes nothing, L + 0 = L and O + 0 * o_c = O, as long as O is
//   nonzero; such chunks are skipped unless some O element is still zero (where the sign of the
//   zero could depend on o_c), in which case the chunk is computed as usual. Pass 1 also skips the
//   scores of a chunk when a bound (|q|_1 max|k| |scale| plus the chunk's largest mask value) puts
//   every pair's chunk maximum 128 below one already computed: its weight is then exactly 0.
#include <stdexcept>
#include <string>

#include "../gc_kernels.h"
#include "gc_flash_dev.cuh"
#include "gc_math.cuh"
#include "gc_tma.cuh"

namespace gcb {
namespace k {

namespace {

constexpr int PF_RH = 64;         // (query row, head) pairs per CTA
constexpr int PF_NT = 512;        // threads per CTA
constexpr int PF_MAXCH = 128;     // chunks per row (n_kv <= 8192)
constexpr int PF_PS = FL_CH + 4;  // floats between the score rows of two pairs
constexpr int PF_KTS = FL_CH + 4; // floats between the transposed K rows of two elements

struct PrefillArgs {
    const char *q;
    int64_t qnb0, qnb1, qnb2, qnb3;
    const char *k, *v;  // rows of 2 * D bytes
    int64_t knb2, knb3, vnb2, vnb3;
    const char *mask;
    int64_t mne2, mne3, mnb1, mnb2, mnb3;
    float scale;
    float *out;
    int64_t oH;
    int64_t Sq, H, Hkv, nkv, nch;
    int *err;
};

template <int D>
constexpr size_t prefill_smem() {
    return (size_t)4 * (D * PF_KTS + PF_RH * (D + 4) + PF_RH * FL_CH + PF_RH * PF_PS + PF_RH * PF_MAXCH + PF_RH) +
           (size_t)2 * 2 * FL_CH * D;
}

__device__ __forceinline__ float f16_round(float x) { return __half2float(__float2half_rn(x)); }

// Stand-in maximum of a chunk whose weight is provably 0: finite (so the merge folds it, as the
// checker folds every finite chunk) and far below any real maximum it is compared with.
constexpr float kNegligible = -3.0e38f;

template <int D>
__global__ void __launch_bounds__(PF_NT, 1) flash_prefill_kernel(PrefillArgs a) {
    constexpr int CPL = D / 32, KC = FL_CH, DG = D / 4, RPT = PF_RH * DG / PF_NT;
    constexpr int QS = D + 4;  // floats between two pairs' query rows (rows land on different banks)
    static_assert(RPT >= 1 && PF_NT % DG == 0, "head size");
    extern __shared__ __align__(128) unsigned char smem[];
    float *Kt = (float *)smem;              // [D][PF_KTS] chunk keys, element-major
    float *Qs = Kt + D * PF_KTS;            // [RH][QS] queries rounded to f16
    float *Ms = Qs + PF_RH * QS;            // [RH][KC] mask values of the chunk
    float *Ps = Ms + PF_RH * KC;            // [RH][PF_PS] scores, then probabilities
    float *mc = Ps + PF_RH * PF_PS;         // [RH][PF_MAXCH] chunk maxima (pass 1)
    float *Mr = mc + PF_RH * PF_MAXCH;      // [RH] overall maxima
    __half *Kraw = (__half *)(Mr + PF_RH);  // [KC][D] bulk-copy target for K
    __half *Vs = Kraw + KC * D;             // [KC][D]
    __shared__ uint64_t bar;
    __shared__ float qL1[PF_RH];   // sum of |q| per pair (bounds the pair's scores)
    __shared__ float Mk[PF_RH];    // pass 1: the largest chunk maximum computed so far
    __shared__ float mmax[PF_RH];  // the chunk's largest mask value per pair
    __shared__ unsigned kmax_bits; // the chunk's largest |k| (float bits, non-negative)

    const int tid = threadIdx.x;
    const int G = (int)(a.H / a.Hkv), R = PF_RH / G;
    const int64_t hk = blockIdx.y, b = blockIdx.z, row0 = (int64_t)blockIdx.x * R;
    const float ninf = -__int_as_float(0x7f800000);
    const char *kbase = a.k + hk * a.knb2 + b * a.knb3;
    const char *vbase = a.v + hk * a.vnb2 + b * a.vnb3;
    // per pair: in range, and the byte offset of its mask row (both without a division per use)
    __shared__ int64_t mrow[PF_RH];
    __shared__ unsigned char pvalid[PF_RH];
    if (tid < PF_RH) {
        const int64_t iq = row0 + tid / G, h = hk * G + tid % G;
        pvalid[tid] = iq < a.Sq;
        mrow[tid] = iq * a.mnb1 + (h % a.mne2) * a.mnb2 + (b % a.mne3) * a.mnb3;
    }
    __syncthreads();
    auto valid = [&](int rh) { return pvalid[rh] != 0; };
    // After a timed-out wait: the error word, and NaN in every output row of this CTA, so that a
    // caller that cannot read the error word (the allocation-free entry point) still sees it.
    auto give_up = [&]() {
        for (int i = tid; i < PF_RH * D; i += PF_NT) {
            const int rh = i / D;
            if (!valid(rh)) continue;
            const int64_t iq = row0 + rh / G, h = hk * G + rh % G;
            a.out[(int64_t)D * (h + a.oH * (iq + a.Sq * b)) + i % D] = __int_as_float(0x7fc00000);
        }
        if (tid == 0 && a.err) atomicExch(a.err, 2);
    };

    pdl_wait();  // q and the K/V cache rows of this call were written by earlier kernels
    if (tid == 0) {
        mbar_init(&bar, 1);
        mbar_fence_init();
    }
    for (int i = tid; i < PF_RH * D; i += PF_NT) {
        const int rh = i / D, e = i - rh * D;
        float x = 0.0f;
        if (valid(rh)) {
            const int64_t iq = row0 + rh / G, h = hk * G + rh % G;
            x = f16_round(*(const float *)(a.q + iq * a.qnb1 + h * a.qnb2 + b * a.qnb3 + e * a.qnb0));
        }
        Qs[rh * QS + e] = x;
    }
    __syncthreads();
    if (tid < PF_RH) {
        float l1 = 0.0f;
        for (int e = 0; e < D; e++) l1 = __fadd_rn(l1, fabsf(Qs[tid * QS + e]));
        qL1[tid] = l1;
        Mk[tid] = -__int_as_float(0x7f800000);
    }
    uint32_t phase = 0;
    bool ok = true;

    // the chunk's keys and (v) values into shared memory, K transposed to floats; mask values
    auto load_chunk = [&](int64_t c, bool with_v) -> bool {
        const int64_t j0 = c * KC;
        const int n = (int)min((int64_t)KC, a.nkv - j0);
        if (tid == 0) {
            kmax_bits = 0u;
            const uint32_t bytes = (uint32_t)(n * D * 2);
            mbar_expect_tx(&bar, with_v ? 2 * bytes : bytes);
            bulk_g2s(Kraw, kbase + j0 * 2 * D, bytes, &bar);
            if (with_v) bulk_g2s(Vs, vbase + j0 * 2 * D, bytes, &bar);
        }
        for (int i = tid; i < PF_RH * KC; i += PF_NT) {
            const int rh = i / KC, j = i - rh * KC;
            float mv = 0.0f;
            if (a.mask && j < n && valid(rh)) mv = __half2float(((const __half *)(a.mask + mrow[rh]))[j0 + j]);
            Ms[i] = mv;
        }
        const bool got = __syncthreads_and(mbar_wait(&bar, phase));
        phase ^= 1u;
        if (!got) return false;
        float kabs = 0.0f;
        for (int i = tid; i < KC * (D / 8); i += PF_NT) {
            const int j = i % KC, eg = i / KC;
            float f[8];
            if (j < n) {
                const uint4 u = *(const uint4 *)(Kraw + j * D + eg * 8);
                const __half2 *h2 = (const __half2 *)&u;
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    const float2 x = __half22float2(h2[t]);
                    f[2 * t] = x.x;
                    f[2 * t + 1] = x.y;
                }
            } else {
#pragma unroll
                for (int t = 0; t < 8; t++) f[t] = 0.0f;
            }
#pragma unroll
            for (int t = 0; t < 8; t++) {
                Kt[(eg * 8 + t) * PF_KTS + j] = f[t];
                kabs = fmaxf(kabs, fabsf(f[t]));
            }
        }
        // per pair: the largest mask value of the chunk's keys (8 threads per pair)
        {
            const int pr = tid >> 3, part = tid & 7;
            float mx = -__int_as_float(0x7f800000);
            for (int j = part * 8; j < part * 8 + 8; j++)
                if (j < n) mx = fmaxf(mx, Ms[pr * KC + j]);
#pragma unroll
            for (int off = 4; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            if (part == 0) mmax[pr] = mx;
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) kabs = fmaxf(kabs, __shfl_xor_sync(0xffffffffu, kabs, off));
        if ((tid & 31) == 0) atomicMax(&kmax_bits, __float_as_uint(kabs));  // NaN bits compare above every finite value
        __syncthreads();
        return true;
    };

    // scores of the thread's 2 pairs x 4 keys -> Ps, and each pair's chunk maximum (on all 16
    // threads of the pair)
    const int kg = tid & 15, rp = tid >> 4;  // keys 4kg.., pairs 2rp, 2rp + 1
    auto scores = [&](int n, float (&m)[2]) {
        float st[2][4][5];
        float res[2][4];
#pragma unroll
        for (int i = 0; i < 32; i++) {
            const int l = (int)(__brev((unsigned)i) >> 27);
            float acc[2][4];
#pragma unroll
            for (int p = 0; p < 2; p++)
#pragma unroll
                for (int u = 0; u < 4; u++) acc[p][u] = 0.0f;
            float qv[2][CPL];  // the leaf's CPL query elements of both pairs, one vector load each
#pragma unroll
            for (int p = 0; p < 2; p++) {
                const float *qr = Qs + (2 * rp + p) * QS + l * CPL;
                if constexpr (CPL == 4) {
                    const float4 t = *(const float4 *)qr;
                    qv[p][0] = t.x, qv[p][1] = t.y, qv[p][2] = t.z, qv[p][3] = t.w;
                } else {
                    const float2 t = *(const float2 *)qr;
                    qv[p][0] = t.x, qv[p][1] = t.y;
                }
            }
#pragma unroll
            for (int e = 0; e < CPL; e++) {
                const int d = l * CPL + e;
                const float4 kv = *(const float4 *)(Kt + d * PF_KTS + 4 * kg);
                const float kk[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
                for (int p = 0; p < 2; p++)
#pragma unroll
                    for (int u = 0; u < 4; u++) acc[p][u] = __fmaf_rn(qv[p][e], kk[u], acc[p][u]);
            }
            // push the lane chain into the pairwise tree (bit i of the count = level carry)
#pragma unroll
            for (int p = 0; p < 2; p++)
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    float v = acc[p][u];
                    int lv = 0;
#pragma unroll
                    for (int bits = i; bits & 1; bits >>= 1, lv++) v = __fadd_rn(st[p][u][lv], v);
                    if (i == 31) res[p][u] = v;
                    else st[p][u][lv] = v;
                }
        }
#pragma unroll
        for (int p = 0; p < 2; p++) {
            const int rh = 2 * rp + p;
            float s[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int j = 4 * kg + u;
                s[u] = j < n ? __fadd_rn(__fmul_rn(res[p][u], a.scale), Ms[rh * KC + j]) : ninf;
            }
            *(float4 *)(Ps + rh * PF_PS + 4 * kg) = make_float4(s[0], s[1], s[2], s[3]);
            float mx = fmaxf(fmaxf(s[0], s[1]), fmaxf(s[2], s[3]));
#pragma unroll
            for (int off = 8; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            m[p] = mx;
        }
    };

    // pass 1: every chunk's maximum
    for (int64_t c = 0; c < a.nch && ok; c++) {
        const int n = (int)min((int64_t)KC, a.nkv - c * KC);
        if (!load_chunk(c, false)) {
            ok = false;
            break;
        }
        // A pair's scores in this chunk are at most |q|_1 max|k| |scale| + its largest mask value (the
        // factor and the 1 cover rounding). When that is 128 below a chunk maximum already computed,
        // the chunk's weight exp(m_c - M) is exactly 0 and m_c does not raise M: every pair of the
        // CTA records a stand-in maximum (finite, weight 0) and the scores are not computed.
        int hidden = 1;
        if (tid < PF_RH && valid(tid)) {
            const float bound = __fadd_rn(__fmul_rn(__fmul_rn(__fmul_rn(qL1[tid], __uint_as_float(kmax_bits)), fabsf(a.scale)), 1.01f), 1.0f);
            hidden = __fadd_rn(bound, mmax[tid]) < __fsub_rn(Mk[tid], 128.0f);
        }
        if (__syncthreads_and(hidden)) {
            if (tid < PF_RH) mc[tid * PF_MAXCH + c] = kNegligible;
            __syncthreads();
            continue;
        }
        float m[2];
        scores(n, m);
        if (kg == 0) {
            mc[(2 * rp) * PF_MAXCH + c] = m[0];
            mc[(2 * rp + 1) * PF_MAXCH + c] = m[1];
            Mk[2 * rp] = fmaxf(Mk[2 * rp], m[0]);
            Mk[2 * rp + 1] = fmaxf(Mk[2 * rp + 1], m[1]);
        }
        __syncthreads();  // Kt and Ms are rewritten by the next chunk
    }
    if (!ok) {
        give_up();
        return;
    }
    if (tid < PF_RH) {
        float M = ninf;
        for (int64_t c = 0; c < a.nch; c++) M = fmaxf(M, mc[tid * PF_MAXCH + c]);
        Mr[tid] = M;
    }
    __syncthreads();

    // pass 2: chunk partials folded in order
    const int dg = tid % DG, rq = tid / DG;
    float O[RPT][4], L[RPT];
#pragma unroll
    for (int i = 0; i < RPT; i++) {
        L[i] = 0.0f;
#pragma unroll
        for (int u = 0; u < 4; u++) O[i][u] = 0.0f;
    }
    for (int64_t c = 0; c < a.nch; c++) {
        int need = 0;
        if (tid < PF_RH && valid(tid)) {
            const float m = mc[tid * PF_MAXCH + c];
            need = m != ninf && gc_expf(__fsub_rn(m, Mr[tid])) != 0.0f;
        }
        if (!__syncthreads_or(need)) {
            int zero = 0;  // a pair that would fold this chunk with weight 0 into a zero element
#pragma unroll
            for (int i = 0; i < RPT; i++) {
                const int rh = rq * RPT + i;
                if (valid(rh) && mc[rh * PF_MAXCH + c] != ninf)
#pragma unroll
                    for (int u = 0; u < 4; u++) zero |= O[i][u] == 0.0f;
            }
            if (!__syncthreads_or(zero)) continue;
        }
        const int n = (int)min((int64_t)KC, a.nkv - c * KC);
        if (!load_chunk(c, true)) {
            ok = false;
            break;
        }
        float m[2];
        scores(n, m);
        // probabilities of the thread's own scores (each pair's max is on all its 16 threads)
#pragma unroll
        for (int p = 0; p < 2; p++) {
            float *row = Ps + (2 * rp + p) * PF_PS + 4 * kg;
            float4 s = *(float4 *)row;
            float sv[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
            for (int u = 0; u < 4; u++) sv[u] = (m[p] != ninf && 4 * kg + u < n) ? gc_expf(__fsub_rn(sv[u], m[p])) : 0.0f;
            *(float4 *)row = make_float4(sv[0], sv[1], sv[2], sv[3]);
        }
        __syncthreads();
        float oc[RPT][4], lc[RPT];
#pragma unroll
        for (int i = 0; i < RPT; i++) {
            lc[i] = 0.0f;
#pragma unroll
            for (int u = 0; u < 4; u++) oc[i][u] = 0.0f;
        }
        for (int j0 = 0; j0 < n; j0 += 4) {
            float4 p4[RPT];
#pragma unroll
            for (int i = 0; i < RPT; i++) p4[i] = *(const float4 *)(Ps + (rq * RPT + i) * PF_PS + j0);
#pragma unroll
            for (int t = 0; t < 4; t++) {
                if (j0 + t >= n) break;
                const uint2 vv = *(const uint2 *)(Vs + (j0 + t) * D + 4 * dg);
                const float2 v01 = __half22float2(*(const __half2 *)&vv.x), v23 = __half22float2(*(const __half2 *)&vv.y);
                const float vf[4] = {v01.x, v01.y, v23.x, v23.y};
#pragma unroll
                for (int i = 0; i < RPT; i++) {
                    const float pj = t == 0 ? p4[i].x : t == 1 ? p4[i].y : t == 2 ? p4[i].z : p4[i].w;
                    lc[i] = __fadd_rn(lc[i], pj);
#pragma unroll
                    for (int u = 0; u < 4; u++) oc[i][u] = __fmaf_rn(pj, vf[u], oc[i][u]);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < RPT; i++) {
            const int rh = rq * RPT + i;
            const float mcc = mc[rh * PF_MAXCH + c];
            if (mcc == ninf) continue;
            const float w = gc_expf(__fsub_rn(mcc, Mr[rh]));
            L[i] = __fmaf_rn(w, lc[i], L[i]);
#pragma unroll
            for (int u = 0; u < 4; u++) O[i][u] = __fmaf_rn(w, oc[i][u], O[i][u]);
        }
        __syncthreads();  // Kt, Vs, Ms and Ps are rewritten by the next chunk
    }
    if (!ok) {
        give_up();
        return;
    }
#pragma unroll
    for (int i = 0; i < RPT; i++) {
        const int rh = rq * RPT + i;
        if (!valid(rh)) continue;
        const float inv = L[i] == 0.0f ? 0.0f : __fdiv_rn(1.0f, L[i]);
        const int64_t iq = row0 + rh / G, h = hk * G + rh % G;
        float *orow = a.out + (int64_t)D * (h + a.oH * (iq + a.Sq * b)) + 4 * dg;
        *(float4 *)orow = make_float4(__fmul_rn(O[i][0], inv), __fmul_rn(O[i][1], inv), __fmul_rn(O[i][2], inv),
                                      __fmul_rn(O[i][3], inv));
    }
}

template <int D>
void launch_prefill(const PrefillArgs &a, int64_t B, cudaStream_t s) {
    auto kern = flash_prefill_kernel<D>;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)prefill_smem<D>());
        attr = true;
    }
    const int R = PF_RH / (int)(a.H / a.Hkv);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((a.Sq + R - 1) / R), (unsigned)a.Hkv, (unsigned)B);
    cfg.blockDim = dim3(PF_NT);
    cfg.dynamicSmemBytes = prefill_smem<D>();
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
    if (e != cudaSuccess) throw std::runtime_error(std::string("CUDA launch of flash_prefill failed: ") + cudaGetErrorString(e));
}

}  // namespace

bool flash_prefill_ok(const TD &q, const TD &kk, const TD &v, const TD &out) {
    const int64_t D = q.ne[0], G = kk.ne[2] ? q.ne[2] / kk.ne[2] : 0;
    if ((D != 64 && D != 128) || q.ne[1] < 16 || G < 1 || PF_RH % G || q.ne[2] % kk.ne[2]) return false;
    if (kk.nb[0] != 2 || v.nb[0] != 2 || kk.nb[1] != 2 * D || v.nb[1] != 2 * D) return false;
    if ((kk.ne[1] + FL_CH - 1) / FL_CH > PF_MAXCH) return false;
    if (((uintptr_t)kk.data | (uintptr_t)v.data | (uintptr_t)kk.nb[2] | (uintptr_t)v.nb[2] | (uintptr_t)kk.nb[3] |
         (uintptr_t)v.nb[3]) % 16)
        return false;
    return out.nb[0] == 4 && out.nb[1] == 4 * D && out.nb[2] % (4 * D) == 0 && out.nb[3] == out.nb[2] * q.ne[1] &&
           (uintptr_t)out.data % 16 == 0;
}

void flash_prefill(const TD &q, const TD &kk, const TD &v, const TD *mask, const TD &out, float scale, int *err,
                   cudaStream_t s) {
    PrefillArgs a{};
    a.q = q.data;
    a.qnb0 = q.nb[0];
    a.qnb1 = q.nb[1];
    a.qnb2 = q.nb[2];
    a.qnb3 = q.nb[3];
    a.k = kk.data;
    a.v = v.data;
    a.knb2 = kk.nb[2];
    a.knb3 = kk.nb[3];
    a.vnb2 = v.nb[2];
    a.vnb3 = v.nb[3];
    a.mne2 = a.mne3 = 1;
    if (mask) {
        a.mask = mask->data;
        a.mne2 = mask->ne[2];
        a.mne3 = mask->ne[3];
        a.mnb1 = mask->nb[1];
        a.mnb2 = mask->nb[2];
        a.mnb3 = mask->nb[3];
    }
    a.scale = scale;
    a.out = (float *)out.data;
    a.oH = out.nb[2] / (4 * q.ne[0]);
    a.Sq = q.ne[1];
    a.H = q.ne[2];
    a.Hkv = kk.ne[2];
    a.nkv = kk.ne[1];
    a.nch = (a.nkv + FL_CH - 1) / FL_CH;
    a.err = err;
    if (q.ne[0] == 64) launch_prefill<64>(a, q.ne[3], s);
    else launch_prefill<128>(a, q.ne[3], s);
}

}  // namespace k
}  // namespace gcb
