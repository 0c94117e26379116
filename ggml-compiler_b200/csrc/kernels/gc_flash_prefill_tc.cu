// Flash attention for prefill calls on the tensor cores (mma.sync m16n8k16, f16 operands, f32
// accumulation), selected by GGML_COMPILER_B200_PREFILL_ATTN=tc. The default prefill kernel
// (gc_flash_prefill.cu) reproduces the CPU checker's summation order bit for bit on the CUDA cores;
// this one gives that up for the tensor cores and stays within the north star's tolerance
// (max-abs 1e-2 on logits): the products are the same exact f16 x f16 products, but the tensor
// core sums them in its own order, and the probabilities are rounded to f16 before they weight V
// (as ggml's f16 V path does).
//
// A CTA takes 64 query rows of one head (4 warps x 16 rows) and walks the K/V chunks of 64 keys in
// order: S = Q K^T (ldmatrix fragments of the f16 Q tile and of the K chunk), S * scale + mask, the
// online softmax in registers (row max and sum over the 4 lanes of a quad), then O += P V with the
// S accumulators reused as the A fragments of P. K/V chunks are double-buffered with cp.async. A
// chunk whose mask hides every (row, key) pair of the CTA (-65504 or -inf, or past n_kv) is
// skipped once every row has seen a visible key: its weights would all be exp(-65504 - max) = 0.
// Output = O / l (0 when every key of a row is -inf).
#include <cstring>
#include <stdexcept>
#include <string>

#include "../gc_kernels.h"
#include "gc_flash_dev.cuh"
#include "gc_tma.cuh"

namespace gcb {
namespace k {

namespace {

constexpr int TC_ROWS = 64;  // query rows per CTA
constexpr int TC_KC = 64;    // keys per chunk
constexpr int TC_NT = 128;   // threads per CTA

struct TcArgs {
    const char *q;
    int64_t qnb0, qnb1, qnb2, qnb3;
    const char *k, *v;  // rows of 2 * D bytes
    int64_t knb2, knb3, vnb2, vnb3;
    const char *mask;
    int64_t mne2, mne3, mnb1, mnb2, mnb3;
    float scale;
    float *out;
    int64_t oH;
    int64_t Sq, H, Hkv, nkv;
};

template <int D>
__host__ __device__ constexpr int tc_ld() { return D + 8; }  // halves between two smem rows (ldmatrix rows on distinct banks)

template <int D>
constexpr size_t tc_smem() { return (size_t)2 * (TC_ROWS * tc_ld<D>() + 2 * 2 * TC_KC * tc_ld<D>()); }

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void cp_async16(void *dst, const void *src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3, const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3, const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_u32(p)));
}

// D (16x8 f32) += A (16x16 f16, row) * B (16x8 f16, col)
__device__ __forceinline__ void mma16816(float *c, const uint32_t *a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 2^x by the hardware approximation (PTX ex2.approx, about 2 ulp; -inf gives 0): the
// probabilities are rounded to f16 right after, so its error is far below the kernel's tolerance
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    uint32_t u;
    memcpy(&u, &h, 4);
    return u;
}

template <int D>
__global__ void __launch_bounds__(TC_NT) flash_prefill_tc_kernel(TcArgs a) {
    constexpr int LD = tc_ld<D>(), NT_O = D / 8, KS = D / 16;
    extern __shared__ __align__(128) unsigned char smem[];
    __half *Qs = (__half *)smem;            // [64][LD]
    __half *Ks = Qs + TC_ROWS * LD;         // [2][64][LD]
    __half *Vs = Ks + 2 * TC_KC * LD;       // [2][64][LD]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tig = lane & 3;
    const int64_t h = blockIdx.y, b = blockIdx.z, row0 = (int64_t)blockIdx.x * TC_ROWS;
    const int64_t hk = h / (a.H / a.Hkv);
    const char *kbase = a.k + hk * a.knb2 + b * a.knb3;
    const char *vbase = a.v + hk * a.vnb2 + b * a.vnb3;
    const int64_t nch = (a.nkv + TC_KC - 1) / TC_KC;
    const float ninf = -__int_as_float(0x7f800000);

    pdl_wait();  // q and the K/V cache rows of this call were written by earlier kernels

    auto load_chunk = [&](int64_t c, int buf) {
        __half *kd = Ks + buf * TC_KC * LD, *vd = Vs + buf * TC_KC * LD;
        for (int i = tid; i < TC_KC * (D / 8); i += TC_NT) {
            const int r = i / (D / 8), e = (i % (D / 8)) * 8;
            const int64_t key = c * TC_KC + r;
            const bool ok = key < a.nkv;
            const int64_t kk = ok ? key : 0;
            cp_async16(kd + r * LD + e, kbase + kk * 2 * D + e * 2, ok);
            cp_async16(vd + r * LD + e, vbase + kk * 2 * D + e * 2, ok);
        }
        cp_async_commit();
    };
    load_chunk(0, 0);
    // the query tile, rounded to f16 (rows past Sq are zero)
    for (int i = tid; i < TC_ROWS * D; i += TC_NT) {
        const int r = i / D, e = i % D;
        const int64_t iq = row0 + r;
        float x = 0.0f;
        if (iq < a.Sq) x = *(const float *)(a.q + iq * a.qnb1 + h * a.qnb2 + b * a.qnb3 + e * a.qnb0);
        Qs[r * LD + e] = __float2half_rn(x);
    }
    __syncthreads();
    // this warp's Q fragments for every 16-wide slice of the head
    uint32_t qf[KS][4];
#pragma unroll
    for (int ks = 0; ks < KS; ks++)
        ldsm_x4(qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], Qs + (warp * 16 + (lane % 16)) * LD + ks * 16 + 8 * (lane / 16));

    const int64_t ra = row0 + warp * 16 + g, rb = ra + 8;  // this thread's two rows
    const char *mra = a.mask ? a.mask + ra * a.mnb1 + (h % a.mne2) * a.mnb2 + (b % a.mne3) * a.mnb3 : nullptr;
    const char *mrb = a.mask ? a.mask + rb * a.mnb1 + (h % a.mne2) * a.mnb2 + (b % a.mne3) * a.mnb3 : nullptr;
    float o[NT_O][4];
#pragma unroll
    for (int j = 0; j < NT_O; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
    float ma = ninf, mb = ninf, la = 0.0f, lb = 0.0f;  // running maxima (log2 units) and partial sums
    const float sl2 = a.scale * 1.4426950408889634f;   // scores in log2 units

    // This thread's mask values of a chunk as f16 pairs (keys k, k + 1 of rows ra and rb), -inf for
    // keys past n_kv and rows past Sq; fetched one chunk ahead so the loads overlap the chunk before.
    // Pairs are one 32-bit load when the mask rows are 4-byte aligned.
    const bool m32 = a.mask && (a.mnb1 % 4 == 0) && ((uintptr_t)mra % 4 == 0);
    auto fetch = [&](int64_t c, uint32_t (&mp)[8][2]) {
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int64_t k0 = c * TC_KC + 8 * j + 2 * tig;
#pragma unroll
            for (int rr = 0; rr < 2; rr++) {
                const bool rowok = (rr == 0 ? ra : rb) < a.Sq;
                const char *mr = rr == 0 ? mra : mrb;
                uint32_t v = 0xFC00FC00u;  // -inf, -inf
                if (rowok && k0 < a.nkv) {
                    if (!a.mask) {
                        v = k0 + 1 < a.nkv ? 0u : 0xFC000000u;
                    } else if (m32 && k0 + 1 < a.nkv) {
                        v = __ldg((const unsigned int *)(mr + k0 * 2));
                    } else {
                        const uint32_t lo = __ldg((const unsigned short *)(mr + k0 * 2));
                        const uint32_t hi = k0 + 1 < a.nkv ? (uint32_t)__ldg((const unsigned short *)(mr + k0 * 2 + 2)) : 0xFC00u;
                        v = lo | (hi << 16);
                    }
                }
                mp[j][rr] = v;
            }
        }
    };
    uint32_t mnext[8][2];
    fetch(0, mnext);

    for (int64_t c = 0; c < nch; c++) {
        const int buf = (int)(c & 1);
        cp_async_wait<0>();
        __syncthreads();  // chunk c landed for every thread; buffer buf ^ 1 is no longer read
        if (c + 1 < nch) load_chunk(c + 1, buf ^ 1);
        // mask values of this thread's 32 scores, and whether the whole CTA's tile is hidden
        float mk[8][4];
        bool hidden = true;
#pragma unroll
        for (int j = 0; j < 8; j++) {
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const uint32_t pr = mnext[j][e >> 1];
                const float m = __half2float(__ushort_as_half((unsigned short)((e & 1) ? pr >> 16 : pr & 0xFFFFu)));
                mk[j][e] = m;
                hidden = hidden && !(m > -65504.0f);
            }
        }
        if (c + 1 < nch) fetch(c + 1, mnext);
        // skip only once each row has seen a visible key: a row whose every key is masked with the
        // finite -65504 still averages V uniformly, as the checker does
        const bool live = (ra >= a.Sq || ma > -40000.0f) && (rb >= a.Sq || mb > -40000.0f);
        if (__syncthreads_and(hidden && live)) continue;
        // S = Q K^T for 16 rows x 64 keys (8 tiles of 8 keys)
        const __half *kc = Ks + buf * TC_KC * LD, *vc = Vs + buf * TC_KC * LD;
        float s[8][4];
#pragma unroll
        for (int j = 0; j < 8; j++) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
        for (int ks = 0; ks < KS; ks++) {
#pragma unroll
            for (int jp = 0; jp < 4; jp++) {  // key tiles 2jp, 2jp + 1
                uint32_t b0, b1, b2, b3;
                ldsm_x4(b0, b1, b2, b3, kc + (16 * jp + (lane % 8) + 8 * (lane / 16)) * LD + ks * 16 + 8 * ((lane / 8) % 2));
                mma16816(s[2 * jp], qf[ks], b0, b1);
                mma16816(s[2 * jp + 1], qf[ks], b2, b3);
            }
        }
        // scale, mask, online softmax (log2 units)
        float cma = ninf, cmb = ninf;
#pragma unroll
        for (int j = 0; j < 8; j++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float v = mk[j][e] == ninf ? ninf : fmaf(s[j][e], sl2, mk[j][e] * 1.4426950408889634f);
                s[j][e] = v;
                if (e < 2) cma = fmaxf(cma, v);
                else cmb = fmaxf(cmb, v);
            }
        cma = fmaxf(cma, __shfl_xor_sync(0xffffffffu, cma, 1));
        cma = fmaxf(cma, __shfl_xor_sync(0xffffffffu, cma, 2));
        cmb = fmaxf(cmb, __shfl_xor_sync(0xffffffffu, cmb, 1));
        cmb = fmaxf(cmb, __shfl_xor_sync(0xffffffffu, cmb, 2));
        const float na = fmaxf(ma, cma), nb = fmaxf(mb, cmb);
        const float aa = na == ninf ? 1.0f : ex2(ma - na), ab = nb == ninf ? 1.0f : ex2(mb - nb);
        ma = na;
        mb = nb;
        la *= aa;
        lb *= ab;
#pragma unroll
        for (int j = 0; j < NT_O; j++) {
            o[j][0] *= aa;
            o[j][1] *= aa;
            o[j][2] *= ab;
            o[j][3] *= ab;
        }
        uint32_t pf[4][4];  // P as A fragments, 4 slices of 16 keys
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float p0 = s[j][0] == ninf ? 0.0f : ex2(s[j][0] - na);
            const float p1 = s[j][1] == ninf ? 0.0f : ex2(s[j][1] - na);
            const float p2 = s[j][2] == ninf ? 0.0f : ex2(s[j][2] - nb);
            const float p3 = s[j][3] == ninf ? 0.0f : ex2(s[j][3] - nb);
            la += p0 + p1;
            lb += p2 + p3;
            pf[j / 2][(j % 2) * 2] = pack_h2(p0, p1);
            pf[j / 2][(j % 2) * 2 + 1] = pack_h2(p2, p3);
        }
        // O += P V: for each 16-key slice, V^T fragments by transposed ldmatrix
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
            const uint32_t ap[4] = {pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3]};
#pragma unroll
            for (int jp = 0; jp < NT_O / 2; jp++) {  // output tiles 2jp, 2jp + 1 (16 head elements)
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(b0, b1, b2, b3, vc + (16 * kk + (lane % 8) + 8 * ((lane / 8) % 2)) * LD + 16 * jp + 8 * (lane / 16));
                mma16816(o[2 * jp], ap, b0, b1);
                mma16816(o[2 * jp + 1], ap, b2, b3);
            }
        }
    }
    cp_async_wait<0>();
    la += __shfl_xor_sync(0xffffffffu, la, 1);
    la += __shfl_xor_sync(0xffffffffu, la, 2);
    lb += __shfl_xor_sync(0xffffffffu, lb, 1);
    lb += __shfl_xor_sync(0xffffffffu, lb, 2);
    const float ia = la > 0.0f ? 1.0f / la : 0.0f, ib = lb > 0.0f ? 1.0f / lb : 0.0f;
#pragma unroll
    for (int j = 0; j < NT_O; j++) {
        const int e = 8 * j + 2 * tig;
        if (ra < a.Sq) {
            float *orow = a.out + (int64_t)D * (h + a.oH * (ra + a.Sq * b)) + e;
            *(float2 *)orow = make_float2(o[j][0] * ia, o[j][1] * ia);
        }
        if (rb < a.Sq) {
            float *orow = a.out + (int64_t)D * (h + a.oH * (rb + a.Sq * b)) + e;
            *(float2 *)orow = make_float2(o[j][2] * ib, o[j][3] * ib);
        }
    }
}

template <int D>
void launch_tc(const TcArgs &a, int64_t B, cudaStream_t s) {
    auto kern = flash_prefill_tc_kernel<D>;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc_smem<D>());
        attr = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((a.Sq + TC_ROWS - 1) / TC_ROWS), (unsigned)a.H, (unsigned)B);
    cfg.blockDim = dim3(TC_NT);
    cfg.dynamicSmemBytes = tc_smem<D>();
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
    if (e != cudaSuccess) throw std::runtime_error(std::string("CUDA launch of flash_prefill_tc failed: ") + cudaGetErrorString(e));
}

}  // namespace

void flash_prefill_tc(const TD &q, const TD &kk, const TD &v, const TD *mask, const TD &out, float scale, cudaStream_t s) {
    TcArgs a{};
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
    if (q.ne[0] == 64) launch_tc<64>(a, q.ne[3], s);
    else launch_tc<128>(a, q.ne[3], s);
}

}  // namespace k
}  // namespace gcb
