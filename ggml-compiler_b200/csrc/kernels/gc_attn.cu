// Generic flash attention: the reference's `flash_attn` node (runtime/src/ops.cpp:217-243 ->
// ggml_flash_attn_ext with f32 accumulation, runtime/include/ggml_compiler_ops.h:124-148).
// q [D, Sq, H, B] f32 (any strides), k/v [D, n_kv, Hkv, B] f16 views of the KV cache, mask
// [n_kv, >= Sq, ...] f16, out [D, H, Sq, B] f32; query head h reads K/V head h / (H / Hkv).
//
// Fixed evaluation order (shared with the CPU checker): the query is rounded to f16; a score is a
// head dot product with lane l owning elements [l*D/32, (l+1)*D/32) (D % 32 == 0; otherwise element
// d on lane d % 32), summed by the butterfly, then times `scale` plus the mask. Keys go in chunks
// of 64: per chunk m = max score, p_j = exp(s_j - m), l = sum p_j and o = sum p_j v_j in key order;
// chunks are merged in order with weights exp(m_c - M), M the overall max, and the output is
// o / l (0 when every key is masked). One warp per (query row, head) runs two passes: the first
// finds M, the second accumulates.
#include <stdexcept>
#include <string>

#include "../gc_kernels.h"
#include "gc_math.cuh"

namespace gcb {
namespace k {

namespace {

constexpr int CH = 64;   // keys per chunk
constexpr int MAXC = 16; // head elements per lane: D <= 512

struct FAk {
    const char *q;
    int64_t D, Sq, H, B, qnb0, qnb1, qnb2, qnb3;
    const char *k;
    int64_t nkv, Hkv, knb1, knb2, knb3;
    const char *v;
    int64_t vnb1, vnb2, vnb3;
    const char *mask;
    int64_t mne1, mne2, mne3, mnb1, mnb2, mnb3;
    float *out;
    float scale;
};

__device__ __forceinline__ int owned(int64_t D, int lane, int j) {  // head element j of this lane, or -1
    if (D % 32 == 0) {
        const int c = (int)(D / 32);
        return j < c ? lane * c + j : -1;
    }
    const int64_t d = lane + 32 * (int64_t)j;
    return d < D ? (int)d : -1;
}

__device__ __forceinline__ float score(const FAk &p, const float *qh, int lane, const char *krow) {
    const __half *kh = (const __half *)krow;
    float acc = 0.0f;
#pragma unroll
    for (int j = 0; j < MAXC; j++) {
        const int d = owned(p.D, lane, j);
        if (d < 0) break;
        acc = __fmaf_rn(qh[j], __half2float(kh[d]), acc);
    }
    return warp_butterfly(acc);
}

__global__ void flash_attn_kernel(FAk p) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = p.Sq * p.H * p.B;
    const int64_t w = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    if (w >= nwarps) return;
    const int64_t iq = w % p.Sq, h = (w / p.Sq) % p.H, b = w / (p.Sq * p.H);
    const int64_t hk = h / (p.H / p.Hkv);
    const char *qrow = p.q + iq * p.qnb1 + h * p.qnb2 + b * p.qnb3;
    const char *kbase = p.k + hk * p.knb2 + b * p.knb3;
    const char *vbase = p.v + hk * p.vnb2 + b * p.vnb3;
    const __half *mrow = p.mask ? (const __half *)(p.mask + iq * p.mnb1 + (h % p.mne2) * p.mnb2 + (b % p.mne3) * p.mnb3)
                                : nullptr;
    float qh[MAXC];
#pragma unroll
    for (int j = 0; j < MAXC; j++) {
        const int d = owned(p.D, lane, j);
        qh[j] = d < 0 ? 0.0f : __half2float(__float2half_rn(*(const float *)(qrow + d * p.qnb0)));
    }
    const float ninf = -__int_as_float(0x7f800000);
    // pass 1: overall maximum score
    float M = ninf;
    for (int64_t j = 0; j < p.nkv; j++) {
        float s = __fmul_rn(score(p, qh, lane, kbase + j * p.knb1), p.scale);
        s = __fadd_rn(s, mrow ? __half2float(mrow[j]) : 0.0f);
        M = fmaxf(M, s);
    }
    // pass 2: per chunk, then merged
    float O[MAXC], o[MAXC];
#pragma unroll
    for (int j = 0; j < MAXC; j++) O[j] = 0.0f;
    float L = 0.0f;
    for (int64_t c0 = 0; c0 < p.nkv; c0 += CH) {
        const int64_t c1 = c0 + CH < p.nkv ? c0 + CH : p.nkv;
        float s[CH];
        float m = ninf;
        for (int64_t j = c0; j < c1; j++) {
            float v = __fmul_rn(score(p, qh, lane, kbase + j * p.knb1), p.scale);
            v = __fadd_rn(v, mrow ? __half2float(mrow[j]) : 0.0f);
            s[j - c0] = v;
            m = fmaxf(m, v);
        }
        if (m == ninf) continue;
#pragma unroll
        for (int jj = 0; jj < MAXC; jj++) o[jj] = 0.0f;
        float l = 0.0f;
        for (int64_t j = c0; j < c1; j++) {
            const float pj = gc_expf(__fsub_rn(s[j - c0], m));
            l = __fadd_rn(l, pj);
            const __half *vr = (const __half *)(vbase + j * p.vnb1);
#pragma unroll
            for (int jj = 0; jj < MAXC; jj++) {
                const int d = owned(p.D, lane, jj);
                if (d < 0) break;
                o[jj] = __fmaf_rn(pj, __half2float(vr[d]), o[jj]);
            }
        }
        const float wgt = gc_expf(__fsub_rn(m, M));
        L = __fmaf_rn(wgt, l, L);
#pragma unroll
        for (int jj = 0; jj < MAXC; jj++) O[jj] = __fmaf_rn(wgt, o[jj], O[jj]);
    }
    const float inv = L == 0.0f ? 0.0f : __fdiv_rn(1.0f, L);
    float *orow = p.out + p.D * (h + p.H * (iq + p.Sq * b));
#pragma unroll
    for (int jj = 0; jj < MAXC; jj++) {
        const int d = owned(p.D, lane, jj);
        if (d < 0) break;
        orow[d] = __fmul_rn(O[jj], inv);
    }
}

}  // namespace

void flash_attn(const TD &q, const TD &kk, const TD &v, const TD *mask, const TD &out, float scale, cudaStream_t s) {
    FAk p{};
    p.q = q.data;
    p.D = q.ne[0];
    p.Sq = q.ne[1];
    p.H = q.ne[2];
    p.B = q.ne[3];
    p.qnb0 = q.nb[0];
    p.qnb1 = q.nb[1];
    p.qnb2 = q.nb[2];
    p.qnb3 = q.nb[3];
    p.k = kk.data;
    p.nkv = kk.ne[1];
    p.Hkv = kk.ne[2];
    p.knb1 = kk.nb[1];
    p.knb2 = kk.nb[2];
    p.knb3 = kk.nb[3];
    p.v = v.data;
    p.vnb1 = v.nb[1];
    p.vnb2 = v.nb[2];
    p.vnb3 = v.nb[3];
    if (mask) {
        p.mask = mask->data;
        p.mne1 = mask->ne[1];
        p.mne2 = mask->ne[2];
        p.mne3 = mask->ne[3];
        p.mnb1 = mask->nb[1];
        p.mnb2 = mask->nb[2];
        p.mnb3 = mask->nb[3];
    } else {
        p.mne2 = p.mne3 = 1;
    }
    p.out = (float *)out.data;
    p.scale = scale;
    if (p.D > 32 * MAXC) throw std::runtime_error("flash_attn: head size above 512");
    const int64_t warps = p.Sq * p.H * p.B;
    flash_attn_kernel<<<(unsigned)((warps + 3) / 4), 128, 0, s>>>(p);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) throw std::runtime_error(std::string("CUDA launch of flash_attn failed: ") + cudaGetErrorString(e));
}

}  // namespace k
}  // namespace gcb
