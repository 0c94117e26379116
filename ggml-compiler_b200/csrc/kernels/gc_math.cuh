// Device arithmetic with a fixed evaluation order: every operation below is one IEEE-rounded
// step (the intrinsics are never contracted into FMAs), so kernels that use them produce the same
// bits on every launch shape. The library is also built with --fmad=false.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace gcb {

// exp(x) by range reduction: n = rint(x log2 e), r = x - n ln2 (ln2 split in two), e^r from the
// degree-7 Taylor polynomial in Horner form, and 2^n applied as two exact power-of-two scalings.
// Relative error about 2 ulp over the float range; the CPU checker uses the same steps.
__device__ __forceinline__ float gc_expf(float x) {
    if (x != x) return x;
    if (x > 88.72283f) return __int_as_float(0x7f800000);
    if (x < -103.972084f) return 0.0f;
    const float n = rintf(__fmul_rn(x, 1.44269504088896341f));
    float r = __fmaf_rn(n, -0.693145751953125f, x);
    r = __fmaf_rn(n, -1.428606765330187e-06f, r);
    float p = 1.98412698e-4f;
    p = __fmaf_rn(p, r, 1.38888889e-3f);
    p = __fmaf_rn(p, r, 8.33333333e-3f);
    p = __fmaf_rn(p, r, 4.16666667e-2f);
    p = __fmaf_rn(p, r, 1.66666667e-1f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int ni = (int)n;
    const int a = ni / 2, b = ni - a;
    return __fmul_rn(__fmul_rn(p, __int_as_float((a + 127) << 23)), __int_as_float((b + 127) << 23));
}

__device__ __forceinline__ float gc_silu(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, gc_expf(-x))); }

// 32-lane butterfly sum: p[i] + p[i ^ off] for off = 16 .. 1. Every lane ends with the same value.
__device__ __forceinline__ float warp_butterfly(float p) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) p = __fadd_rn(p, __shfl_xor_sync(0xffffffffu, p, off));
    return p;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}

// 256-way double tree over a block of 256 threads: thread t holds partial t; returns the total to
// every thread. `sh` must hold 256 doubles.
__device__ __forceinline__ double block_tree256(double p, double *sh) {
    const int t = threadIdx.x;
    sh[t] = p;
    __syncthreads();
#pragma unroll
    for (int off = 128; off >= 32; off >>= 1) {
        if (t < off) sh[t] = __dadd_rn(sh[t], sh[t + off]);
        __syncthreads();
    }
    if (t < 32) {  // the last five levels in warp 0: lane t adds lane t + off, the same pairs
        double v = sh[t];
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) v = __dadd_rn(v, __shfl_down_sync(0xffffffffu, v, off));
        if (t == 0) sh[0] = v;
    }
    __syncthreads();
    const double r = sh[0];
    __syncthreads();
    return r;
}

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

}  // namespace gcb
