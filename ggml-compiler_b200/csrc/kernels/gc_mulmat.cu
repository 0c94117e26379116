// Generic mul_mat for any shape the programs produce (GQA-style batch broadcast, strided
// activations): the semantics of the reference's `mul_mat` node (runtime/src/ops.cpp:107-119,
// runtime/include/ggml_compiler_ops.h:116-122), out[n, m, i2, i3] = sum_k a[k, n, i2/r2, i3/r3] *
// b[k, m, i2, i3].
//
// Quantized weights follow ggml's CPU arithmetic: each activation row is converted to Q8_0 blocks
// (d = amax/127 as fp16, codes = nearest-even(x * 127/amax)), the per-block integer dot products
// are exact, and the block results are summed in f32 in a fixed order: block b feeds lane b % 32 of
// a warp (fma of d_w*d_x and the integer sum), then a butterfly over the 32 lanes. f16 weights
// round the activation to f16 first; f32 weights use it as is; element k then feeds lane k % 32.
//
// This is the correctness path for every shape; the decode-time fused GEMVs (gc_gemv.cu) and the
// tensor-core prefill GEMM replace it on the hot path. Weights in the other block formats that stay
// in their GGUF layout (q4_1, q5_1, K-quants) go to mul_mat_block (gc_blockq.cu).
#include <algorithm>
#include <cstdlib>
#include <stdexcept>
#include <string>

#include "../gc_kernels.h"
#include "gc_math.cuh"
#include "gc_qweight.cuh"

namespace gcb {
namespace k {

namespace {

void check_launch(const char *what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) throw std::runtime_error(std::string("CUDA launch of ") + what + " failed: " + cudaGetErrorString(e));
}

struct MMk {
    const char *a;
    const uint16_t *as;
    int atype;
    int64_t K, N, A2, A3;
    int64_t anb1, anb2, anb3;
    const char *b;
    int btype;
    int64_t M, B2, B3;
    int64_t bnb0, bnb1, bnb2, bnb3;
    float *out;
};

// One warp per 32-element block of an activation row: Q8_0 with the x86 rounding rule.
__global__ void act_quant_kernel(MMk p, int8_t *qx, uint16_t *dx) {
    const int lane = threadIdx.x & 31;
    const int64_t nb = p.K / 32;
    const int64_t nblk = nb * p.M * p.B2 * p.B3;
    for (int64_t w = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; w < nblk;
         w += ((int64_t)gridDim.x * blockDim.x) >> 5) {
        const int64_t blk = w % nb;
        int64_t r = w / nb;  // activation row index over (m, i2, i3)
        const int64_t m = r % p.M, i2 = (r / p.M) % p.B2, i3 = r / (p.M * p.B2);
        const char *row = p.b + m * p.bnb1 + i2 * p.bnb2 + i3 * p.bnb3;
        const float x = *(const float *)(row + (blk * 32 + lane) * p.bnb0);
        const float amax = warp_max(fabsf(x));
        const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
        qx[r * p.K + blk * 32 + lane] = (int8_t)__float2int_rn(__fmul_rn(x, id));
        if (lane == 0) dx[r * nb + blk] = f2h(__fdiv_rn(amax, 127.0f));
    }
}

__device__ __forceinline__ int block_isum(int atype, const char *codes, const int8_t *xq) {
    const int4 *x4 = (const int4 *)xq;
    const int4 xa = x4[0], xb = x4[1];
    const int xs[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
    int s = 0;
    if (atype == T_Q4_0) {
        const uint4 w = *(const uint4 *)codes;
        const unsigned ws[4] = {w.x, w.y, w.z, w.w};
        int sx = 0;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            s = __dp4a((int)(ws[i] & 0x0f0f0f0fu), xs[i], s);
            s = __dp4a((int)((ws[i] >> 4) & 0x0f0f0f0fu), xs[4 + i], s);
            sx = __dp4a(0x01010101, xs[i], sx);
            sx = __dp4a(0x01010101, xs[4 + i], sx);
        }
        s -= 8 * sx;
    } else {
        const int4 w0 = *(const int4 *)codes, w1 = *(const int4 *)(codes + 16);
        const int ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int i = 0; i < 8; i++) s = __dp4a(ws[i], xs[i], s);
    }
    return s;
}

// One warp per output element (n, m, i2, i3), quantized weight (tiled layout, rows flattened).
__global__ void mm_quant_kernel(MMk p, const int8_t *qx, const uint16_t *dx) {
    const int lane = threadIdx.x & 31;
    const int64_t nb = p.K / 32;
    const int64_t nout = p.N * p.M * p.B2 * p.B3;
    const QW wq{p.a, nb, p.atype == T_Q4_0 ? 16 : 32};
    for (int64_t w = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; w < nout;
         w += ((int64_t)gridDim.x * blockDim.x) >> 5) {
        const int64_t n = w % p.N;
        const int64_t r = w / p.N;  // (m, i2, i3)
        const int64_t i2 = (r / p.M) % p.B2, i3 = r / (p.M * p.B2);
        const int64_t a2 = i2 / (p.B2 / p.A2), a3 = i3 / (p.B3 / p.A3);
        const int64_t arow = n + p.N * (a2 + p.A2 * a3);
        const int8_t *xrow = qx + r * p.K;
        const uint16_t *xd = dx + r * nb;
        float acc = 0.0f;
        for (int64_t blk = lane; blk < nb; blk += 32) {
            const int isum = block_isum(p.atype, qw_code(wq, arow, blk), xrow + blk * 32);
            const float dd = __fmul_rn(h2f(qw_scale(wq, arow, blk)), h2f(xd[blk]));
            acc = __fmaf_rn(dd, (float)isum, acc);
        }
        acc = warp_butterfly(acc);
        if (lane == 0) p.out[w] = acc;
    }
}

// Nine or more activation rows: one thread per output element (n, m, i2, i3), every block of the
// row fma'd in order into one sum (the order the tensor-core GEMM and the CPU checker use).
// Consecutive threads take consecutive weight rows of one activation row.
__global__ void mm_quant_seq_kernel(MMk p, const int8_t *qx, const uint16_t *dx) {
    const int64_t nb = p.K / 32;
    const int64_t nout = p.N * p.M * p.B2 * p.B3;
    const QW wq{p.a, nb, p.atype == T_Q4_0 ? 16 : 32};
    for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < nout; w += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = w % p.N;
        const int64_t r = w / p.N;  // (m, i2, i3)
        const int64_t i2 = (r / p.M) % p.B2, i3 = r / (p.M * p.B2);
        const int64_t a2 = i2 / (p.B2 / p.A2), a3 = i3 / (p.B3 / p.A3);
        const int64_t arow = n + p.N * (a2 + p.A2 * a3);
        const int8_t *xrow = qx + r * p.K;
        const uint16_t *xd = dx + r * nb;
        float acc = 0.0f;
        for (int64_t blk = 0; blk < nb; blk++) {
            const int isum = block_isum(p.atype, qw_code(wq, arow, blk), xrow + blk * 32);
            const float dd = __fmul_rn(h2f(qw_scale(wq, arow, blk)), h2f(xd[blk]));
            acc = __fmaf_rn(dd, (float)isum, acc);
        }
        p.out[w] = acc;
    }
}

__device__ __forceinline__ float lda(int t, const char *p) {
    return t == T_F16 ? __half2float(*(const __half *)p) : (t == T_BF16 ? __bfloat162float(*(const __nv_bfloat16 *)p) : *(const float *)p);
}

// One warp per output element, f32/f16 weight. An f16 weight sees the activation rounded to f16.
__global__ void mm_float_kernel(MMk p, int64_t anb0) {
    const int lane = threadIdx.x & 31;
    const int64_t nout = p.N * p.M * p.B2 * p.B3;
    for (int64_t w = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; w < nout;
         w += ((int64_t)gridDim.x * blockDim.x) >> 5) {
        const int64_t n = w % p.N;
        const int64_t r = w / p.N;
        const int64_t m = r % p.M, i2 = (r / p.M) % p.B2, i3 = r / (p.M * p.B2);
        const int64_t a2 = i2 / (p.B2 / p.A2), a3 = i3 / (p.B3 / p.A3);
        const char *arow = p.a + n * p.anb1 + a2 * p.anb2 + a3 * p.anb3;
        const char *brow = p.b + m * p.bnb1 + i2 * p.bnb2 + i3 * p.bnb3;
        float acc = 0.0f;
        for (int64_t k = lane; k < p.K; k += 32) {
            float x = lda(p.btype, brow + k * p.bnb0);
            if (p.atype == T_F16) x = __half2float(__float2half_rn(x));
            else if (p.atype == T_BF16) x = __bfloat162float(__float2bfloat16_rn(x));
            acc = __fmaf_rn(lda(p.atype, arow + k * anb0), x, acc);
        }
        acc = warp_butterfly(acc);
        if (lane == 0) p.out[w] = acc;
    }
}

unsigned warps_grid(int64_t warps) {
    int64_t b = (warps + 7) / 8;
    if (b > 148 * 32) b = 148 * 32;
    return (unsigned)(b < 1 ? 1 : b);
}

MMk make(const TD &a, const TD &b, const TD &out) {
    MMk p{};
    p.a = a.data;
    p.as = a.scales;
    p.atype = (int)a.type;
    p.K = a.ne[0];
    p.N = a.ne[1];
    p.A2 = a.ne[2];
    p.A3 = a.ne[3];
    p.anb1 = a.nb[1];
    p.anb2 = a.nb[2];
    p.anb3 = a.nb[3];
    p.b = b.data;
    p.btype = (int)b.type;
    p.M = b.ne[1];
    p.B2 = b.ne[2];
    p.B3 = b.ne[3];
    p.bnb0 = b.nb[0];
    p.bnb1 = b.nb[1];
    p.bnb2 = b.nb[2];
    p.bnb3 = b.nb[3];
    p.out = (float *)out.data;
    return p;
}

}  // namespace

size_t mul_mat_scratch_bytes(const TD &a, const TD &b) {
    if (raw_block_type(a.type)) return mul_mat_block_scratch_bytes(a, b);
    if (a.type != T_Q4_0 && a.type != T_Q8_0) return 0;
    const int64_t rows = b.ne[1] * b.ne[2] * b.ne[3];
    const size_t q = (size_t)(rows * a.ne[0]);
    return (q + 255) / 256 * 256 + (size_t)(rows * (a.ne[0] / 32)) * 2 + 256;
}

void mul_mat(const TD &a, const TD &b, const TD &out, void *scratch, cudaStream_t s, int *err) {
    if (raw_block_type(a.type)) {
        mul_mat_block(a, b, out, scratch, s);
        return;
    }
    MMk p = make(a, b, out);
    const int64_t nout = p.N * p.M * p.B2 * p.B3;
    if (a.type == T_Q4_0 || a.type == T_Q8_0) {
        const int64_t rows = p.M * p.B2 * p.B3;
        int8_t *qx = (int8_t *)scratch;
        uint16_t *dx = (uint16_t *)((char *)scratch + ((size_t)(rows * p.K) + 255) / 256 * 256);
        act_quant_kernel<<<warps_grid(rows * (p.K / 32)), 256, 0, s>>>(p, qx, dx);
        check_launch("act_quant");
        if (gemm_tc_ok(a, b) && !std::getenv("GCB_NO_TC_GEMM")) {
            gemm_tc(a, p.M, qx, dx, (float *)out.data, err, s);
        } else if (p.M >= GEMM_MIN_ROWS) {
            mm_quant_seq_kernel<<<(unsigned)std::min<int64_t>((nout + 255) / 256, 1 << 20), 256, 0, s>>>(p, qx, dx);
        } else {
            mm_quant_kernel<<<warps_grid(nout), 256, 0, s>>>(p, qx, dx);
        }
        check_launch("mul_mat_q");
    } else {
        mm_float_kernel<<<warps_grid(nout), 256, 0, s>>>(p, a.nb[0]);
        check_launch("mul_mat_f");
    }
}

}  // namespace k
}  // namespace gcb
