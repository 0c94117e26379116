// Generic kernels for the LLM op subset of ggml-compiler programs: copies and casts, broadcast
// binary ops, unary ops, row norms, softmax, rope, row gather/scatter, argmax, swiglu and a few
// layout ops. Every kernel takes strided views (ggml's ne/nb). The reductions follow the fixed
// orders the CPU checker restates (see gc_math.cuh), so results do not depend on the launch shape.
#include <algorithm>
#include <cstdio>
#include <stdexcept>
#include <string>

#include "../gc_kernels.h"
#include "gc_blockq.cuh"
#include "gc_math.cuh"
#include "gc_qweight.cuh"

namespace gcb {

size_t TD::elsize() const {
    switch (type) {
        case T_F32: case T_I32: return 4;
        case T_F16: case T_BF16: case T_I16: return 2;
        case T_I8: return 1;
        case T_I64: case T_F64: return 8;
        default: return 0;
    }
}

size_t quant_code_bytes(Type t) { return t == T_Q4_0 ? 16 : (t == T_Q8_0 ? 32 : 0); }

void set_contiguous(TD &t) {
    if (t.type == T_Q4_0 || t.type == T_Q8_0) {
        t.nb[0] = 1;
        t.nb[1] = (int64_t)(t.ne[0] / 32 * quant_code_bytes(t.type));
    } else if (is_quantized(t.type)) {  // other block formats: GGUF rows (ggml's nb)
        const TypeTraits *tr = type_traits(t.type);
        t.nb[0] = tr ? tr->block_size : 0;
        t.nb[1] = (int64_t)row_size(t.type, t.ne[0]);
    } else {
        t.nb[0] = (int64_t)t.elsize();
        t.nb[1] = t.nb[0] * t.ne[0];
    }
    t.nb[2] = t.nb[1] * t.ne[1];
    t.nb[3] = t.nb[2] * t.ne[2];
}

bool TD::contiguous() const {
    TD c = *this;
    set_contiguous(c);
    for (int i = 0; i < 4; i++)
        if (ne[i] > 1 && nb[i] != c.nb[i]) return false;
    return true;
}

size_t TD::nbytes() const {
    TD c = *this;
    set_contiguous(c);
    return (size_t)(c.nb[3] * ne[3]);
}

namespace k {

namespace {

struct Dk {  // kernel-side view
    char *data;
    int type;
    int64_t ne0, ne1, ne2, ne3;
    int64_t nb0, nb1, nb2, nb3;
};

Dk dk(const TD &t) {
    return Dk{t.data, (int)t.type, t.ne[0], t.ne[1], t.ne[2], t.ne[3], t.nb[0], t.nb[1], t.nb[2], t.nb[3]};
}

void check_launch(const char *what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) throw std::runtime_error(std::string("CUDA launch of ") + what + " failed: " + cudaGetErrorString(e));
}

unsigned blocks_for(int64_t n, int threads) {
    int64_t b = (n + threads - 1) / threads;
    if (b > 148 * 64) b = 148 * 64;
    return (unsigned)(b < 1 ? 1 : b);
}

__device__ __forceinline__ char *at(const Dk &t, int64_t i0, int64_t i1, int64_t i2, int64_t i3) {
    return t.data + i0 * t.nb0 + i1 * t.nb1 + i2 * t.nb2 + i3 * t.nb3;
}

__device__ __forceinline__ char *at_lin(const Dk &t, int64_t i) {
    const int64_t i0 = i % t.ne0;
    i /= t.ne0;
    const int64_t i1 = i % t.ne1;
    i /= t.ne1;
    const int64_t i2 = i % t.ne2;
    const int64_t i3 = i / t.ne2;
    return at(t, i0, i1, i2, i3);
}

__device__ __forceinline__ float ldf(const char *p, int type) {
    switch (type) {
        case T_F32: return *(const float *)p;
        case T_F16: return __half2float(*(const __half *)p);
        case T_BF16: return __bfloat162float(*(const __nv_bfloat16 *)p);
        case T_I32: return (float)*(const int32_t *)p;
        default: return 0.0f;
    }
}

__device__ __forceinline__ void stf(char *p, int type, float v) {
    switch (type) {
        case T_F32: *(float *)p = v; break;
        case T_F16: *(__half *)p = __float2half_rn(v); break;
        case T_BF16: *(__nv_bfloat16 *)p = __float2bfloat16_rn(v); break;
        case T_I32: *(int32_t *)p = (int32_t)v; break;
        default: break;
    }
}

// ------------------------------------------------------------------------------------------------

// GGUF blocks (row-major, 18 or 34 bytes) -> the tiled device layout (gc_qweight.cuh).
__global__ void repack_kernel(int type, const uint8_t *raw, int64_t rows, int64_t nb, char *dst) {
    const int bs = type == T_Q4_0 ? 18 : 34;
    const int cb = type == T_Q4_0 ? 16 : 32;
    const QW w{dst, nb, cb};
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < rows * nb; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = t / nb, blk = t % nb;
        const uint8_t *src = raw + t * bs;
        char *code = (char *)qw_code(w, row, blk);
        uint32_t words[8];
        for (int i = 0; i < cb / 4; i++)
            words[i] = (uint32_t)src[2 + 4 * i] | ((uint32_t)src[3 + 4 * i] << 8) | ((uint32_t)src[4 + 4 * i] << 16) |
                       ((uint32_t)src[5 + 4 * i] << 24);
        *(uint4 *)code = make_uint4(words[0], words[1], words[2], words[3]);
        if (cb == 32) *(uint4 *)(code + 16) = make_uint4(words[4], words[5], words[6], words[7]);
        const int64_t g = blk / QSEG, sb = qw_seg_blocks(nb, g);
        uint16_t *sc = (uint16_t *)(dst + qw_piece_off(nb, cb, row / QTR, g) + QTR * sb * cb);
        sc[(row % QTR) * sb + blk % QSEG] = (uint16_t)(src[0] | (src[1] << 8));
    }
}

__global__ void copy_kernel(Dk src, Dk dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const char *s = at_lin(src, i);
        char *d = at_lin(dst, i);
        if (src.type == dst.type) {
            switch (src.type) {
                case T_F32: case T_I32: *(uint32_t *)d = *(const uint32_t *)s; break;
                case T_F16: case T_BF16: *(uint16_t *)d = *(const uint16_t *)s; break;
                default: break;
            }
        } else if (src.type == T_I32 && dst.type == T_F32) {
            *(float *)d = (float)*(const int32_t *)s;
        } else if (src.type == T_F32 && dst.type == T_I32) {
            *(int32_t *)d = (int32_t)*(const float *)s;
        } else {
            stf(d, dst.type, ldf(s, src.type));
        }
    }
}

__device__ __forceinline__ float binop(int op, float a, float b) {
    switch (op) {
        case ADD: return __fadd_rn(a, b);
        case SUB: return __fsub_rn(a, b);
        case MUL: return __fmul_rn(a, b);
        default: return __fdiv_rn(a, b);
    }
}

// Contiguous f32 operands: four elements per step. b either has a's shape (bper4 = 0) or is one
// contiguous row of bper4 * 4 elements repeated over a's rows.
__global__ void binary_f32x4_kernel(int op, const float4 *a, const float4 *b, float4 *out, int64_t n4, int64_t bper4) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
        const float4 x = a[i], y = b[bper4 ? i % bper4 : i];
        out[i] = make_float4(binop(op, x.x, y.x), binop(op, x.y, y.y), binop(op, x.z, y.z), binop(op, x.w, y.w));
    }
}

__global__ void binary_kernel(int op, Dk a, Dk b, Dk out, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t r = i;
        const int64_t i0 = r % a.ne0;
        r /= a.ne0;
        const int64_t i1 = r % a.ne1;
        r /= a.ne1;
        const int64_t i2 = r % a.ne2;
        const int64_t i3 = r / a.ne2;
        const float x = ldf(at(a, i0, i1, i2, i3), a.type);
        const float y = ldf(at(b, i0 % b.ne0, i1 % b.ne1, i2 % b.ne2, i3 % b.ne3), b.type);
        stf(at(out, i0, i1, i2, i3), out.type, binop(op, x, y));
    }
}

__device__ float unop(int op, float x, float p0, float p1) {
    switch (op) {
        case SCALE: return __fadd_rn(__fmul_rn(x, p0), p1);
        case CLAMP: return fminf(fmaxf(x, p0), p1);
        case SILU: return gc_silu(x);
        case NEG: return -x;
        case ABS: return fabsf(x);
        case SQR: return __fmul_rn(x, x);
        case SQRT: return __fsqrt_rn(x);
        case EXP: return gc_expf(x);
        case LOG: return logf(x);
        case RELU: return x > 0.0f ? x : 0.0f;
        case TANH: return tanhf(x);
        case SIGMOID: return __fdiv_rn(1.0f, __fadd_rn(1.0f, gc_expf(-x)));
        case STEP: return x > 0.0f ? 1.0f : 0.0f;
        case SIN: return sinf(x);
        case COS: return cosf(x);
        case SOFTPLUS: return x > 20.0f ? x : log1pf(gc_expf(x));
        case GELU_TANH: {
            const float inner = __fmul_rn(0.7978845608f, __fadd_rn(x, __fmul_rn(0.044715f, __fmul_rn(__fmul_rn(x, x), x))));
            return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner)));
        }
        case GELU_ERF: return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, erff(__fmul_rn(x, 0.70710678118654752f))));
        default: return x;
    }
}

__global__ void unary_kernel(int op, Dk x, Dk out, int64_t n, float p0, float p1) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        stf(at_lin(out, i), out.type, unop(op, ldf(at_lin(x, i), x.type), p0, p1));
}

// One block of 256 threads per row; the sum of squares is a double 256-way tree.
__global__ void rms_norm_kernel(Dk x, Dk out, float eps) {
    __shared__ double sh[256];
    const int64_t row = blockIdx.x;
    const int64_t i1 = row % x.ne1, i2 = (row / x.ne1) % x.ne2, i3 = row / (x.ne1 * x.ne2);
    const float *xr = (const float *)at(x, 0, i1, i2, i3);
    float *yr = (float *)at(out, 0, i1, i2, i3);
    double p = 0.0;
    for (int64_t i = threadIdx.x; i < x.ne0; i += 256) p = __dadd_rn(p, (double)__fmul_rn(xr[i], xr[i]));
    const double tot = block_tree256(p, sh);
    const float mean = __double2float_rn(__ddiv_rn(tot, (double)x.ne0));
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    for (int64_t i = threadIdx.x; i < x.ne0; i += 256) yr[i] = __fmul_rn(xr[i], scale);
}

// ggml_norm: (x - mean) / sqrt(var + eps), both sums as double 256-way trees.
__global__ void norm_kernel(Dk x, Dk out, float eps) {
    __shared__ double sh[256];
    const int64_t row = blockIdx.x;
    const int64_t i1 = row % x.ne1, i2 = (row / x.ne1) % x.ne2, i3 = row / (x.ne1 * x.ne2);
    const float *xr = (const float *)at(x, 0, i1, i2, i3);
    float *yr = (float *)at(out, 0, i1, i2, i3);
    double p = 0.0;
    for (int64_t i = threadIdx.x; i < x.ne0; i += 256) p = __dadd_rn(p, (double)xr[i]);
    const float mean = __double2float_rn(__ddiv_rn(block_tree256(p, sh), (double)x.ne0));
    double q = 0.0;
    for (int64_t i = threadIdx.x; i < x.ne0; i += 256) {
        const float v = __fsub_rn(xr[i], mean);
        yr[i] = v;
        q = __dadd_rn(q, (double)__fmul_rn(v, v));
    }
    const float var = __double2float_rn(__ddiv_rn(block_tree256(q, sh), (double)x.ne0));
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    __syncthreads();
    for (int64_t i = threadIdx.x; i < x.ne0; i += 256) yr[i] = __fmul_rn(yr[i], scale);
}

// softmax(x * scale + mask) per row. The row is staged in `out` (same shape, contiguous rows).
__global__ void soft_max_kernel(Dk x, Dk mask, int has_mask, Dk out, float scale) {
    __shared__ double sh[256];
    __shared__ float smax[8];
    const int64_t row = blockIdx.x;
    const int64_t i1 = row % x.ne1, i2 = (row / x.ne1) % x.ne2, i3 = row / (x.ne1 * x.ne2);
    const char *xr = at(x, 0, i1, i2, i3);
    float *yr = (float *)at(out, 0, i1, i2, i3);
    const char *mr = has_mask ? at(mask, 0, i1, i2 % mask.ne2, i3 % mask.ne3) : nullptr;
    float mx = -__int_as_float(0x7f800000);
    for (int64_t i = threadIdx.x; i < x.ne0; i += 256) {
        float w = __fmul_rn(ldf(xr + i * x.nb0, x.type), scale);
        w = __fadd_rn(w, has_mask ? ldf(mr + i * mask.nb0, mask.type) : 0.0f);
        yr[i] = w;
        mx = fmaxf(mx, w);
    }
    mx = warp_max(mx);
    if ((threadIdx.x & 31) == 0) smax[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = smax[0];
    for (int w = 1; w < 8; w++) mx = fmaxf(mx, smax[w]);
    double p = 0.0;
    for (int64_t i = threadIdx.x; i < x.ne0; i += 256) {
        const float e = gc_expf(__fsub_rn(yr[i], mx));
        yr[i] = e;
        p = __dadd_rn(p, (double)e);
    }
    const float inv = __double2float_rn(__ddiv_rn(1.0, block_tree256(p, sh)));
    for (int64_t i = threadIdx.x; i < x.ne0; i += 256) yr[i] = __fmul_rn(yr[i], inv);
}

// rope: one thread per rotated pair. x [D, H, S, B] (rows may be strided), pos [S] i32.
// The cos/sin table [npos][n_dims/2][2] is built on the host with the CPU's libm; positions
// outside it compute the angle on the device the same way, with CUDA's cosf/sinf.
__global__ void rope_kernel(int neox, Dk x, const int32_t *pos, Dk out, int n_dims, const float *table, int64_t npos,
                            float theta_scale, float freq_scale, float attn_factor, const float *ff) {
    const int64_t D = x.ne0, H = x.ne1, S = x.ne2, B = x.ne3;
    const int half = n_dims / 2;
    const int64_t per_row = D - half;  // half rotated pairs + (D - n_dims) passthrough elements
    const int64_t n = per_row * H * S * B;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t % per_row;
        int64_t r = t / per_row;
        const int64_t h = r % H;
        r /= H;
        const int64_t s = r % S;
        const int64_t b = r / S;
        const float *xr = (const float *)at(x, 0, h, s, b);
        float *yr = (float *)at(out, 0, h, s, b);
        if (i >= half) {  // elements past n_dims pass through
            const int64_t d = n_dims + (i - half);
            yr[d] = xr[d];
            continue;
        }
        const int32_t p = pos[s];
        float c, sn;
        if (p >= 0 && p < npos && table) {
            c = table[(p * half + i) * 2];
            sn = table[(p * half + i) * 2 + 1];
        } else {
            float theta = (float)p;
            for (int64_t k = 0; k < i; k++) theta = __fmul_rn(theta, theta_scale);
            float tt = ff ? __fdiv_rn(theta, ff[i]) : theta;
            tt = __fmul_rn(freq_scale, tt);
            c = __fmul_rn(cosf(tt), attn_factor);
            sn = __fmul_rn(sinf(tt), attn_factor);
        }
        const int64_t j0 = neox ? i : 2 * i, j1 = neox ? i + half : 2 * i + 1;
        const float x0 = xr[j0], x1 = xr[j1];
        yr[j0] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
        yr[j1] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
    }
}

// get_rows: out[:, i10, i11, i12] = table[:, idx[i10, i11, i12], i11, i12] as f32.
__global__ void get_rows_kernel(Dk tab, Dk idx, Dk out) {
    const int64_t n = out.ne0 * out.ne1 * out.ne2 * out.ne3;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i0 = t % out.ne0;
        int64_t r = t / out.ne0;
        const int64_t i10 = r % out.ne1;
        r /= out.ne1;
        const int64_t i11 = r % out.ne2;
        const int64_t i12 = r / out.ne2;
        const int64_t row = *(const int32_t *)at(idx, i10, i11, i12, 0);
        float v = 0.0f;
        if (row >= 0 && row < tab.ne1) {
            if (tab.type == T_Q4_0 || tab.type == T_Q8_0) {
                const QW w{tab.data, tab.ne0 / 32, tab.type == T_Q4_0 ? 16 : 32};
                const int64_t rr = row + tab.ne1 * (i11 + tab.ne2 * i12);
                const char *codes = qw_code(w, rr, i0 / 32);
                const float d = h2f(qw_scale(w, rr, i0 / 32));
                const int j = (int)(i0 % 32);
                int q;
                if (tab.type == T_Q8_0) {
                    q = (int8_t)codes[j];
                } else {
                    const uint8_t byte = (uint8_t)codes[j & 15];
                    q = (j < 16 ? (byte & 15) : (byte >> 4)) - 8;
                }
                v = __fmul_rn(d, (float)q);
            } else if (tab.type == T_Q4_1 || tab.type == T_Q5_1 || tab.type == T_Q4_K || tab.type == T_Q5_K ||
                       tab.type == T_Q6_K) {
                v = dequant_raw(tab.type, (const uint8_t *)tab.data + row * tab.nb1 + i11 * tab.nb2 + i12 * tab.nb3, i0);
            } else {
                v = ldf(at(tab, i0, row, i11, i12), tab.type);
            }
        }
        stf(at(out, i0, i10, i11, i12), out.type, v);
    }
}

// set_rows: dst[:, idx[i], i2, i3] = src[:, i, i2, i3]; out-of-range indices are skipped and flagged.
__global__ void set_rows_kernel(Dk dst, Dk src, Dk idx, int *err) {
    const int64_t n = src.ne0 * src.ne1 * src.ne2 * src.ne3;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i0 = t % src.ne0;
        int64_t r = t / src.ne0;
        const int64_t i1 = r % src.ne1;
        r /= src.ne1;
        const int64_t i2 = r % src.ne2;
        const int64_t i3 = r / src.ne2;
        const int64_t row = *(const int32_t *)at(idx, i1, i2 % idx.ne1, i3 % idx.ne2, 0);
        if (row < 0 || row >= dst.ne1) {
            if (err) atomicExch(err, 1);
            continue;
        }
        stf(at(dst, i0, row, i2, i3), dst.type, ldf(at(src, i0, i1, i2, i3), src.type));
    }
}

// argmax over ne0 for each row: first index of the maximum.
__global__ void argmax_kernel(Dk x, Dk out) {
    __shared__ float sv[32];
    __shared__ int32_t si[32];
    const int64_t row = blockIdx.x;
    const char *xr = at(x, 0, row % x.ne1, (row / x.ne1) % x.ne2, row / (x.ne1 * x.ne2));
    float best = -__int_as_float(0x7f800000);
    int32_t bi = 0x7fffffff;
    for (int64_t i = threadIdx.x; i < x.ne0; i += blockDim.x) {
        const float v = ldf(xr + i * x.nb0, x.type);
        if (v > best || (v == best && (int32_t)i < bi)) {
            best = v;
            bi = (int32_t)i;
        }
    }
    for (int off = 16; off >= 1; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, off);
        const int32_t oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (ov > best || (ov == best && oi < bi)) {
            best = ov;
            bi = oi;
        }
    }
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        sv[w] = best;
        si[w] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int k = 1; k < nw; k++)
            if (sv[k] > best || (sv[k] == best && si[k] < bi)) {
                best = sv[k];
                bi = si[k];
            }
        if (bi == 0x7fffffff) bi = 0;
        *(int32_t *)at(out, row, 0, 0, 0) = bi;
    }
}

// argmax of long rows over `gridDim.x` CTAs per row: each CTA reduces one slice of f32 elements
// (contiguous rows) to its (max, first index) pair, and the last CTA of the row to finish combines
// the pairs in slice order with the same rule, so the result is the first index of the maximum.
__global__ void argmax_split_kernel(const float *x, int64_t ne0, int64_t ld, int32_t *out, float2 *part, int *counters) {
    __shared__ float sv[32];
    __shared__ int32_t si[32];
    __shared__ int last;
    const int64_t row = blockIdx.y, P = gridDim.x, p = blockIdx.x;
    const int64_t chunk = (ne0 + P - 1) / P, i0 = p * chunk, i1 = min(ne0, i0 + chunk);
    const float *xr = x + row * ld;
    float best = -__int_as_float(0x7f800000);
    int32_t bi = 0x7fffffff;
    for (int64_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
        const float v = xr[i];
        if (v > best || (v == best && (int32_t)i < bi)) {
            best = v;
            bi = (int32_t)i;
        }
    }
    for (int off = 16; off >= 1; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, off);
        const int32_t oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (ov > best || (ov == best && oi < bi)) {
            best = ov;
            bi = oi;
        }
    }
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        sv[w] = best;
        si[w] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int k = 1; k < nw; k++)
            if (sv[k] > best || (sv[k] == best && si[k] < bi)) {
                best = sv[k];
                bi = si[k];
            }
        part[row * P + p] = make_float2(best, __int_as_float(bi));
        __threadfence();
        last = atomicAdd(&counters[row], 1) == (int)P - 1;
        if (last) {
            counters[row] = 0;
            __threadfence();
            best = -__int_as_float(0x7f800000);
            bi = 0x7fffffff;
            for (int64_t k = 0; k < P; k++) {
                const float2 q = __ldcg(&part[row * P + k]);
                const int32_t qi = __float_as_int(q.y);
                if (q.x > best || (q.x == best && qi < bi)) {
                    best = q.x;
                    bi = qi;
                }
            }
            if (bi == 0x7fffffff) bi = 0;
            out[row] = bi;
        }
    }
}

__global__ void swiglu_f32x4_kernel(const float4 *g, const float4 *u, float4 *out, int64_t n4) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
        const float4 a = g[i], b = u[i];
        out[i] = make_float4(__fmul_rn(gc_silu(a.x), b.x), __fmul_rn(gc_silu(a.y), b.y), __fmul_rn(gc_silu(a.z), b.z),
                             __fmul_rn(gc_silu(a.w), b.w));
    }
}

__global__ void swiglu_kernel(Dk g, Dk u, Dk out, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float a = ldf(at_lin(g, i), g.type), b = ldf(at_lin(u, i), u.type);
        stf(at_lin(out, i), out.type, __fmul_rn(gc_silu(a), b));
    }
}

__global__ void sum_rows_kernel(Dk x, Dk out, float scale) {
    __shared__ double sh[256];
    const int64_t row = blockIdx.x;
    const int64_t i1 = row % x.ne1, i2 = (row / x.ne1) % x.ne2, i3 = row / (x.ne1 * x.ne2);
    const char *xr = at(x, 0, i1, i2, i3);
    double p = 0.0;
    for (int64_t i = threadIdx.x; i < x.ne0; i += 256) p = __dadd_rn(p, (double)ldf(xr + i * x.nb0, x.type));
    const double tot = block_tree256(p, sh);
    if (threadIdx.x == 0) stf(at(out, 0, i1, i2, i3), out.type, __fmul_rn(__double2float_rn(tot), scale));
}

__global__ void repeat_kernel(Dk x, Dk out, int64_t n) {
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        int64_t r = t;
        const int64_t i0 = r % out.ne0;
        r /= out.ne0;
        const int64_t i1 = r % out.ne1;
        r /= out.ne1;
        const int64_t i2 = r % out.ne2;
        const int64_t i3 = r / out.ne2;
        stf(at(out, i0, i1, i2, i3), out.type, ldf(at(x, i0 % x.ne0, i1 % x.ne1, i2 % x.ne2, i3 % x.ne3), x.type));
    }
}

__global__ void concat_kernel(Dk a, Dk b, Dk out, int dim, int64_t n) {
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        int64_t r = t;
        int64_t i[4];
        i[0] = r % out.ne0;
        r /= out.ne0;
        i[1] = r % out.ne1;
        r /= out.ne1;
        i[2] = r % out.ne2;
        i[3] = r / out.ne2;
        const int64_t ane[4] = {a.ne0, a.ne1, a.ne2, a.ne3};
        float v;
        if (i[dim] < ane[dim]) {
            v = ldf(at(a, i[0], i[1], i[2], i[3]), a.type);
        } else {
            i[dim] -= ane[dim];
            v = ldf(at(b, i[0], i[1], i[2], i[3]), b.type);
            i[dim] += ane[dim];
        }
        stf(at(out, i[0], i[1], i[2], i[3]), out.type, v);
    }
}

__global__ void arange_kernel(float *out, int64_t n, float start, float step) {
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x)
        out[t] = __fadd_rn(start, __fmul_rn((float)t, step));
}

__global__ void fill_kernel(float *out, int64_t n, float v) {
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) out[t] = v;
}

}  // namespace

void repack_quant(Type t, const uint8_t *raw, int64_t nrows, int64_t K, char *dst, cudaStream_t s) {
    const int64_t nblocks = nrows * (K / 32);
    repack_kernel<<<blocks_for(nblocks, 256), 256, 0, s>>>((int)t, raw, nrows, K / 32, dst);
    check_launch("repack_quant");
}

size_t quant_device_bytes(Type t, int64_t rows, int64_t K) { return (size_t)qw_total_bytes(rows, K / 32, (int)quant_code_bytes(t)); }

void copy(const TD &src, const TD &dst, cudaStream_t s) {
    const int64_t n = dst.nelements();
    if (n == 0) return;
    copy_kernel<<<blocks_for(n, 256), 256, 0, s>>>(dk(src), dk(dst), n);
    check_launch("copy");
}

namespace {
// Contiguous f32 with 16-byte aligned data and a multiple of 4 elements.
bool f32x4_ok(const TD &t) { return t.type == T_F32 && t.contiguous() && (uintptr_t)t.data % 16 == 0 && t.nelements() % 4 == 0; }
}  // namespace

void binary(int op, const TD &a, const TD &b, const TD &out, cudaStream_t s) {
    const int64_t n = a.nelements();
    if (f32x4_ok(a) && f32x4_ok(b) && f32x4_ok(out) && out.nelements() == n) {
        const bool same = b.nelements() == n && b.ne[0] == a.ne[0] && b.ne[1] == a.ne[1] && b.ne[2] == a.ne[2];
        const bool row = b.ne[0] == a.ne[0] && b.nelements() == b.ne[0];  // one row broadcast over a's rows
        if (same || row) {
            binary_f32x4_kernel<<<blocks_for(n / 4, 256), 256, 0, s>>>(op, (const float4 *)a.data, (const float4 *)b.data,
                                                                       (float4 *)out.data, n / 4, same ? 0 : b.ne[0] / 4);
            check_launch("binary");
            return;
        }
    }
    binary_kernel<<<blocks_for(n, 256), 256, 0, s>>>(op, dk(a), dk(b), dk(out), n);
    check_launch("binary");
}

void unary(int op, const TD &x, const TD &out, float p0, float p1, cudaStream_t s) {
    const int64_t n = x.nelements();
    unary_kernel<<<blocks_for(n, 256), 256, 0, s>>>(op, dk(x), dk(out), n, p0, p1);
    check_launch("unary");
}

void rms_norm(const TD &x, const TD &out, float eps, cudaStream_t s) {
    rms_norm_kernel<<<(unsigned)x.nrows(), 256, 0, s>>>(dk(x), dk(out), eps);
    check_launch("rms_norm");
}

void norm(const TD &x, const TD &out, float eps, cudaStream_t s) {
    norm_kernel<<<(unsigned)x.nrows(), 256, 0, s>>>(dk(x), dk(out), eps);
    check_launch("norm");
}

void soft_max(const TD &x, const TD *mask, const TD &out, float scale, cudaStream_t s) {
    Dk m{};
    if (mask) m = dk(*mask);
    soft_max_kernel<<<(unsigned)x.nrows(), 256, 0, s>>>(dk(x), m, mask ? 1 : 0, dk(out), scale);
    check_launch("soft_max");
}

void rope_neox(const TD &x, const TD &pos, const TD &out, int n_dims, const float *table, int64_t npos,
               float theta_scale, float freq_scale, float attn_factor, const float *ff, cudaStream_t s) {
    const int64_t n = (x.ne[0] - n_dims / 2) * x.ne[1] * x.ne[2] * x.ne[3];
    rope_kernel<<<blocks_for(n, 256), 256, 0, s>>>(1, dk(x), (const int32_t *)pos.data, dk(out), n_dims, table, npos,
                                                   theta_scale, freq_scale, attn_factor, ff);
    check_launch("rope");
}

void rope_norm(const TD &x, const TD &pos, const TD &out, int n_dims, const float *table, int64_t npos,
               float theta_scale, float freq_scale, float attn_factor, const float *ff, cudaStream_t s) {
    const int64_t n = (x.ne[0] - n_dims / 2) * x.ne[1] * x.ne[2] * x.ne[3];
    rope_kernel<<<blocks_for(n, 256), 256, 0, s>>>(0, dk(x), (const int32_t *)pos.data, dk(out), n_dims, table, npos,
                                                   theta_scale, freq_scale, attn_factor, ff);
    check_launch("rope");
}

void get_rows(const TD &table, const TD &idx, const TD &out, cudaStream_t s) {
    const int64_t n = out.nelements();
    get_rows_kernel<<<blocks_for(n, 256), 256, 0, s>>>(dk(table), dk(idx), dk(out));
    check_launch("get_rows");
}

void set_rows(const TD &dst, const TD &src, const TD &idx, int *err, cudaStream_t s) {
    const int64_t n = src.nelements();
    set_rows_kernel<<<blocks_for(n, 256), 256, 0, s>>>(dk(dst), dk(src), dk(idx), err);
    check_launch("set_rows");
}

void argmax(const TD &x, const TD &out, cudaStream_t s) {
    argmax_kernel<<<(unsigned)x.nrows(), 1024, 0, s>>>(dk(x), dk(out));
    check_launch("argmax");
}

int argmax_split_parts(const TD &x) {
    if (x.type != T_F32 || x.nb[0] != 4 || !x.contiguous() || x.ne[0] < 16384) return 0;
    return (int)std::min<int64_t>(128, (x.ne[0] + 4095) / 4096);
}

void argmax_split(const TD &x, const TD &out, void *scratch, int *counters, cudaStream_t s) {
    const int P = argmax_split_parts(x);
    argmax_split_kernel<<<dim3((unsigned)P, (unsigned)x.nrows()), 256, 0, s>>>((const float *)x.data, x.ne[0], x.nb[1] / 4,
                                                                               (int32_t *)out.data, (float2 *)scratch, counters);
    check_launch("argmax_split");
}

void swiglu(const TD &g, const TD &u, const TD &out, cudaStream_t s) {
    const int64_t n = g.nelements();
    if (f32x4_ok(g) && f32x4_ok(u) && f32x4_ok(out) && u.nelements() == n && out.nelements() == n) {
        swiglu_f32x4_kernel<<<blocks_for(n / 4, 256), 256, 0, s>>>((const float4 *)g.data, (const float4 *)u.data,
                                                                  (float4 *)out.data, n / 4);
        check_launch("swiglu");
        return;
    }
    swiglu_kernel<<<blocks_for(n, 256), 256, 0, s>>>(dk(g), dk(u), dk(out), n);
    check_launch("swiglu");
}

void sum_rows(const TD &x, const TD &out, float scale, cudaStream_t s) {
    sum_rows_kernel<<<(unsigned)x.nrows(), 256, 0, s>>>(dk(x), dk(out), scale);
    check_launch("sum_rows");
}

void repeat(const TD &x, const TD &out, cudaStream_t s) {
    const int64_t n = out.nelements();
    repeat_kernel<<<blocks_for(n, 256), 256, 0, s>>>(dk(x), dk(out), n);
    check_launch("repeat");
}

void concat(const TD &a, const TD &b, const TD &out, int dim, cudaStream_t s) {
    const int64_t n = out.nelements();
    concat_kernel<<<blocks_for(n, 256), 256, 0, s>>>(dk(a), dk(b), dk(out), dim, n);
    check_launch("concat");
}

void arange(const TD &out, float start, float step, cudaStream_t s) {
    const int64_t n = out.nelements();
    arange_kernel<<<blocks_for(n, 256), 256, 0, s>>>((float *)out.data, n, start, step);
    check_launch("arange");
}

void fill_f32(float *dst, int64_t n, float v, cudaStream_t s) {
    if (n <= 0) return;
    fill_kernel<<<blocks_for(n, 256), 256, 0, s>>>(dst, n, v);
    check_launch("fill");
}


}  // namespace k
}  // namespace gcb
