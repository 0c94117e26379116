// Device side of a driver loop (a `loop` step of an entry's driver, program format 2+).
//
// The per-iteration bookkeeping runs in two one-block kernels that read the iteration index from
// device memory (LoopDev::iter), so one captured iteration is valid for every iteration with the
// same symbol binding:
//   loop_begin:  counters := start + i, mask rows for counter positions (0 up to the position,
//                -inf after), per-iteration scalars, slice rows i of their sources;
//   loop_end:    collect rows i, the stop test (LoopDev::stop := 1 once a stop id is seen), i += 1,
//                and, inside a conditional WHILE graph node, the node's condition for the next
//                iteration: not stopped and i below LoopDev::end.
// loop_guard sets the condition before the WHILE node runs its first iteration.
//
// The batched decode step's two kernels live here too: the per-sequence causal mask rows, built
// from the positions at the start of each step, and the greedy hand-over between steps.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <stdexcept>
#include <string>

#include "../gc_kernels.h"

namespace gcb {
namespace k {

namespace {

__device__ void copy_bytes(char *dst, const char *src, int64_t n) {
    if (((uintptr_t)dst | (uintptr_t)src | (uintptr_t)n) % 16 == 0) {
        for (int64_t i = threadIdx.x; i < n / 16; i += blockDim.x) ((int4 *)dst)[i] = ((const int4 *)src)[i];
    } else {
        for (int64_t i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
    }
}

__global__ void loop_begin_kernel(LoopDev L) {
    const int32_t i = *L.iter;
    if (threadIdx.x < L.n_counters) *L.counter[threadIdx.x] = L.start[threadIdx.x] + i;
    const float ninf = -__int_as_float(0x7f800000);
    for (int k = 0; k < L.n_masks; k++) {
        const int64_t pos = (int64_t)L.start[L.mask_counter[k]] + i, row = L.mask_row[k];
        for (int64_t j = threadIdx.x; j < L.mask_n[k]; j += blockDim.x) L.mask[k][j] = j % row <= pos ? 0.0f : ninf;
    }
    for (int k = 0; k < L.n_scalars; k++) {
        const float v = L.scalar_vals[k][i];
        for (int64_t j = threadIdx.x; j < L.scalar_n[k]; j += blockDim.x) L.scalar[k][j] = v;
    }
    for (int k = 0; k < L.n_slices; k++)
        copy_bytes(L.slice_dst[k], L.slice_src[k] + (int64_t)i * L.slice_bytes[k], L.slice_bytes[k]);
}

__global__ void loop_end_kernel(LoopDev L, cudaGraphConditionalHandle cond, int use_cond) {
    const int32_t i = *L.iter;
    for (int k = 0; k < L.n_collect; k++)
        copy_bytes(L.collect_dst[k] + (int64_t)i * L.collect_bytes[k], L.collect_src[k], L.collect_bytes[k]);
    __syncthreads();  // every thread has read *iter
    if (threadIdx.x == 0) {
        int stop = *L.stop;
        for (int k = 0; k < L.n_until; k++) {
            const int32_t v = *L.until_val[k];
            for (int t = 0; t < L.n_ids[k]; t++) stop |= v == L.until_ids[k][t];
        }
        *L.stop = stop;
        *L.iter = i + 1;
        if (use_cond) cudaGraphSetConditional(cond, !stop && i + 1 < *L.end ? 1u : 0u);
    }
}

__global__ void loop_guard_kernel(const int32_t *iter, const int32_t *stop, const int32_t *end,
                                  cudaGraphConditionalHandle cond) {
    cudaGraphSetConditional(cond, *stop == 0 && *iter < *end ? 1u : 0u);
}

__global__ void batch_mask_kernel(__half *mask, const int32_t *pos, int n, int64_t window) {
    const __half zero = __float2half_rn(0.0f), ninf = __ushort_as_half((unsigned short)0xfc00u);
    for (int b = blockIdx.y; b < n; b += gridDim.y) {
        const int64_t p = pos[b];
        for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < window; j += (int64_t)gridDim.x * blockDim.x)
            mask[(int64_t)b * window + j] = j <= p ? zero : ninf;
    }
}

__global__ void batch_advance_kernel(int32_t *tok, int32_t *pos, const int32_t *next, int32_t *out, int32_t *step, int n) {
    const int i = threadIdx.x;
    const int32_t s = *step;
    __syncthreads();  // every thread has read the step before thread 0 moves it
    if (i < n) {
        tok[i] = next[i];
        pos[i] += 1;
        if (out) out[(int64_t)s * n + i] = next[i];
    }
    if (i == 0) *step = s + 1;
}

}  // namespace

void batch_mask(__half *mask, const int32_t *pos, int n, int64_t window, cudaStream_t s) {
    const unsigned bx = (unsigned)std::min<int64_t>((window + 255) / 256, 16);
    batch_mask_kernel<<<dim3(bx, (unsigned)n), 256, 0, s>>>(mask, pos, n, window);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) throw std::runtime_error(std::string("batch_mask launch: ") + cudaGetErrorString(e));
}

void batch_advance(int32_t *tok, int32_t *pos, const int32_t *next, int32_t *out, int32_t *step, int n, cudaStream_t s) {
    batch_advance_kernel<<<1, 32, 0, s>>>(tok, pos, next, out, step, n);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) throw std::runtime_error(std::string("batch_advance launch: ") + cudaGetErrorString(e));
}

void loop_begin(const LoopDev &L, cudaStream_t s) {
    loop_begin_kernel<<<1, 256, 0, s>>>(L);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) throw std::runtime_error(std::string("loop_begin launch: ") + cudaGetErrorString(e));
}

void loop_end(const LoopDev &L, cudaGraphConditionalHandle cond, bool use_cond, cudaStream_t s) {
    loop_end_kernel<<<1, 256, 0, s>>>(L, cond, use_cond ? 1 : 0);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) throw std::runtime_error(std::string("loop_end launch: ") + cudaGetErrorString(e));
}

void loop_guard(const LoopDev &L, cudaGraphConditionalHandle cond, cudaStream_t s) {
    loop_guard_kernel<<<1, 1, 0, s>>>(L.iter, L.stop, L.end, cond);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) throw std::runtime_error(std::string("loop_guard launch: ") + cudaGetErrorString(e));
}

}  // namespace k
}  // namespace gcb
