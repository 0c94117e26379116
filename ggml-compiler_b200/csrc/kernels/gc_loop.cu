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
#include <cuda_runtime.h>

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

}  // namespace

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
