// Tensor-parallel exchange over NVLink peer memory: after a step whose rows are split over the
// ranks (each rank computed one slice of every row of a buffer), every rank ends up with the whole
// buffer, bit for bit what one GPU computes.
//
// Each rank owns a window (ipc-exported device memory, mapped by every peer): a flag word per
// sender, then two slots that each hold an image of the exchanged buffer. One exchange, on every
// rank, in the same order, run by one CTA per peer (the pairs do not wait for one another):
//   1. seq = this rank's exchange count + 1; slot = seq & 1.
//   2. Push: the rank's own slice of every row -> the same bytes of the slot image in each peer's
//      window (16-byte stores over NVLink).
//   3. Publish: system-scope fence, then flag[rank] = seq in each peer's window (release store).
//   4. Wait (bounded): flag[p] >= seq in the local window for every peer p (acquire loads).
//   5. Pull: every peer's slice from the local slot image -> the local buffer.
// A slot is rewritten two exchanges later. By then the writer has passed the wait of the exchange
// in between, whose flag the reader sets only after its own earlier exchange (the one reading the
// slot) has finished: stream order on the reader, so no slot is overwritten while it is read.
//
// The kernel is launched with programmatic stream serialization and triggers its dependents at
// once, so the next GEMV streams its weights while the exchange waits; every kernel reads its
// inputs only after griddepcontrol.wait, which covers the exchange's writes.
//
// Waits give up after a time limit and set error word 4 (and skip the pull); a rank whose error
// word is already set does not wait at all, so a dead peer costs one time-out, not one per
// exchange.
#include <stdexcept>
#include <string>

#include "../gc_kernels.h"
#include "gc_tma.cuh"

namespace gcb {
namespace k {

namespace {

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Copies `rows` rows of `bytes` (a multiple of 16) from src (stride ls) to dst (stride ld).
// `cg`: load through L2 only (data that another GPU wrote).
__device__ __forceinline__ void copy_rows(char *dst, int64_t ld, const char *src, int64_t ls, int64_t rows, int64_t bytes,
                                          bool cg) {
    const int64_t per = bytes / 16, n = rows * per;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        const int64_t r = i / per, c = (i - r * per) * 16;
        const int4 *s = (const int4 *)(src + r * ls + c);
        *(int4 *)(dst + r * ld + c) = cg ? __ldcg(s) : *s;
    }
}

// One CTA per peer p: push this rank's slice into p's window, publish to p, wait for p's flag,
// pull p's slice. The pairs run in parallel; the last CTA to finish advances the exchange count.
__global__ void __launch_bounds__(256) tp_exchange_kernel(TpExchange x) {
    __shared__ unsigned s_seq;
    __shared__ int s_fail;
    // Launched early (PDL): let the next kernel start too (its weight stream reads nothing this
    // kernel writes; its griddepcontrol.wait covers the rest), then wait for the slices' producer.
    pdl_trigger();
    pdl_wait();
    const int p = (int)blockIdx.x < x.rank ? (int)blockIdx.x : (int)blockIdx.x + 1;  // this CTA's peer
    if (threadIdx.x == 0) {
        s_seq = *x.seq + 1;
        s_fail = *(volatile int *)x.err != 0;
    }
    __syncthreads();
    const unsigned seq = s_seq;
    const int64_t slot_off = TP_FLAG_BYTES + (int64_t)(seq & 1u) * x.slot_bytes;
    const int64_t own0 = x.col[x.rank], own = x.col[x.rank + 1] - own0;
    if (!s_fail) copy_rows(x.win[p] + slot_off + own0, x.row_bytes, x.buf + own0, x.ld, x.rows, own, false);
    __syncthreads();
    if (threadIdx.x == 0 && !s_fail) {
        __threadfence_system();
        st_release_sys((unsigned *)x.win[p] + x.rank, seq);
        const unsigned *flag = (const unsigned *)x.win[x.rank] + p;
        const uint64_t t0 = globaltimer();
        while ((int)(ld_acquire_sys(flag) - seq) < 0) {
            if (globaltimer() - t0 > x.timeout_ns) {
                atomicCAS(x.err, 0, 4);
                s_fail = 1;
                break;
            }
            __nanosleep(64);
        }
    }
    __syncthreads();
    if (!s_fail)
        copy_rows(x.buf + x.col[p], x.ld, x.win[x.rank] + slot_off + x.col[p], x.row_bytes, x.rows, x.col[p + 1] - x.col[p],
                  true);
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(x.done, 1u) == gridDim.x - 1) {  // every CTA has read the count: advance it
            *x.done = 0;
            *x.seq = seq;
        }
    }
}

}  // namespace

bool tp_exchange_ok(const TpExchange &x) {
    if (x.world < 2 || x.world > TP_MAX || x.rank < 0 || x.rank >= x.world || x.rows < 1) return false;
    if (x.col[0] != 0 || x.col[x.world] != x.row_bytes || x.row_bytes > x.ld) return false;
    for (int r = 0; r < x.world; r++)
        if (x.col[r] % 16 || x.col[r + 1] < x.col[r]) return false;
    if (x.row_bytes % 16 || x.ld % 16) return false;
    return x.rows * x.row_bytes <= x.slot_bytes;
}

void tp_exchange(const TpExchange &x, cudaStream_t s) {
    if (!tp_exchange_ok(x) || (uintptr_t)x.buf % 16)
        throw std::runtime_error("tp_exchange: slices are not 16-byte aligned or exceed the window slot");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(x.world - 1));
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, tp_exchange_kernel, x);
    if (e != cudaSuccess) throw std::runtime_error(std::string("CUDA launch of tp_exchange failed: ") + cudaGetErrorString(e));
}

}  // namespace k
}  // namespace gcb
