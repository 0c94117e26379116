// ggml_compiler_b200_flash_attn_static: the split-KV flash attention kernel (gc_flash.cu) on
// caller-owned device buffers, with its scratch in a static device array, so a call allocates no
// device memory at all.
//
// Who needs it: code that runs one attention step through the C ABI without a loaded program (no
// ggml_compiler_model, hence no call-site arena), inside a host framework that owns the device
// memory, e.g. a custom op in another engine's decode loop. Such a caller cannot let the library
// allocate: the framework's caching allocator already holds the free memory, so cudaMalloc may fail,
// and cudaMalloc / cudaFree synchronise the whole device, stalling the framework's other streams in
// the middle of a step.
//
// The scratch (g_scratch, 4 MiB + 16 KiB + 256 B, zero when the module loads) holds:
//   [0, 4 MiB)               chunk partials (m, l, o[head_dim]) of every (query row, head, chunk);
//                            written before they are read, no initial value needed
//   [4 MiB, 4 MiB + 16 KiB)  up to 4096 arrival counters, one per (query row, K/V head): these must be
//                            zero when a launch starts; each call zeroes them on its stream first
//   [4 MiB + 16 KiB, +256 B) the error word the kernel sets when a bounded wait expires (2 s); the
//                            call zeroes it first and does not read it back (that would synchronise):
//                            the kernel also writes NaN into the output rows it could not compute,
//                            which is how a caller sees the failure
// The first call on each device does the set-up: with that device current it looks up the array's
// device address (cudaGetSymbolAddress), which also makes the driver load the library's device
// code there if it has not yet; make that first call before any stream capture on that device.
// There is one scratch per device: calls whose executions overlap (other streams, other threads)
// race on it and corrupt each other's results; order them (one stream, or events).
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <mutex>
#include <stdexcept>
#include <string>

#include "ggml_compiler_b200.h"
#include "../gc_kernels.h"

void gcb_set_last_error(const std::string &msg);  // gc_capi.cpp

namespace {

constexpr size_t kPartBytes = 4u << 20;
constexpr size_t kMaxCounters = 4096;
constexpr size_t kCounterOff = kPartBytes;
constexpr size_t kErrOff = kCounterOff + kMaxCounters * sizeof(int);
constexpr size_t kScratchBytes = kErrOff + 256;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

std::mutex g_mu;
char *g_addr[kMaxDevices] = {};

// The scratch's device address on the current device (looked up once per device).
char *scratch_on(int dev) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_addr[dev]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
        if (e != cudaSuccess || !p)
            throw std::runtime_error(std::string("flash_attn_static: cudaGetSymbolAddress of the static scratch failed: ") +
                                     cudaGetErrorString(e));
        g_addr[dev] = (char *)p;
    }
    return g_addr[dev];
}

std::string mib(size_t b) {
    char buf[32];
    std::snprintf(buf, sizeof buf, "%.2f MiB", (double)b / (1 << 20));
    return buf;
}

}  // namespace

extern "C" GGML_COMPILER_API int ggml_compiler_b200_flash_attn_static(const float *q, const void *k, const void *v,
                                                                      const void *mask, float *out, int64_t head_dim,
                                                                      int64_t n_q, int64_t n_head, int64_t n_kv,
                                                                      int64_t n_head_kv, int64_t kv_head_stride,
                                                                      float scale, void *stream) {
    using gcb::TD;
    try {
        if (!q || !k || !v || !out) throw std::runtime_error("flash_attn_static: q, k, v and out must not be NULL");
        if (head_dim <= 0 || head_dim > 256 || head_dim % 32)
            throw std::runtime_error("flash_attn_static: head_dim must be a multiple of 32 up to 256, got " +
                                     std::to_string(head_dim));
        if (n_q < 1 || n_kv < 1 || n_head_kv < 1 || n_head < n_head_kv || n_head % n_head_kv)
            throw std::runtime_error("flash_attn_static: needs n_q, n_kv >= 1 and n_head a multiple of n_head_kv");
        if (kv_head_stride < n_kv) throw std::runtime_error("flash_attn_static: kv_head_stride must be at least n_kv");
        if (((uintptr_t)k | (uintptr_t)v) % 16)
            throw std::runtime_error("flash_attn_static: k and v must be 16-byte aligned");

        TD tq, tk, tv, tm, to;
        tq.data = (char *)q;
        tq.type = gcb::T_F32;
        const int64_t qne[4] = {head_dim, n_q, n_head, 1};
        for (int i = 0; i < 4; i++) tq.ne[i] = qne[i];
        gcb::set_contiguous(tq);
        for (TD *t : {&tk, &tv}) {
            t->data = (char *)(t == &tk ? k : v);
            t->type = gcb::T_F16;
            const int64_t ne[4] = {head_dim, n_kv, n_head_kv, 1};
            for (int i = 0; i < 4; i++) t->ne[i] = ne[i];
            t->nb[0] = 2;
            t->nb[1] = 2 * head_dim;
            t->nb[2] = 2 * head_dim * kv_head_stride;
            t->nb[3] = t->nb[2] * n_head_kv;
        }
        if (mask) {
            tm.data = (char *)mask;
            tm.type = gcb::T_F16;
            const int64_t mne[4] = {n_kv, n_q, 1, 1};
            for (int i = 0; i < 4; i++) tm.ne[i] = mne[i];
            gcb::set_contiguous(tm);
        }
        to.data = (char *)out;
        to.type = gcb::T_F32;
        const int64_t one[4] = {head_dim, n_head, n_q, 1};
        for (int i = 0; i < 4; i++) to.ne[i] = one[i];
        gcb::set_contiguous(to);

        // calls the prefill kernel takes (16+ query rows, head size 64 or 128) merge inside each CTA
        // and use no partials or counters; the limits bind the split kernel's calls only
        const bool in_cta = gcb::k::flash_prefill_ok(tq, tk, tv, to);
        const size_t part = in_cta ? 0 : gcb::k::flash_split_scratch_bytes(tq, tk);
        const size_t ncnt = in_cta ? 0 : gcb::k::flash_split_counters(tq, tk);
        if (part > kPartBytes)
            throw std::runtime_error("flash_attn_static: n_q " + std::to_string(n_q) + ", n_head " + std::to_string(n_head) +
                                     ", n_kv " + std::to_string(n_kv) + " need " + mib(part) +
                                     " of chunk partials; the static scratch holds " + mib(kPartBytes));
        if (ncnt > kMaxCounters)
            throw std::runtime_error("flash_attn_static: " + std::to_string(ncnt) + " arrival counters needed, at most " +
                                     std::to_string(kMaxCounters));

        int dev = 0;
        const cudaError_t ge = cudaGetDevice(&dev);
        if (ge != cudaSuccess) throw std::runtime_error(std::string("flash_attn_static: ") + cudaGetErrorString(ge));
        if (dev < 0 || dev >= kMaxDevices) throw std::runtime_error("flash_attn_static: device index out of range");
        char *base = scratch_on(dev);
        cudaStream_t s = (cudaStream_t)stream;
        const cudaError_t me = cudaMemsetAsync(base + kCounterOff, 0, kScratchBytes - kCounterOff, s);
        if (me != cudaSuccess) throw std::runtime_error(std::string("flash_attn_static: ") + cudaGetErrorString(me));
        gcb::k::flash_attn_split(tq, tk, tv, mask ? &tm : nullptr, to, scale, base, (int *)(base + kCounterOff),
                                 (int *)(base + kErrOff), s);
        return 0;
    } catch (const std::exception &e) {
        gcb_set_last_error(e.what());
    } catch (...) {
        gcb_set_last_error("flash_attn_static: unknown error");
    }
    return -1;
}
