/*
 * ggml_compiler_b200.h - extensions of the B200 backend beyond the reference's C ABI.
 *
 * None of these has a counterpart in the reference (runtime/include/ggml_compiler_rt.h); they
 * expose the device-side timing and per-kernel statistics a benchmark needs. Same error
 * conventions as ggml_compiler_rt.h: 0 / -1 results, ggml_compiler_last_error() on failure.
 */
#ifndef GGML_COMPILER_B200_H
#define GGML_COMPILER_B200_H

#include "ggml_compiler_rt.h"

#ifdef __cplusplus
extern "C" {
#endif

/* The cudaStream_t every kernel of model m is launched on (a caller may record CUDA events on it). */
GGML_COMPILER_API void * ggml_compiler_b200_stream(const ggml_compiler_model * m);

/* Device time (CUDA events on the model's stream) of the last ggml_compiler_run_entry, in ms. */
GGML_COMPILER_API double ggml_compiler_b200_last_device_ms(const ggml_compiler_model * m);

/* on != 0: time every kernel launch with CUDA events (serialises launches; no CUDA graphs) and
   accumulate per-kernel-family statistics; on == 0: back to graph replay. */
GGML_COMPILER_API int ggml_compiler_b200_set_profiling(ggml_compiler_model * m, int on);
GGML_COMPILER_API int ggml_compiler_b200_n_kernel_stats(const ggml_compiler_model * m);
/* Statistics of kernel family i since profiling was turned on: total device ms, launches and the
   algorithmic bytes those launches move (weights, activations, KV cache). */
GGML_COMPILER_API int ggml_compiler_b200_kernel_stats(const ggml_compiler_model * m, int i, const char ** kind,
                                                      double * ms, int * launches, double * bytes);

/* Snapshots of driver values, typically state values such as a KV cache: the whole storage of
   value `name` (sized for the value's largest binding, ggml_compiler_b200_value_bytes) copied to or
   from host memory, after the model's queued work. nbytes must equal that size. Saving and
   restoring a sequence's cache, or handing a cache to another process, uses these. No counterpart
   in the reference, whose state is reachable only through reset (ggml_compiler_rt.h:152-153). */
GGML_COMPILER_API int64_t ggml_compiler_b200_value_bytes(const ggml_compiler_model * m, const char * name);
GGML_COMPILER_API int ggml_compiler_b200_read_value(ggml_compiler_model * m, const char * name, void * dst, size_t nbytes);
GGML_COMPILER_API int ggml_compiler_b200_write_value(ggml_compiler_model * m, const char * name, const void * src,
                                                     size_t nbytes);

/* Tensor parallelism over NVLink peer memory. No counterpart in the reference, which runs on one
   device (ggml_compiler_rt.h:57-62, options.device). Processes 0 .. world-1 (2..8), one GPU each,
   load the same program. Each calls tp_init before its first run; it exports this rank's exchange
   window and writes an opaque handle (the return value is its size, at most cap bytes). The caller
   moves the handles between the processes with its own transport (torch.distributed, MPI, a file)
   and every rank calls tp_connect with all ranks' handles concatenated in rank order. From then on
   the decode GEMVs compute only this rank's rows (the QKV projection and attention its heads) and
   the slices are exchanged through the peers' windows; every result stays identical to one GPU's.
   All ranks must make the same sequence of runs; an exchange whose peer never arrives gives up
   after 60 s (GGML_COMPILER_B200_TP_TIMEOUT_MS) and the run fails. window_bytes: 0 for 64 MiB (two
   slots of half of it each bound the largest exchanged buffer). Returns -1 on failure. */
GGML_COMPILER_API int ggml_compiler_b200_tp_init(ggml_compiler_model * m, int rank, int world, size_t window_bytes,
                                                 void * handle, size_t cap);
GGML_COMPILER_API int ggml_compiler_b200_tp_connect(ggml_compiler_model * m, const void * handles, size_t nbytes);

/* Batched decode: one decode step for up to 16 sequences, each weight matrix streamed once per 8
   sequences instead of once per sequence. No counterpart in the reference, which decodes one
   sequence per model (ggml_compiler/llm.py:64 builds the decode entry for batch 1).
   seq_slots gives model m n (1..16) sequence slots, each a zeroed copy of every state value (the KV
   caches); calling it again drops the earlier slots. seq_copy copies the whole state from slot src
   to slot dst, -1 naming the model's own state, the one the program's entries read and write: run
   a prompt through the `prefill` entry, then copy the state into the sequence's slot.
   decode_batch runs the stage of `entry` (normally "decode": fused decode layers, an output head)
   for sequences 0..n-1 at once: token tokens[i] at position positions[i] of the sequence in slot i,
   whose K/V rows are written there and whose keys 0..positions[i] are attended (the causal mask
   the single-sequence entry takes from its caller). logits: host f32 [n][vocab] or NULL; next:
   host i32 [n], each row's argmax, or NULL. Row i equals, bit for bit, what `entry` gives for that
   sequence alone. Positions must lie inside the KV cache; a stage with nodes outside the fused
   decode layer is refused.
   generate_batch runs `steps` greedy steps from tokens first[i] at positions start[i]: every step
   feeds each sequence's argmax back on the device, with no host round trip in between; out: host
   i32 [steps][n] (NULL: not copied). No stop tokens: every sequence runs all steps.
   ggml_compiler_b200_last_device_ms gives the device time of the last call. */
GGML_COMPILER_API int ggml_compiler_b200_seq_slots(ggml_compiler_model * m, int n);
GGML_COMPILER_API int ggml_compiler_b200_seq_copy(ggml_compiler_model * m, int dst, int src);
GGML_COMPILER_API int ggml_compiler_b200_decode_batch(ggml_compiler_model * m, const char * entry, int n,
                                                      const int32_t * tokens, const int32_t * positions,
                                                      float * logits, int32_t * next);
GGML_COMPILER_API int ggml_compiler_b200_generate_batch(ggml_compiler_model * m, const char * entry, int n,
                                                        const int32_t * first, const int32_t * start, int steps,
                                                        int32_t * out);

/* Split-KV flash attention on caller-owned device buffers that allocates no device memory: the
   kernel the flash_attn node runs (reference: runtime/src/ops.cpp:217-240 -> ggml_flash_attn_ext,
   runtime/include/ggml_compiler_ops.h:133-135), with its scratch in a static device array of the
   library. No counterpart in the reference, which has no entry point for a single op.
   For callers without a loaded program that must not allocate: a custom op inside another engine's
   decode loop, whose caching allocator owns the free device memory and which cudaMalloc / cudaFree
   would stall by synchronising the device.
     q     f32 [n_head][n_q][head_dim]                  (ggml ne {head_dim, n_q, n_head, 1})
     k, v  f16, row j of K/V head h at element (h * kv_head_stride + j) * head_dim; 16-byte aligned
     mask  f16 [n_q][n_kv], added to the scaled scores, the same for every head; NULL for none
     out   f32 [n_q][n_head][head_dim]                  (ggml ne {head_dim, n_head, n_q, 1})
   head_dim a multiple of 32 up to 256, n_head a multiple of n_head_kv, kv_head_stride >= n_kv.
   Limit: a call that the per-chunk kernel runs (fewer than 16 query rows, or a head_dim other than
   64 and 128) needs n_q x n_head x ceil(n_kv / 64) x (head_dim + 2) x 4 bytes <= 4 MiB of chunk
   partials and n_q x n_head_kv <= 4096 arrival counters; larger calls are rejected (-1,
   ggml_compiler_last_error()). Calls of 16+ rows with head_dim 64 or 128 merge inside each CTA and
   need no scratch, so no size limit applies to them.
   A bounded wait in the kernel that expires (2 s) leaves NaN in the output rows it could not
   compute: check the output for NaN to detect it.
   Asynchronous on `stream` (a cudaStream_t; NULL: the legacy default stream) of the current device.
   The arrival counters in the scratch must be zero when the kernel starts: each call zeroes them on
   `stream` first. The first call on a device does the set-up (looks up the scratch's device address);
   make it before any stream capture on that device. One scratch per device: calls whose executions
   overlap race on it and return garbage; order them on one stream or with events. */
GGML_COMPILER_API int ggml_compiler_b200_flash_attn_static(const float * q, const void * k, const void * v,
                                                           const void * mask, float * out, int64_t head_dim,
                                                           int64_t n_q, int64_t n_head, int64_t n_kv,
                                                           int64_t n_head_kv, int64_t kv_head_stride, float scale,
                                                           void * stream);

#ifdef __cplusplus
}
#endif

#endif /* GGML_COMPILER_B200_H */
