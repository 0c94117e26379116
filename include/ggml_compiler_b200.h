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

#ifdef __cplusplus
}
#endif

#endif /* GGML_COMPILER_B200_H */
