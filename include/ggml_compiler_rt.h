/*
 * ggml_compiler_rt.h - the C ABI of the B200 (sm_100a) backend for ggml-compiler programs.
 *
 * This header declares the same functions, enums and structs, with the same layouts, as the
 * reference runtime's runtime/include/ggml_compiler_rt.h (khanhnd61-vr/ggml-compiler). A program
 * compiled by `ggml-compiler compile` (a GGUF holding weights plus the `ggml_compiler.program`
 * JSON) loads and runs through this library unchanged. The reference's Python bindings
 * (ggml_compiler/runtime/session.py:75-122) bind these symbols through $GGML_COMPILER_RT.
 *
 * Conventions (reference runtime/include/ggml_compiler_rt.h:9-18):
 * - an int result is 0 on success and -1 on failure; a pointer result is NULL on failure;
 *   ggml_compiler_last_error() then describes the failure (per thread);
 * - shapes are reported in PyTorch order (outermost dimension first);
 * - a program may have symbols (sequence length, KV length) that size some tensors at run time;
 *   every symbol starts at its maximum, and infos and byte sizes follow the current binding.
 *
 * This backend runs on NVIDIA B200 GPUs only. Every stage runs as hand-written CUDA kernels; there
 * is no CPU backend and no CPU fallback. Loading with GGML_COMPILER_BACKEND_CPU fails with an
 * error, and ggml_compiler_has_backend(CPU) is false. Quantized weights may be Q4_0, Q8_0, q4_1,
 * q5_0, q5_1, iq4_nl, q4_K, q5_K or q6_K (the decode layers fuse for Q4_0, Q8_0, q5_0 and iq4_nl).
 */
#ifndef GGML_COMPILER_RT_H
#define GGML_COMPILER_RT_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#if defined(_WIN32)
#    ifdef GGML_COMPILER_RT_BUILD
#        define GGML_COMPILER_API __declspec(dllexport)
#    else
#        define GGML_COMPILER_API __declspec(dllimport)
#    endif
#else
#    define GGML_COMPILER_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define GGML_COMPILER_MAX_RANK 8

/* Opaque model handle (reference ggml_compiler_rt.h:43). */
typedef struct ggml_compiler_model ggml_compiler_model;

/* Backend selector (reference ggml_compiler_rt.h:45-49). AUTO picks the first GPU. */
typedef enum {
    GGML_COMPILER_BACKEND_CPU  = 0,
    GGML_COMPILER_BACKEND_CUDA = 1,
    GGML_COMPILER_BACKEND_AUTO = 2,
} ggml_compiler_backend;

/* Element types the C API reports for program inputs and outputs (reference :51-55). */
typedef enum {
    GGML_COMPILER_DTYPE_F32 = 0,
    GGML_COMPILER_DTYPE_F16 = 1,
    GGML_COMPILER_DTYPE_I32 = 2,
} ggml_compiler_dtype;

/* Load options (reference :57-62). n_threads is accepted and ignored (no CPU work to thread);
   allow_cpu_fallback must be false: this backend never falls back to the CPU. */
typedef struct {
    ggml_compiler_backend backend;
    int                   device;
    int                   n_threads;
    bool                  allow_cpu_fallback;
} ggml_compiler_options;

/* One program input or output, for the current symbol binding (reference :64-70). */
typedef struct {
    const char *        name;  /* valid while the model lives */
    ggml_compiler_dtype dtype;
    int                 ndim;
    int64_t             shape[GGML_COMPILER_MAX_RANK];
    size_t              nbytes;
} ggml_compiler_tensor_info;

/* Timing of the last run (reference :72-75). ms_total is host wall time of the whole run, which
   ends with the device idle; n_calls counts stage calls. */
typedef struct {
    double ms_total;
    int    n_calls;
} ggml_compiler_stats;

/* reference ggml_compiler_rt.h:77 */
GGML_COMPILER_API const char *          ggml_compiler_version(void);
/* reference :78 - message of the last failure on the calling thread ("" if none). */
GGML_COMPILER_API const char *          ggml_compiler_last_error(void);
/* reference :79 - backend AUTO, device 0, n_threads 0, no CPU fallback. */
GGML_COMPILER_API ggml_compiler_options ggml_compiler_default_options(void);
/* reference :81 - true for CUDA and AUTO when a GPU this build runs on is present. */
GGML_COMPILER_API bool                  ggml_compiler_has_backend(ggml_compiler_backend backend);

/* reference :86-87 - encode nrows rows of n_per_row f32 values in a ggml block type, byte for
   byte as ggml's reference encoder stores them. Types: "q8_0", "q4_0", "q4_1", "q5_0", "q5_1"
   (also "f32", "f16", "bf16"); iq4_nl and the K-quants are computed with but not encoded here.
   Returns the bytes written, or 0 on error (unknown or unencodable type, n_per_row not a multiple
   of the block size, dst_size too small). Host code; needs no GPU. */
GGML_COMPILER_API size_t ggml_compiler_quantize(const char * type, const float * src, int64_t nrows,
                                                int64_t n_per_row, void * dst, size_t dst_size);
/* reference :89 - bytes of one row of n elements of that type; 0 if the type is unknown. */
GGML_COMPILER_API size_t ggml_compiler_row_size(const char * type, int64_t n);

/* reference :91 - read the GGUF, parse its program, upload weights, allocate values and KV
   state (zeroed), and plan every call site's kernels. */
GGML_COMPILER_API ggml_compiler_model * ggml_compiler_load(const char * path, const ggml_compiler_options * opt);
/* reference :94 - a string value of the GGUF's metadata, or NULL. */
GGML_COMPILER_API const char * ggml_compiler_metadata(const ggml_compiler_model * m, const char * key);
/* reference :95 */
GGML_COMPILER_API void         ggml_compiler_free(ggml_compiler_model * m);
/* reference :96 - "CUDA0"-style name of the device the model runs on. */
GGML_COMPILER_API const char * ggml_compiler_backend_name(const ggml_compiler_model * m);

/* Entry points (reference :98-113). The first entry is the default one. */
GGML_COMPILER_API int          ggml_compiler_n_entries(const ggml_compiler_model * m);
GGML_COMPILER_API const char * ggml_compiler_entry_name(const ggml_compiler_model * m, int e);
GGML_COMPILER_API int          ggml_compiler_entry_n_inputs(const ggml_compiler_model * m, int e);
GGML_COMPILER_API int          ggml_compiler_entry_n_outputs(const ggml_compiler_model * m, int e);
GGML_COMPILER_API int          ggml_compiler_entry_input_info(const ggml_compiler_model * m, int e, int i,
                                                              ggml_compiler_tensor_info * info);
GGML_COMPILER_API int          ggml_compiler_entry_output_info(const ggml_compiler_model * m, int e, int i,
                                                               ggml_compiler_tensor_info * info);
/* reference :111 - run one entry point by name; its inputs must have been set. */
GGML_COMPILER_API int          ggml_compiler_run_entry(ggml_compiler_model * m, const char * entry);
/* reference :113 - zero the program's state (the KV cache). */
GGML_COMPILER_API int          ggml_compiler_reset(ggml_compiler_model * m);

/* The default entry's inputs and outputs (reference :115-118). */
GGML_COMPILER_API int ggml_compiler_n_inputs(const ggml_compiler_model * m);
GGML_COMPILER_API int ggml_compiler_n_outputs(const ggml_compiler_model * m);
GGML_COMPILER_API int ggml_compiler_input_info(const ggml_compiler_model * m, int i, ggml_compiler_tensor_info * info);
GGML_COMPILER_API int ggml_compiler_output_info(const ggml_compiler_model * m, int i, ggml_compiler_tensor_info * info);

/* Symbols (reference :120-127). */
GGML_COMPILER_API int ggml_compiler_n_symbols(const ggml_compiler_model * m);
GGML_COMPILER_API int ggml_compiler_symbol_info(const ggml_compiler_model * m, int i, const char ** name,
                                                int64_t * min, int64_t * max, int64_t * value);
GGML_COMPILER_API int ggml_compiler_set_symbol(ggml_compiler_model * m, const char * name, int64_t value);
GGML_COMPILER_API int ggml_compiler_set_input_shape(ggml_compiler_model * m, const char * name, int ndim,
                                                    const int64_t * shape);

/* reference :130-133 - host buffers; nbytes must equal the size for the current binding. */
GGML_COMPILER_API int ggml_compiler_set_input(ggml_compiler_model * m, const char * name, const void * data,
                                              size_t nbytes);
GGML_COMPILER_API int ggml_compiler_run(ggml_compiler_model * m);
GGML_COMPILER_API int ggml_compiler_get_output(ggml_compiler_model * m, const char * name, void * dst, size_t nbytes);

/* reference :135-139 - timings of the last run. Stage times come from CUDA events. */
GGML_COMPILER_API int ggml_compiler_last_stats(const ggml_compiler_model * m, ggml_compiler_stats * st);
GGML_COMPILER_API int ggml_compiler_n_stages(const ggml_compiler_model * m);
GGML_COMPILER_API int ggml_compiler_stage_stats(const ggml_compiler_model * m, int i, const char ** name, double * ms,
                                                int * n_calls);

/* --- Compiled stage builders (reference :141-172) ---------------------------------------------
 * The reference lets C++ generated by `ggml-compiler compile --emit cpp` build a stage's ggml graph
 * itself. This backend has no ggml graphs, so it cannot take a builder: the hooks below exist so
 * such a binary links, and ggml_compiler_load_with fails with a clear error when given builders.
 * With n_builders == 0 it is ggml_compiler_load. */
struct ggml_context;
struct ggml_tensor;
typedef struct ggml_compiler_stage_build ggml_compiler_stage_build;
typedef int (*ggml_compiler_build_fn)(ggml_compiler_stage_build * b);

typedef struct {
    const char *           stage;
    ggml_compiler_build_fn build;
} ggml_compiler_builder;

GGML_COMPILER_API struct ggml_context * ggml_compiler_build_ctx(ggml_compiler_stage_build * b);
GGML_COMPILER_API bool                  ggml_compiler_build_gpu(ggml_compiler_stage_build * b);
GGML_COMPILER_API bool                  ggml_compiler_build_supports(ggml_compiler_stage_build * b,
                                                                     const struct ggml_tensor * t);
GGML_COMPILER_API struct ggml_tensor *  ggml_compiler_build_param(ggml_compiler_stage_build * b, int i);
GGML_COMPILER_API struct ggml_tensor *  ggml_compiler_build_weight(ggml_compiler_stage_build * b,
                                                                   const char * gguf_name);
GGML_COMPILER_API int64_t               ggml_compiler_build_symbol(ggml_compiler_stage_build * b, int i);
GGML_COMPILER_API void                  ggml_compiler_build_output(ggml_compiler_stage_build * b, int i,
                                                                   struct ggml_tensor * t);
GGML_COMPILER_API ggml_compiler_model * ggml_compiler_load_with(const char * path, const ggml_compiler_options * opt,
                                                                const ggml_compiler_builder * builders,
                                                                int n_builders);

#ifdef __cplusplus
}
#endif

#endif /* GGML_COMPILER_RT_H */
