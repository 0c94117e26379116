// The C ABI (include/ggml_compiler_rt.h) over the executor. Same conventions as the reference's
// C API (runtime/src/ggml_compiler_rt.cpp:825-1170): every entry point catches exceptions, returns
// -1 / NULL / 0 and leaves a per-thread message for ggml_compiler_last_error().
#include <cuda_runtime.h>

#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "ggml_compiler_rt.h"
#include "ggml_compiler_b200.h"
#include "gc_model.h"

#ifndef GCB_VERSION
#define GCB_VERSION "0.1.0"
#endif

using gcb::Model;

struct ggml_compiler_model {
    Model m;
};

struct ggml_compiler_stage_build {
    int unused;
};

void gcb_set_last_error(const std::string &msg);

namespace {

thread_local std::string g_error;

void set_error(const std::string &msg) { g_error = msg; }

template <typename F>
auto guarded(F &&f, decltype(f()) on_error) -> decltype(f()) {
    try {
        return f();
    } catch (const std::exception &e) {
        set_error(e.what());
    } catch (...) {
        set_error("unknown error");
    }
    return on_error;
}

int fill_info(const ggml_compiler_model *mm, const gcb::TensorSpec &v, const std::vector<int64_t> &b,
              ggml_compiler_tensor_info *info) {
    if (!info) {
        set_error("info is NULL");
        return -1;
    }
    const auto shape = v.shape_at(b);
    switch (v.type) {
        case gcb::T_F32: info->dtype = GGML_COMPILER_DTYPE_F32; break;
        case gcb::T_F16: info->dtype = GGML_COMPILER_DTYPE_F16; break;
        case gcb::T_I32: info->dtype = GGML_COMPILER_DTYPE_I32; break;
        default: set_error("value '" + v.name + "' has a type the C API cannot describe"); return -1;
    }
    if (shape.size() > GGML_COMPILER_MAX_RANK) {
        set_error("value '" + v.name + "' has rank above GGML_COMPILER_MAX_RANK");
        return -1;
    }
    info->name = v.name.c_str();
    info->ndim = (int)shape.size();
    for (size_t i = 0; i < shape.size(); i++) info->shape[i] = shape[i];
    info->nbytes = mm->m.nbytes_of(v, b);
    return 0;
}

// Binds the symbols an input's shape fixes. Each dim that reads exactly one symbol not yet fixed
// pins it: dims are nondecreasing in their symbol, so the smallest value in the symbol's range
// whose dim reaches the given size is found by bisection and must hit it exactly. Two passes let a
// symbol fixed by one dim settle another dim's expression; the whole shape is then re-checked.
void solve_shape(Model &m, const gcb::TensorSpec &v, const std::vector<int64_t> &shape) {
    if (shape.size() != v.shape_expr.size())
        throw std::runtime_error("input '" + v.name + "' has rank " + std::to_string(v.shape_expr.size()) + ", got " +
                                 std::to_string(shape.size()));
    std::vector<int64_t> b = m.binding;
    uint64_t fixed = 0;
    for (int pass = 0; pass < 2; pass++)
        for (size_t i = 0; i < shape.size(); i++) {
            const gcb::DimExpr &dim = v.shape_expr[i];
            const uint64_t open = dim.reads() & ~fixed;
            if (!open || (open & (open - 1))) continue;  // no unknown symbol, or more than one
            const int k = __builtin_ctzll(open);
            const gcb::Symbol &sy = m.prog.symbols[(size_t)k];
            int64_t lo = sy.min, hi = sy.max;
            while (lo < hi) {
                b[(size_t)k] = lo + (hi - lo) / 2;
                if (dim.eval(b) < shape[i]) lo = b[(size_t)k] + 1;
                else hi = b[(size_t)k];
            }
            b[(size_t)k] = lo;
            if (dim.eval(b) != shape[i])
                throw std::runtime_error("input '" + v.name + "': no " + sy.name + " in [" + std::to_string(sy.min) + ", " +
                                         std::to_string(sy.max) + "] gives dim " + std::to_string(i) + " = " +
                                         std::to_string(shape[i]));
            fixed |= 1ull << k;
        }
    const auto got = v.shape_at(b);
    if (got != shape) {
        std::string want, have;
        for (auto d : shape) want += (want.empty() ? "" : ", ") + std::to_string(d);
        for (auto d : got) have += (have.empty() ? "" : ", ") + std::to_string(d);
        throw std::runtime_error("input '" + v.name + "' cannot have shape [" + want +
                                 "] (with the other symbols as bound, it is [" + have + "])");
    }
    m.binding = b;
}

bool has_b200() {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    for (int i = 0; i < n; i++) {
        cudaDeviceProp p{};
        if (cudaGetDeviceProperties(&p, i) == cudaSuccess && p.major == 10) return true;
    }
    return false;
}

}  // namespace

// The per-thread error message, for C entry points defined in other files (kernels/gc_flash_static.cu).
void gcb_set_last_error(const std::string &msg) { set_error(msg); }

extern "C" {

const char *ggml_compiler_version(void) { return "ggml_compiler_rt " GCB_VERSION " (B200 sm_100a backend)"; }

const char *ggml_compiler_last_error(void) { return g_error.c_str(); }

ggml_compiler_options ggml_compiler_default_options(void) {
    ggml_compiler_options o{};
    o.backend = GGML_COMPILER_BACKEND_AUTO;
    o.device = 0;
    o.n_threads = 0;
    o.allow_cpu_fallback = false;
    return o;
}

bool ggml_compiler_has_backend(ggml_compiler_backend backend) {
    if (backend == GGML_COMPILER_BACKEND_CPU) return false;
    return has_b200();
}

size_t ggml_compiler_row_size(const char *type, int64_t n) {
    try {
        if (!type) throw std::runtime_error("type is NULL");
        const gcb::TypeTraits *t = gcb::type_by_name(type);
        if (!t) throw std::runtime_error(std::string("unknown tensor type '") + type + "'");
        return gcb::row_size(t->type, n);
    } catch (const std::exception &e) {
        set_error(e.what());
        return 0;
    }
}

size_t ggml_compiler_quantize(const char *type, const float *src, int64_t nrows, int64_t n_per_row, void *dst,
                              size_t dst_size) {
    try {
        if (!type || !src || !dst) throw std::runtime_error("NULL argument");
        const gcb::TypeTraits *t = gcb::type_by_name(type);
        if (!t) throw std::runtime_error(std::string("unknown tensor type '") + type + "'");
        if (t->type != gcb::T_Q4_0 && t->type != gcb::T_Q8_0 && t->type != gcb::T_Q4_1 && t->type != gcb::T_Q5_0 &&
            t->type != gcb::T_Q5_1 && t->type != gcb::T_F32 && t->type != gcb::T_F16 && t->type != gcb::T_BF16)
            throw std::runtime_error(std::string("this backend encodes q4_0, q4_1, q5_0, q5_1, q8_0, f16, bf16 and f32; not '") +
                                     type + "' (it computes with iq4_nl and the K-quants stored by another encoder)");
        if (n_per_row <= 0 || nrows < 0) throw std::runtime_error("bad row count or length");
        if (n_per_row % t->block)
            throw std::runtime_error("row length " + std::to_string(n_per_row) + " is not a multiple of " + type +
                                     "'s block size " + std::to_string(t->block));
        if (dst_size < gcb::row_size(t->type, n_per_row) * (size_t)nrows) throw std::runtime_error("destination buffer too small");
        return gcb::quantize_rows(t->type, src, nrows, n_per_row, (uint8_t *)dst);
    } catch (const std::exception &e) {
        set_error(e.what());
        return 0;
    }
}

ggml_compiler_model *ggml_compiler_load(const char *path, const ggml_compiler_options *opt) {
    return ggml_compiler_load_with(path, opt, nullptr, 0);
}

ggml_compiler_model *ggml_compiler_load_with(const char *path, const ggml_compiler_options *opt,
                                             const ggml_compiler_builder *builders, int n_builders) {
    const ggml_compiler_options o = opt ? *opt : ggml_compiler_default_options();
    return guarded(
        [&]() -> ggml_compiler_model * {
            if (!path) throw std::runtime_error("path is NULL");
            if (n_builders > 0 || builders)
                throw std::runtime_error("compiled stage builders (ggml-compiler compile --emit cpp) build ggml graphs; "
                                         "this backend has no ggml and cannot run them");
            auto mm = std::make_unique<ggml_compiler_model>();
            mm->m.load(path, (int)o.backend, o.device, o.allow_cpu_fallback);
            return mm.release();
        },
        nullptr);
}

struct ggml_context *ggml_compiler_build_ctx(ggml_compiler_stage_build *) { return nullptr; }
bool ggml_compiler_build_gpu(ggml_compiler_stage_build *) { return true; }
bool ggml_compiler_build_supports(ggml_compiler_stage_build *, const struct ggml_tensor *) { return false; }
struct ggml_tensor *ggml_compiler_build_param(ggml_compiler_stage_build *, int) {
    set_error("stage builders are not supported by this backend");
    return nullptr;
}
struct ggml_tensor *ggml_compiler_build_weight(ggml_compiler_stage_build *, const char *) {
    set_error("stage builders are not supported by this backend");
    return nullptr;
}
int64_t ggml_compiler_build_symbol(ggml_compiler_stage_build *, int) { return 1; }
void ggml_compiler_build_output(ggml_compiler_stage_build *, int, struct ggml_tensor *) {}

const char *ggml_compiler_metadata(const ggml_compiler_model *mm, const char *key) {
    if (!mm || !key) return nullptr;
    const std::string *s = mm->m.gguf.get_string(key);
    return s ? s->c_str() : nullptr;
}

void ggml_compiler_free(ggml_compiler_model *mm) { delete mm; }

const char *ggml_compiler_backend_name(const ggml_compiler_model *mm) { return mm ? mm->m.backend_name.c_str() : nullptr; }

int ggml_compiler_n_entries(const ggml_compiler_model *mm) { return mm ? (int)mm->m.entries.size() : -1; }

const char *ggml_compiler_entry_name(const ggml_compiler_model *mm, int e) {
    if (!mm || e < 0 || e >= (int)mm->m.entries.size()) {
        set_error("entry index out of range");
        return nullptr;
    }
    return mm->m.entries[(size_t)e].spec->name.c_str();
}

int ggml_compiler_entry_n_inputs(const ggml_compiler_model *mm, int e) {
    return mm && e >= 0 && e < (int)mm->m.entries.size() ? (int)mm->m.entries[(size_t)e].inputs.size() : -1;
}

int ggml_compiler_entry_n_outputs(const ggml_compiler_model *mm, int e) {
    return mm && e >= 0 && e < (int)mm->m.entries.size() ? (int)mm->m.entries[(size_t)e].outputs.size() : -1;
}

int ggml_compiler_entry_input_info(const ggml_compiler_model *mm, int e, int i, ggml_compiler_tensor_info *info) {
    if (!mm || e < 0 || e >= (int)mm->m.entries.size() || i < 0 || i >= (int)mm->m.entries[(size_t)e].inputs.size()) {
        set_error("input index out of range");
        return -1;
    }
    return fill_info(mm, *mm->m.entries[(size_t)e].inputs[(size_t)i], mm->m.binding, info);
}

int ggml_compiler_entry_output_info(const ggml_compiler_model *mm, int e, int i, ggml_compiler_tensor_info *info) {
    if (!mm || e < 0 || e >= (int)mm->m.entries.size() || i < 0 || i >= (int)mm->m.entries[(size_t)e].outputs.size()) {
        set_error("output index out of range");
        return -1;
    }
    return fill_info(mm, *mm->m.entries[(size_t)e].outputs[(size_t)i], mm->m.binding, info);
}

int ggml_compiler_n_inputs(const ggml_compiler_model *mm) { return ggml_compiler_entry_n_inputs(mm, 0); }
int ggml_compiler_n_outputs(const ggml_compiler_model *mm) { return ggml_compiler_entry_n_outputs(mm, 0); }
int ggml_compiler_input_info(const ggml_compiler_model *mm, int i, ggml_compiler_tensor_info *info) {
    return ggml_compiler_entry_input_info(mm, 0, i, info);
}
int ggml_compiler_output_info(const ggml_compiler_model *mm, int i, ggml_compiler_tensor_info *info) {
    return ggml_compiler_entry_output_info(mm, 0, i, info);
}

int ggml_compiler_run_entry(ggml_compiler_model *mm, const char *entry) {
    return guarded(
        [&]() {
            if (!mm || !entry) throw std::runtime_error("NULL argument");
            mm->m.run_entry(entry);
            return 0;
        },
        -1);
}

int ggml_compiler_run(ggml_compiler_model *mm) {
    if (!mm) {
        set_error("model is NULL");
        return -1;
    }
    return ggml_compiler_run_entry(mm, mm->m.entries[0].spec->name.c_str());
}

int ggml_compiler_reset(ggml_compiler_model *mm) {
    return guarded(
        [&]() {
            if (!mm) throw std::runtime_error("model is NULL");
            mm->m.reset_state();
            return 0;
        },
        -1);
}

int ggml_compiler_n_symbols(const ggml_compiler_model *mm) { return mm ? (int)mm->m.prog.symbols.size() : -1; }

int ggml_compiler_symbol_info(const ggml_compiler_model *mm, int i, const char **name, int64_t *min, int64_t *max,
                              int64_t *value) {
    if (!mm || i < 0 || i >= (int)mm->m.prog.symbols.size()) {
        set_error("symbol index out of range");
        return -1;
    }
    const gcb::Symbol &sy = mm->m.prog.symbols[(size_t)i];
    if (name) *name = sy.name.c_str();
    if (min) *min = sy.min;
    if (max) *max = sy.max;
    if (value) *value = mm->m.binding[(size_t)i];
    return 0;
}

int ggml_compiler_set_symbol(ggml_compiler_model *mm, const char *name, int64_t value) {
    return guarded(
        [&]() {
            if (!mm || !name) throw std::runtime_error("NULL argument");
            const int i = mm->m.prog.symbol_index(name);
            if (i < 0) throw std::runtime_error("no symbol named '" + std::string(name) + "'");
            const gcb::Symbol &sy = mm->m.prog.symbols[(size_t)i];
            if (value < sy.min || value > sy.max)
                throw std::runtime_error("symbol '" + sy.name + "' = " + std::to_string(value) + " is outside [" +
                                         std::to_string(sy.min) + ", " + std::to_string(sy.max) + "]");
            mm->m.binding[(size_t)i] = value;
            return 0;
        },
        -1);
}

int ggml_compiler_set_input_shape(ggml_compiler_model *mm, const char *name, int ndim, const int64_t *shape) {
    return guarded(
        [&]() {
            if (!mm || !name || (ndim > 0 && !shape)) throw std::runtime_error("NULL argument");
            if (!mm->m.input_set.count(name)) throw std::runtime_error("no input named '" + std::string(name) + "'");
            solve_shape(mm->m, *mm->m.values.at(name).spec, std::vector<int64_t>(shape, shape + ndim));
            return 0;
        },
        -1);
}

int ggml_compiler_set_input(ggml_compiler_model *mm, const char *name, const void *data, size_t nbytes) {
    return guarded(
        [&]() {
            if (!mm || !name || !data) throw std::runtime_error("NULL argument");
            if (!mm->m.input_set.count(name)) throw std::runtime_error("no input named '" + std::string(name) + "'");
            const auto &v = mm->m.values.at(name);
            const size_t want = mm->m.nbytes_of(*v.spec, mm->m.binding);
            if (nbytes != want)
                throw std::runtime_error("input '" + std::string(name) + "' needs " + std::to_string(want) + " bytes, got " +
                                         std::to_string(nbytes));
            gcb::cuda_check(cudaSetDevice(mm->m.device), "cudaSetDevice");
            gcb::cuda_check(cudaMemcpyAsync(v.buf.get(), data, nbytes, cudaMemcpyHostToDevice, mm->m.stream), "set_input");
            gcb::cuda_check(cudaStreamSynchronize(mm->m.stream), "set_input");
            mm->m.input_set[name] = true;
            return 0;
        },
        -1);
}

int ggml_compiler_get_output(ggml_compiler_model *mm, const char *name, void *dst, size_t nbytes) {
    return guarded(
        [&]() {
            if (!mm || !name || !dst) throw std::runtime_error("NULL argument");
            for (const auto &e : mm->m.entries) {
                for (const gcb::TensorSpec *v : e.outputs) {
                    if (v->name != name) continue;
                    const size_t have = mm->m.nbytes_of(*v, mm->m.binding);
                    if (nbytes != have)
                        throw std::runtime_error("output '" + std::string(name) + "' has " + std::to_string(have) +
                                                 " bytes, buffer has " + std::to_string(nbytes));
                    gcb::cuda_check(cudaSetDevice(mm->m.device), "cudaSetDevice");
                    gcb::cuda_check(cudaMemcpyAsync(dst, mm->m.values.at(name).buf.get(), nbytes, cudaMemcpyDeviceToHost,
                                                    mm->m.stream),
                                    "get_output");
                    gcb::cuda_check(cudaStreamSynchronize(mm->m.stream), "get_output");
                    return 0;
                }
            }
            throw std::runtime_error("no output named '" + std::string(name) + "'");
        },
        -1);
}

int ggml_compiler_last_stats(const ggml_compiler_model *mm, ggml_compiler_stats *st) {
    if (!mm || !st) {
        set_error("NULL argument");
        return -1;
    }
    st->ms_total = mm->m.last_ms;
    st->n_calls = mm->m.last_calls;
    return 0;
}

int ggml_compiler_n_stages(const ggml_compiler_model *mm) { return mm ? (int)mm->m.prog.stages.size() : -1; }

int ggml_compiler_stage_stats(const ggml_compiler_model *mm, int i, const char **name, double *ms, int *n_calls) {
    if (!mm || i < 0 || i >= (int)mm->m.prog.stages.size()) {
        set_error("stage index out of range");
        return -1;
    }
    if (name) *name = mm->m.prog.stages[(size_t)i].name.c_str();
    if (ms) *ms = mm->m.stage_stats[(size_t)i].ms;
    if (n_calls) *n_calls = mm->m.stage_stats[(size_t)i].calls;
    return 0;
}

// --- extensions (include/ggml_compiler_b200.h) ---------------------------------------------------

void *ggml_compiler_b200_stream(const ggml_compiler_model *mm) { return mm ? (void *)mm->m.stream : nullptr; }

double ggml_compiler_b200_last_device_ms(const ggml_compiler_model *mm) { return mm ? mm->m.last_device_ms : -1.0; }

int ggml_compiler_b200_set_profiling(ggml_compiler_model *mm, int on) {
    if (!mm) {
        set_error("model is NULL");
        return -1;
    }
    mm->m.profiling = on != 0;
    if (on) mm->m.kstats.clear();
    return 0;
}

int ggml_compiler_b200_tp_init(ggml_compiler_model *mm, int rank, int world, size_t window_bytes, void *handle, size_t cap) {
    if (!mm || !handle) {
        set_error("model and handle must not be NULL");
        return -1;
    }
    if (cap < sizeof(cudaIpcMemHandle_t)) {
        set_error("tp_init: the handle needs " + std::to_string(sizeof(cudaIpcMemHandle_t)) + " bytes");
        return -1;
    }
    try {
        cudaIpcMemHandle_t h;
        mm->m.tp_init(rank, world, window_bytes, &h);
        std::memcpy(handle, &h, sizeof h);
        return (int)sizeof h;
    } catch (const std::exception &e) {
        set_error(e.what());
        return -1;
    }
}

int ggml_compiler_b200_tp_connect(ggml_compiler_model *mm, const void *handles, size_t nbytes) {
    if (!mm || !handles) {
        set_error("model and handles must not be NULL");
        return -1;
    }
    if (nbytes != (size_t)mm->m.tp.world * sizeof(cudaIpcMemHandle_t)) {
        set_error("tp_connect: expected " + std::to_string(mm->m.tp.world) + " handles of " +
                  std::to_string(sizeof(cudaIpcMemHandle_t)) + " bytes");
        return -1;
    }
    try {
        std::vector<cudaIpcMemHandle_t> hs((size_t)mm->m.tp.world);
        std::memcpy(hs.data(), handles, nbytes);
        mm->m.tp_connect(hs.data());
        return 0;
    } catch (const std::exception &e) {
        set_error(e.what());
        return -1;
    }
}

int64_t ggml_compiler_b200_value_bytes(const ggml_compiler_model *mm, const char *name) {
    return guarded(
        [&]() -> int64_t {
            if (!mm || !name) throw std::runtime_error("NULL argument");
            auto it = mm->m.values.find(name);
            if (it == mm->m.values.end()) throw std::runtime_error("no value named '" + std::string(name) + "'");
            return (int64_t)it->second.buf.size();
        },
        (int64_t)-1);
}

static int copy_value(ggml_compiler_model *mm, const char *name, void *host, size_t nbytes, bool to_host) {
    return guarded(
        [&]() {
            if (!mm || !name || !host) throw std::runtime_error("NULL argument");
            auto it = mm->m.values.find(name);
            if (it == mm->m.values.end()) throw std::runtime_error("no value named '" + std::string(name) + "'");
            gcb::DevBuf &b = it->second.buf;
            if (nbytes != b.size())
                throw std::runtime_error("value '" + std::string(name) + "' holds " + std::to_string(b.size()) +
                                         " bytes, buffer has " + std::to_string(nbytes));
            gcb::cuda_check(cudaSetDevice(mm->m.device), "cudaSetDevice");
            gcb::cuda_check(cudaMemcpyAsync(to_host ? host : b.get(), to_host ? (const void *)b.get() : host, nbytes,
                                            to_host ? cudaMemcpyDeviceToHost : cudaMemcpyHostToDevice, mm->m.stream),
                            "value copy");
            gcb::cuda_check(cudaStreamSynchronize(mm->m.stream), "value copy");
            return 0;
        },
        -1);
}

int ggml_compiler_b200_read_value(ggml_compiler_model *mm, const char *name, void *dst, size_t nbytes) {
    return copy_value(mm, name, dst, nbytes, true);
}

int ggml_compiler_b200_write_value(ggml_compiler_model *mm, const char *name, const void *src, size_t nbytes) {
    return copy_value(mm, name, const_cast<void *>(src), nbytes, false);
}

int ggml_compiler_b200_seq_slots(ggml_compiler_model *mm, int n) {
    return guarded(
        [&]() {
            if (!mm) throw std::runtime_error("NULL model");
            mm->m.seq_slots(n);
            return 0;
        },
        -1);
}

int ggml_compiler_b200_seq_copy(ggml_compiler_model *mm, int dst, int src) {
    return guarded(
        [&]() {
            if (!mm) throw std::runtime_error("NULL model");
            mm->m.seq_copy(dst, src);
            return 0;
        },
        -1);
}

int ggml_compiler_b200_decode_batch(ggml_compiler_model *mm, const char *entry, int n, const int32_t *tokens,
                                    const int32_t *positions, float *logits, int32_t *next) {
    return guarded(
        [&]() {
            if (!mm || !entry) throw std::runtime_error("NULL argument");
            mm->m.decode_batch(entry, n, tokens, positions, logits, next);
            return 0;
        },
        -1);
}

int ggml_compiler_b200_generate_batch(ggml_compiler_model *mm, const char *entry, int n, const int32_t *first,
                                      const int32_t *start, int steps, int32_t *out) {
    return guarded(
        [&]() {
            if (!mm || !entry) throw std::runtime_error("NULL argument");
            mm->m.generate_batch(entry, n, first, start, steps, out);
            return 0;
        },
        -1);
}

int ggml_compiler_b200_n_kernel_stats(const ggml_compiler_model *mm) { return mm ? (int)mm->m.kstats.size() : -1; }

int ggml_compiler_b200_kernel_stats(const ggml_compiler_model *mm, int i, const char **kind, double *ms, int *launches,
                                    double *bytes) {
    if (!mm || i < 0 || i >= (int)mm->m.kstats.size()) {
        set_error("kernel stats index out of range");
        return -1;
    }
    auto it = mm->m.kstats.begin();
    std::advance(it, i);
    if (kind) *kind = it->first.c_str();
    if (ms) *ms = it->second.ms;
    if (launches) *launches = it->second.launches;
    if (bytes) *bytes = it->second.bytes;
    return 0;
}

}  // extern "C"
