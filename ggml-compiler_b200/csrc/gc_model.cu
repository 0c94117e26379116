#include "gc_model.h"
#include "gc_fused.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <stdexcept>

namespace gcb {

void cuda_check(cudaError_t e, const char *what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

DevBuf &DevBuf::operator=(DevBuf &&o) noexcept {
    if (this != &o) {
        release();
        p_ = o.p_;
        n_ = o.n_;
        o.p_ = nullptr;
        o.n_ = 0;
    }
    return *this;
}

void DevBuf::alloc(size_t n) {
    release();
    if (n == 0) return;
    cuda_check(cudaMalloc(&p_, n), "cudaMalloc");
    n_ = n;
    cuda_check(cudaMemset(p_, 0, n), "cudaMemset");
}

void DevBuf::release() {
    if (p_) cudaFree(p_);
    p_ = nullptr;
    n_ = 0;
}

namespace {

bool symbolic(const TensorSpec &v) {
    for (const auto &d : v.ne_x)
        if (!d.is_const()) return true;
    return false;
}

struct FileCloser {
    void operator()(FILE *f) const { std::fclose(f); }
};

__global__ void set_i32_kernel(int32_t *p, int32_t v) { *p = v; }

}  // namespace

Model::~Model() {
    if (device >= 0) cudaSetDevice(device);
    if (stream) cudaStreamSynchronize(stream);
    for (auto &c : calls)
        if (c.graph) cudaGraphExecDestroy(c.graph);
    for (size_t r = 0; r < tp.win.size(); r++)
        if ((int)r != tp.rank && tp.win[r]) cudaIpcCloseMemHandle(tp.win[r]);
    for (auto &e : event_pool) {
        cudaEventDestroy(e.first);
        cudaEventDestroy(e.second);
    }
    if (d_err) cudaFree(d_err);
    for (auto e : run_ev)
        if (e) cudaEventDestroy(e);
    calls.clear();
    weights.clear();
    values.clear();
    rope_tables.clear();
    counter_bufs.clear();
    if (stream) cudaStreamDestroy(stream);
}

size_t Model::nbytes_of(const TensorSpec &v, const std::vector<int64_t> &b) const {
    const auto ne = eval_ne(v, b);
    return row_size(v.type, ne[0]) * (size_t)(ne[1] * ne[2] * ne[3]);
}

void Model::load(const char *path, int backend, int dev, bool allow_cpu_fallback) {
    if (allow_cpu_fallback)
        throw std::runtime_error("allow_cpu_fallback is not available: this backend runs every node on the GPU");
    if (backend == 0)
        throw std::runtime_error("the CPU backend is not available: this library runs ggml-compiler programs on NVIDIA B200 "
                                 "GPUs only (use GGML_COMPILER_BACKEND_CUDA or AUTO)");
    gguf.open(path);
    const std::string *ptext = gguf.get_string("ggml_compiler.program");
    if (!ptext)
        throw std::runtime_error(std::string("'") + path +
                                 "' has no ggml_compiler.program; it was not written by ggml-compiler compile");
    prog = parse_program(*ptext);
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        throw std::runtime_error("no CUDA device available");
    }
    if (dev < 0 || dev >= n)
        throw std::runtime_error("device index " + std::to_string(dev) + " out of range; " + std::to_string(n) +
                                 " GPU device(s) found");
    device = dev;
    cuda_check(cudaSetDevice(device), "cudaSetDevice");
    cudaDeviceProp prop{};
    cuda_check(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
    if (prop.major != 10)
        throw std::runtime_error("device " + std::to_string(device) + " (" + prop.name + ", sm_" +
                                 std::to_string(prop.major) + std::to_string(prop.minor) +
                                 ") is not a B200: this library is built for sm_100a");
    backend_name = "CUDA" + std::to_string(device);


    cuda_check(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreate");
    cuda_check(cudaMalloc(&d_err, sizeof(int)), "cudaMalloc");
    cuda_check(cudaMemset(d_err, 0, sizeof(int)), "cudaMemset");
    if (const char *p = std::getenv("GGML_COMPILER_PROFILE")) profile_path = p;
    if (const char *p = std::getenv("GGML_COMPILER_B200_TRACE")) trace_path = p;
    if (const char *g = std::getenv("GGML_COMPILER_B200_GRAPHS")) use_graphs = std::atoi(g) != 0;
    if (const char *g = std::getenv("GGML_COMPILER_B200_DECODE_KERNEL")) use_decode_kernel = std::atoi(g) != 0;
    if (const char *g = std::getenv("GCB_L2_PREFETCH_MB")) l2_prefetch_bytes = (int64_t)(std::atof(g) * (1 << 20));
    if (const char *g = std::getenv("GCB_STREAM_EVICT_FIRST")) stream_evict_first = std::atoi(g) != 0;

    load_weights();
    for (const auto &sy : prog.symbols) binding.push_back(sy.max);
    prog.bind(binding);
    alloc_values();
    stage_stats.assign(prog.stages.size(), StageStat{});
    bind_values();
    // rope tables cover every row of the largest state tensor (the KV cache length)
    for (const auto &name : prog.state) {
        const auto &v = values.at(name);
        rope_positions = std::max<int64_t>(rope_positions, v.spec->ne[1]);
    }
    for (auto &e : prog.entries) build_ops(e.driver);
    built = binding;
    cuda_check(cudaStreamSynchronize(stream), "load");
}

void Model::load_weights() {
    std::unique_ptr<FILE, FileCloser> f(std::fopen(gguf.path().c_str(), "rb"));
    if (!f) throw std::runtime_error("cannot open '" + gguf.path() + "'");
    const size_t chunk = 64u << 20;
    char *pinned[2] = {nullptr, nullptr};
    cudaEvent_t done[2];
    for (int i = 0; i < 2; i++) {
        cuda_check(cudaMallocHost(&pinned[i], chunk), "cudaMallocHost");
        cuda_check(cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming), "cudaEventCreate");
    }
    DevBuf raw;  // staging for quantized tensors before repacking
    int slot = 0;
    try {
        for (const auto &t : gguf.tensors()) {
            Weight w;
            w.td.type = t.type;
            for (int i = 0; i < 4; i++) w.td.ne[i] = t.ne[i];
            const bool q = t.type == T_Q4_0 || t.type == T_Q8_0;
            char *dst;
            if (q) {
                if (raw.size() < t.nbytes) raw.alloc(t.nbytes);
                dst = raw.get();
            } else {
                w.data.alloc(t.nbytes);
                dst = w.data.get();
            }
            if (std::fseek(f.get(), (long)(gguf.data_offset() + t.offset), SEEK_SET) != 0)
                throw std::runtime_error("seek failed for tensor " + t.name);
            for (size_t done_b = 0; done_b < t.nbytes;) {
                const size_t nb = std::min(chunk, t.nbytes - done_b);
                cuda_check(cudaEventSynchronize(done[slot]), "cudaEventSynchronize");
                if (std::fread(pinned[slot], 1, nb, f.get()) != nb) throw std::runtime_error("short read for tensor " + t.name);
                cuda_check(cudaMemcpyAsync(dst + done_b, pinned[slot], nb, cudaMemcpyHostToDevice, stream), "cudaMemcpyAsync");
                cuda_check(cudaEventRecord(done[slot], stream), "cudaEventRecord");
                slot ^= 1;
                done_b += nb;
            }
            if (q) {
                const int64_t K = t.ne[0], rows = t.ne[1] * t.ne[2] * t.ne[3];
                w.data.alloc(k::quant_device_bytes(t.type, rows, K));
                k::repack_quant(t.type, (const uint8_t *)raw.get(), rows, K, w.data.get(), stream);
                cuda_check(cudaStreamSynchronize(stream), "repack");
            }
            w.td.data = w.data.get();
            set_contiguous(w.td);
            weights.emplace(t.name, std::move(w));
        }
    } catch (...) {
        cudaStreamSynchronize(stream);
        for (int i = 0; i < 2; i++) {
            cudaFreeHost(pinned[i]);
            cudaEventDestroy(done[i]);
        }
        throw;
    }
    cuda_check(cudaStreamSynchronize(stream), "weight upload");
    for (int i = 0; i < 2; i++) {
        cudaFreeHost(pinned[i]);
        cudaEventDestroy(done[i]);
    }
}

void Model::alloc_values() {
    for (const auto &v : prog.values) {
        int64_t most = 1;
        if (!symbolic(v)) {
            most = v.ne[0] * v.ne[1] * v.ne[2] * v.ne[3];
        } else {  // the largest size over the corners of the symbols it uses
            std::vector<bool> used(prog.symbols.size(), false);
            for (const auto &d : v.ne_x) d.symbols(used);
            std::vector<size_t> idx;
            for (size_t k = 0; k < used.size(); k++)
                if (used[k]) idx.push_back(k);
            std::vector<int64_t> b = binding;
            for (size_t mask = 0; mask < ((size_t)1 << idx.size()); mask++) {
                for (size_t k = 0; k < idx.size(); k++)
                    b[idx[k]] = (mask >> k) & 1 ? prog.symbols[idx[k]].max : prog.symbols[idx[k]].min;
                const auto ne = eval_ne(v, b);
                most = std::max(most, ne[0] * ne[1] * ne[2] * ne[3]);
            }
        }
        const TypeTraits *tr = type_traits(v.type);
        if (!tr || tr->block != 1)
            throw std::runtime_error("value '" + v.name + "' has type " + type_name(v.type) + ", which a driver value cannot have");
        Value val;
        val.spec = &v;
        val.buf.alloc((size_t)most * tr->block_size);
        values.emplace(v.name, std::move(val));
    }
    for (const auto &e : prog.entries) {
        Entry en;
        en.spec = &e;
        for (const auto &name : e.inputs) {
            auto it = values.find(name);
            if (it == values.end()) throw std::runtime_error("input '" + name + "' is not a declared value");
            en.inputs.push_back(it->second.spec);
            input_set[name] = false;
        }
        for (const auto &name : e.outputs) {
            auto it = values.find(name);
            if (it == values.end()) throw std::runtime_error("output '" + name + "' is not a declared value");
            en.outputs.push_back(it->second.spec);
        }
        entries.push_back(std::move(en));
    }
    for (const auto &name : prog.state)
        if (!values.count(name)) throw std::runtime_error("state '" + name + "' is not a declared value");
}

void Model::bind_values() {
    for (auto &kv : values) {
        Value &v = kv.second;
        v.td = TD{};
        v.td.data = v.buf.get();
        v.td.type = v.spec->type;
        for (int i = 0; i < 4; i++) v.td.ne[i] = v.spec->ne[i];
        set_contiguous(v.td);
    }
}

void Model::build_ops(std::vector<DriverOp> &ops) {
    for (auto &d : ops) {
        if (d.kind == DriverOp::Kind::Call) {
            if (d.call_site >= 0) {
                // rebinding: a stage is replanned only if it reads a symbol whose value changed
                CallSite &c = calls[(size_t)d.call_site];
                for (size_t k = 0; k < binding.size() && k < built.size(); k++)
                    if (binding[k] != built[k] && c.stage->uses[k]) c.stale = true;
                continue;
            }
            CallSite c;
            for (size_t i = 0; i < prog.stages.size(); i++) {
                if (prog.stages[i].name == d.stage) {
                    c.stage = &prog.stages[i];
                    c.stage_index = (int)i;
                }
            }
            if (!c.stage) throw std::runtime_error("driver calls unknown stage '" + d.stage + "'");
            d.call_site = (int)calls.size();
            calls.push_back(std::move(c));
            plan_call_site(*this, calls.back(), d);  // plan now: unsupported nodes fail the load
            continue;
        }
        auto val = [&](const std::string &name) -> Value & {
            auto it = values.find(name);
            if (it == values.end()) throw std::runtime_error("loop uses undeclared value '" + name + "'");
            return it->second;
        };
        for (const auto &cp : d.carry) {
            const Value &a = val(cp.first), &b = val(cp.second);
            if (a.spec->type != b.spec->type || a.td.ne[0] != b.td.ne[0] || a.td.ne[1] != b.td.ne[1] ||
                a.td.ne[2] != b.td.ne[2] || a.td.ne[3] != b.td.ne[3])
                throw std::runtime_error("loop carry '" + cp.first + "' does not match its initial value '" + cp.second + "'");
        }
        for (const auto &sc : d.scalars)
            if (val(sc.first).spec->type != T_F32) throw std::runtime_error("loop scalar '" + sc.first + "' must be f32");
        for (const auto &sl : d.slices) {
            const Value &a = val(sl.first), &b = val(sl.second);
            if (a.spec->type != b.spec->type || b.td.nelements() != a.td.nelements() * d.n)
                throw std::runtime_error("loop slice '" + sl.first + "' does not match its source '" + sl.second + "'");
        }
        for (const auto &c : d.counters) {
            if (val(c.first).spec->type != T_I32 || val(c.second).spec->type != T_I32)
                throw std::runtime_error("loop counter '" + c.first + "' must be i32");
        }
        for (const auto &mk : d.masks)
            if (val(mk.first).spec->type != T_F32) throw std::runtime_error("loop mask '" + mk.first + "' must be f32");
        for (const auto &u : d.until)
            if (val(u.first).spec->type != T_I32) throw std::runtime_error("loop stop value '" + u.first + "' must be i32");
        for (const auto &c : d.collect) (void)val(c.first), (void)val(c.second);
        build_ops(d.body);
    }
}

void Model::rebind() {
    if (binding == built) return;
    prog.bind(binding);
    bind_values();
    for (auto &e : prog.entries) build_ops(e.driver);
    built = binding;
}

std::pair<cudaEvent_t, cudaEvent_t> Model::events() {
    if (events_used == event_pool.size()) {
        cudaEvent_t a, b;
        cuda_check(cudaEventCreate(&a), "cudaEventCreate");
        cuda_check(cudaEventCreate(&b), "cudaEventCreate");
        event_pool.emplace_back(a, b);
    }
    return event_pool[events_used++];
}

void Model::collect_times() {
    for (const auto &p : pending) {
        float ms = 0;
        cuda_check(cudaEventElapsedTime(&ms, p.a, p.b), "cudaEventElapsedTime");
        stage_stats[(size_t)p.stage].ms += ms;
    }
    pending.clear();
    events_used = 0;
}

void Model::run_call(const DriverOp &d) {
    CallSite &c = calls[(size_t)d.call_site];
    if (c.stale) plan_call_site(*this, c, d);
    const bool per_step = profiling || !profile_path.empty();
    if (events_used > 4096) {  // long loops: fold finished timings so the event pool stays small
        cuda_check(cudaStreamSynchronize(stream), "stage timing");
        collect_times();
    }
    auto ev = events();
    cuda_check(cudaEventRecord(ev.first, stream), "cudaEventRecord");
    if (per_step) {
        for (const auto &st : c.steps) {
            cudaEvent_t a, b;
            cuda_check(cudaEventCreate(&a), "cudaEventCreate");
            cuda_check(cudaEventCreate(&b), "cudaEventCreate");
            cuda_check(cudaEventRecord(a, stream), "cudaEventRecord");
            st.run(stream);
            cuda_check(cudaEventRecord(b, stream), "cudaEventRecord");
            cuda_check(cudaEventSynchronize(b), "step");
            float ms = 0;
            cudaEventElapsedTime(&ms, a, b);
            cudaEventDestroy(a);
            cudaEventDestroy(b);
            KernelStat &ks = kstats[st.kind];
            ks.ms += ms;
            ks.bytes += st.bytes;
            ks.launches++;
            if (!profile_path.empty())
                profile_lines.push_back(c.stage->name + "\t" + st.node + "\t" + st.kind + "\t" + std::to_string(ms));
        }
    } else if (use_graphs) {
        if (!c.graph_ok) {
            if (c.graph) {
                cudaGraphExecDestroy(c.graph);
                c.graph = nullptr;
            }
            cudaGraph_t g = nullptr;
            cuda_check(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
            try {
                for (const auto &st : c.steps) st.run(stream);
            } catch (...) {
                cudaStreamEndCapture(stream, &g);
                if (g) cudaGraphDestroy(g);
                throw;
            }
            cuda_check(cudaStreamEndCapture(stream, &g), "cudaStreamEndCapture");
            cuda_check(cudaGraphInstantiate(&c.graph, g, 0), "cudaGraphInstantiate");
            cudaGraphDestroy(g);
            c.graph_ok = true;
        }
        cuda_check(cudaGraphLaunch(c.graph, stream), "cudaGraphLaunch");
    } else {
        for (const auto &st : c.steps) st.run(stream);
    }
    cuda_check(cudaEventRecord(ev.second, stream), "cudaEventRecord");
    pending.push_back({c.stage_index, ev.first, ev.second});
    stage_stats[(size_t)c.stage_index].calls++;
    last_calls++;
}

void Model::run_ops(const std::vector<DriverOp> &ops) {
    for (const auto &d : ops) {
        if (d.kind == DriverOp::Kind::Call) {
            run_call(d);
            continue;
        }
        for (const auto &cp : d.carry) {
            const Value &src = values.at(cp.second);
            Value &dst = values.at(cp.first);
            cuda_check(cudaMemcpyAsync(dst.td.data, src.td.data, src.td.nbytes(), cudaMemcpyDeviceToDevice, stream), "carry");
        }
        const int n = d.n_symbol >= 0 ? (int)binding[(size_t)d.n_symbol] : d.n;
        std::vector<int32_t> starts;
        for (const auto &c : d.counters) {
            int32_t v = 0;
            cuda_check(cudaMemcpyAsync(&v, values.at(c.second).td.data, 4, cudaMemcpyDeviceToHost, stream), "counter");
            cuda_check(cudaStreamSynchronize(stream), "counter");
            starts.push_back(v);
        }
        for (const auto &c : d.collect) {
            Value &dst = values.at(c.first);
            cuda_check(cudaMemsetAsync(dst.buf.get(), 0, dst.buf.size(), stream), "collect");
        }
        std::vector<int64_t> ext;
        for (int i = 0; i < n; i++) {
            for (const auto &sc : d.scalars) {
                Value &v = values.at(sc.first);
                k::fill_f32((float *)v.td.data, v.td.nelements(), sc.second[(size_t)i], stream);
            }
            for (const auto &sl : d.slices) {
                Value &dst = values.at(sl.first);
                const Value &src = values.at(sl.second);
                const size_t nb = dst.td.nbytes();
                cuda_check(cudaMemcpyAsync(dst.td.data, src.td.data + (size_t)i * nb, nb, cudaMemcpyDeviceToDevice, stream),
                           "slice");
            }
            for (size_t k = 0; k < d.counters.size(); k++) {
                set_i32_kernel<<<1, 1, 0, stream>>>((int32_t *)values.at(d.counters[k].first).td.data, starts[k] + i);
                cuda_check(cudaGetLastError(), "counter");
            }
            if (!d.bind.empty()) {
                ext = binding;
                for (int32_t v : starts) ext.push_back((int64_t)v + i);
                for (const auto &b : d.bind) {
                    const int64_t v = b.second.eval(ext);
                    const Symbol &sy = prog.symbols[(size_t)b.first];
                    if (v < sy.min || v > sy.max)
                        throw std::runtime_error("loop binds " + sy.name + " = " + std::to_string(v) + ", outside its range");
                    binding[(size_t)b.first] = v;
                }
                rebind();
            }
            for (const auto &mk : d.masks) {
                Value &v = values.at(mk.first);
                const int64_t pos = (int64_t)starts[(size_t)mk.second] + i;
                // the mask is written through a device copy of its counter value: graphs stay valid
                k::causal_mask_row((float *)v.buf.get(), v.td.nelements(), v.td.ne[0],
                                   (const int32_t *)values.at(d.counters[(size_t)mk.second].first).td.data, stream);
                (void)pos;
            }
            run_ops(d.body);
            for (const auto &c : d.collect) {
                Value &dst = values.at(c.first);
                const Value &src = values.at(c.second);
                const size_t nb = nbytes_of(*src.spec, binding);
                cuda_check(cudaMemcpyAsync(dst.buf.get() + (size_t)i * nb, src.td.data, nb, cudaMemcpyDeviceToDevice, stream),
                           "collect");
            }
            bool stop = false;
            for (const auto &u : d.until) {
                int32_t v = 0;
                cuda_check(cudaMemcpyAsync(&v, values.at(u.first).td.data, 4, cudaMemcpyDeviceToHost, stream), "until");
                cuda_check(cudaStreamSynchronize(stream), "until");
                stop = stop || std::find(u.second.begin(), u.second.end(), v) != u.second.end();
            }
            if (stop) break;
        }
    }
}

void Model::run_entry(const std::string &name) {
    const Entry *e = nullptr;
    for (const auto &en : entries)
        if (en.spec->name == name) e = &en;
    if (!e) throw std::runtime_error("no entry point named '" + name + "'");
    for (const TensorSpec *v : e->inputs)
        if (!input_set.at(v->name)) throw std::runtime_error("input '" + v->name + "' was never set");
    cuda_check(cudaSetDevice(device), "cudaSetDevice");
    rebind();
    for (auto &st : stage_stats) st = StageStat{};
    last_calls = 0;
    pending.clear();
    events_used = 0;
    const auto t0 = std::chrono::steady_clock::now();
    if (!run_ev[0]) {
        cuda_check(cudaEventCreate(&run_ev[0]), "cudaEventCreate");
        cuda_check(cudaEventCreate(&run_ev[1]), "cudaEventCreate");
    }
    cuda_check(cudaEventRecord(run_ev[0], stream), "cudaEventRecord");
    run_ops(e->spec->driver);
    cuda_check(cudaEventRecord(run_ev[1], stream), "cudaEventRecord");
    cuda_check(cudaStreamSynchronize(stream), ("entry '" + name + "'").c_str());
    last_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    float dms = 0;
    cuda_check(cudaEventElapsedTime(&dms, run_ev[0], run_ev[1]), "cudaEventElapsedTime");
    last_device_ms = dms;
    collect_times();
    int err = 0;
    cuda_check(cudaMemcpy(&err, d_err, sizeof err, cudaMemcpyDeviceToHost), "error word");
    if (err) {
        cudaMemset(d_err, 0, sizeof(int));
        if (err == 2)
            throw std::runtime_error("entry '" + name + "': a kernel's pipeline wait timed out (results are invalid)");
        if (err == 3)
            throw std::runtime_error("entry '" + name + "': a wait in the decode kernel timed out (results are invalid)");
        if (err == 4)
            throw std::runtime_error("entry '" + name + "': a tensor-parallel exchange timed out waiting for a peer rank "
                                     "(results are invalid)");
        throw std::runtime_error("entry '" + name + "': a set_rows index was outside its destination (row skipped)");
    }
    if (!trace_path.empty()) write_trace();
    if (!profile_path.empty() && !profile_lines.empty()) {
        if (FILE *f = std::fopen(profile_path.c_str(), "a")) {
            for (const auto &l : profile_lines) std::fprintf(f, "%s\n", l.c_str());
            std::fclose(f);
        }
        profile_lines.clear();
    }
}

void Model::reset_state() {
    cuda_check(cudaSetDevice(device), "cudaSetDevice");
    for (const auto &name : prog.state) {
        Value &v = values.at(name);
        cuda_check(cudaMemsetAsync(v.buf.get(), 0, v.buf.size(), stream), "reset");
    }
    cuda_check(cudaStreamSynchronize(stream), "reset");
}

void Model::tp_init(int rank, int world, size_t window_bytes, cudaIpcMemHandle_t *handle) {
    if (world < 2 || world > k::TP_MAX || rank < 0 || rank >= world)
        throw std::runtime_error("tensor parallel: world must be 2.." + std::to_string(k::TP_MAX) + " and 0 <= rank < world");
    if (tp.connected || !tp.win.empty()) throw std::runtime_error("tensor parallel: this model already joined a group");
    cuda_check(cudaSetDevice(device), "cudaSetDevice");
    if (window_bytes == 0) window_bytes = (size_t)64 << 20;
    tp.slot_bytes = (window_bytes / 2) / 256 * 256;
    if (tp.slot_bytes < 256) throw std::runtime_error("tensor parallel: window too small");
    tp.rank = rank;
    tp.world = world;
    tp.window.alloc((size_t)k::TP_FLAG_BYTES + 2 * tp.slot_bytes);
    tp.seq.alloc(sizeof(unsigned));
    tp.done.alloc(sizeof(unsigned));
    cuda_check(cudaIpcGetMemHandle(handle, tp.window.get()), "cudaIpcGetMemHandle");
    if (const char *e = std::getenv("GGML_COMPILER_B200_TP_TIMEOUT_MS")) tp.timeout_ns = (uint64_t)std::atoll(e) * 1000000ull;
}

void Model::tp_connect(const cudaIpcMemHandle_t *handles) {
    if (tp.window.size() == 0) throw std::runtime_error("tensor parallel: tp_init first");
    if (tp.connected) throw std::runtime_error("tensor parallel: already connected");
    cuda_check(cudaSetDevice(device), "cudaSetDevice");
    tp.win.assign((size_t)tp.world, nullptr);
    for (int r = 0; r < tp.world; r++) {
        if (r == tp.rank) {
            tp.win[(size_t)r] = tp.window.get();
            continue;
        }
        void *p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, handles[r], cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess)
            throw std::runtime_error("tensor parallel: mapping the window of rank " + std::to_string(r) + " failed: " +
                                     cudaGetErrorString(e));
        tp.win[(size_t)r] = (char *)p;
    }
    tp.connected = true;
    for (auto &c : calls) {
        c.stale = true;
        c.graph_ok = false;
    }
}

int *Model::counters(const std::string &key, size_t n) {
    auto it = counter_bufs.find(key);
    if (it != counter_bufs.end() && it->second.size() >= n * sizeof(int)) return (int *)it->second.get();
    cuda_check(cudaStreamSynchronize(stream), "counters");
    DevBuf b;
    b.alloc(std::max<size_t>(n, 1) * sizeof(int));  // zero-filled
    int *p = (int *)b.get();
    counter_bufs[key] = std::move(b);
    return p;
}

const float *Model::rope_table(int n_dims, float base, float scale, float attn, const std::string &ff_key,
                               const float *ff, int64_t *npos) {
    char key[256];
    std::snprintf(key, sizeof key, "%d/%a/%a/%a/%s", n_dims, base, scale, attn, ff_key.c_str());
    auto it = rope_tables.find(key);
    *npos = rope_positions;
    if (it != rope_tables.end()) return (const float *)it->second.get();
    // ggml's rope cache: theta starts at the position and is multiplied by theta_scale once per
    // frequency; cos and sin come from the host libm.
    const int half = n_dims / 2;
    std::vector<float> cs((size_t)(rope_positions * half * 2));
    const float theta_scale = ::powf(base, -2.0f / (float)n_dims);
    for (int64_t p = 0; p < rope_positions; p++) {
        float theta = (float)p;
        for (int i = 0; i < half; i++) {
            const float t = scale * (ff ? theta / ff[i] : theta);
            cs[(size_t)((p * half + i) * 2)] = ::cosf(t) * attn;
            cs[(size_t)((p * half + i) * 2 + 1)] = ::sinf(t) * attn;
            theta *= theta_scale;
        }
    }
    DevBuf buf;
    buf.alloc(cs.size() * 4);
    cuda_check(cudaMemcpy(buf.get(), cs.data(), cs.size() * 4, cudaMemcpyHostToDevice), "rope table");
    const float *p = (const float *)buf.get();
    rope_tables.emplace(key, std::move(buf));
    return p;
}

// One text line per traced phase and CTA: label, CTA, then the four stamps in ns relative to the
// earliest phase start of the call site.
void Model::write_trace() {
    FILE *f = std::fopen(trace_path.c_str(), "w");
    if (!f) return;
    const int nctas = k::mega_ctas();
    for (auto &c : calls) {
        if (!c.trace.size() || c.trace_labels.empty()) continue;
        std::vector<uint64_t> h(c.trace.size() / 8);
        cuda_check(cudaMemcpy(h.data(), c.trace.get(), c.trace.size(), cudaMemcpyDeviceToHost), "trace");
        uint64_t t0 = ~0ull;
        for (size_t i = 0; i < h.size(); i += 4)
            if (h[i]) t0 = std::min(t0, h[i]);
        std::fprintf(f, "# stage %s ctas %d phases %zu\n", c.stage->name.c_str(), nctas, c.trace_labels.size());
        for (const auto &r : c.trace_runs) {
            const uint64_t *run = &h[(size_t)nctas * r.first * 4];  // [CTA][phase of the run][4]
            for (size_t p = 0; p < r.second; p++)
                for (int cta = 0; cta < nctas; cta++) {
                    const uint64_t *st = run + ((size_t)cta * r.second + p) * 4;
                    std::fprintf(f, "%s\t%d", c.trace_labels[r.first + p].c_str(), cta);
                    for (int k = 0; k < 4; k++) std::fprintf(f, "\t%lld", st[k] ? (long long)(st[k] - t0) : -1ll);
                    std::fprintf(f, "\n");
                }
        }
        cuda_check(cudaMemset(c.trace.get(), 0, c.trace.size()), "trace");
    }
    std::fclose(f);
}

}  // namespace gcb
