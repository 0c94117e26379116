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


struct FileCloser {
    void operator()(FILE *f) const { std::fclose(f); }
};

__global__ void set_i32_kernel(int32_t *p, int32_t v) { *p = v; }

}  // namespace

Model::~Model() {
    if (device >= 0) cudaSetDevice(device);
    if (stream) cudaStreamSynchronize(stream);
    loops.clear();
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
    const auto ne = v.ne_at(b);
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
    if (const char *g = std::getenv("GGML_COMPILER_B200_GRAPHS")) use_graphs = std::atoi(g) != 0;
    if (const char *g = std::getenv("GGML_COMPILER_B200_DEVICE_LOOPS")) use_device_loops = std::atoi(g) != 0;
    if (const char *p = std::getenv("GGML_COMPILER_B200_TRACE")) trace_path = p;
    if (const char *g = std::getenv("GCB_L2_PREFETCH_MB")) l2_prefetch_bytes = (int64_t)(std::atof(g) * (1 << 20));
    if (const char *g = std::getenv("GCB_STREAM_EVICT_FIRST")) stream_evict_first = std::atoi(g) != 0;
    if (const char *g = std::getenv("GCB_ACT_HANDOFF")) act_handoff = std::atoi(g);
    if (const char *g = std::getenv("GCB_PROLOGUE_HOLD")) prologue_hold = std::atoi(g);
    if (const char *g = std::getenv("GCB_PRODUCER_WAIT_AFTER_ATTN")) producer_wait_after_attn = std::atoi(g);
    if (const char *g = std::getenv("GCB_KV_PREFETCH")) kv_prefetch = std::atoi(g);
    if (const char *g = std::getenv("GCB_ATTN_OVERLAP")) attn_overlap = std::atoi(g) != 0;
    if (const char *g = std::getenv("GCB_QKV_ONE_PER_SM")) qkv_one_per_sm = std::atoi(g) != 0;
    if (const char *g = std::getenv("GGML_COMPILER_B200_PREFILL_ATTN")) prefill_attn_tc = std::strcmp(g, "tc") == 0;

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
    bound = binding;
    for (auto &e : prog.entries) prepare(e.driver);
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
            // Q4_0 / Q8_0 are repacked into the tiled layout; q5_0 / iq4_nl expanded into it as Q8_0
            const bool q = t.type == T_Q4_0 || t.type == T_Q8_0 || k::expands_to_q8_0(t.type);
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
                if (k::expands_to_q8_0(t.type)) {
                    w.td.type = T_Q8_0;
                    w.data.alloc(k::quant_device_bytes(T_Q8_0, rows, K));
                    k::expand_to_q8_0(t.type, (const uint8_t *)raw.get(), rows, K, w.data.get(), stream);
                } else {
                    w.data.alloc(k::quant_device_bytes(t.type, rows, K));
                    k::repack_quant(t.type, (const uint8_t *)raw.get(), rows, K, w.data.get(), stream);
                }
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
        if (!v.reads) {
            most = v.ne[0] * v.ne[1] * v.ne[2] * v.ne[3];
        } else {  // the largest size over the corners of the box of the symbols it reads
            std::vector<size_t> idx;
            for (size_t k = 0; k < prog.symbols.size(); k++)
                if ((v.reads >> k) & 1u) idx.push_back(k);
            std::vector<int64_t> b = binding;
            for (size_t corner = 0; corner < ((size_t)1 << idx.size()); corner++) {
                for (size_t k = 0; k < idx.size(); k++)
                    b[idx[k]] = (corner >> k) & 1 ? prog.symbols[idx[k]].max : prog.symbols[idx[k]].min;
                const auto ne = v.ne_at(b);
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

// Every call of every entry gets its call site, planned once at load for the load binding, so a
// node this backend cannot run fails the load and names itself. Loops are checked here too.
void Model::prepare(std::vector<DriverStep> &steps) {
    for (DriverStep &d : steps) {
        if (d.is_loop) {
            const LoopSpec &L = *d.loop;
            auto val = [&](const std::string &name) -> const Value & {
                auto it = values.find(name);
                if (it == values.end()) throw std::runtime_error("loop uses undeclared value '" + name + "'");
                return it->second;
            };
            auto typed = [&](const std::string &name, Type t, const char *what) {
                if (val(name).spec->type != t)
                    throw std::runtime_error(std::string("loop ") + what + " '" + name + "' must be " + type_name(t));
            };
            for (const auto &c : L.carry) {
                const TD &x = val(c.dst).td, &y = val(c.src).td;
                if (x.type != y.type || x.ne[0] != y.ne[0] || x.ne[1] != y.ne[1] || x.ne[2] != y.ne[2] || x.ne[3] != y.ne[3])
                    throw std::runtime_error("loop carry '" + c.dst + "' does not match its initial value '" + c.src + "'");
            }
            for (const auto &c : L.counters) typed(c.value, T_I32, "counter"), typed(c.start, T_I32, "counter start");
            for (const auto &mk : L.masks) typed(mk.value, T_F32, "mask");
            for (const auto &sc : L.scalars) typed(sc.value, T_F32, "scalar");
            for (const auto &u : L.until) typed(u.value, T_I32, "stop value");
            for (const auto &sl : L.slices) {
                const TD &x = val(sl.dst).td, &y = val(sl.src).td;
                if (x.type != y.type || y.nelements() != x.nelements() * L.trips)
                    throw std::runtime_error("loop slice '" + sl.dst + "' does not match its source '" + sl.src + "'");
            }
            for (const auto &c : L.collect) (void)val(c.dst), (void)val(c.src);
            prepare(d.loop->body);
            continue;
        }
        if (d.call_site >= 0) continue;
        CallSite site;
        site.stage = &prog.stages[(size_t)d.stage];
        site.stage_index = d.stage;
        site.step = &d;
        d.call_site = (int)calls.size();
        calls.push_back(std::move(site));
        plan_for(calls.back());
    }
}

void Model::rebind() {
    if (binding == bound) return;
    prog.bind(binding);
    bind_values();
    bound = binding;
}

SitePlan &Model::plan_for(CallSite &site) {
    rebind();
    std::vector<int64_t> key;
    for (size_t k = 0; k < binding.size(); k++)
        if (site.stage->reads_symbol(k)) key.push_back(binding[k]);
    for (auto &p : site.plans)
        if (p->key == key) {
            p->last_use = ++plan_clock;
            return *p;
        }
    if (site.plans.size() >= CallSite::kPlansPerSite) {
        // the plan least recently used goes; launches already queued may still read its arena
        cuda_check(cudaStreamSynchronize(stream), "dropping a plan");
        auto old = std::min_element(site.plans.begin(), site.plans.end(),
                                    [](const auto &x, const auto &y) { return x->last_use < y->last_use; });
        site.plans.erase(old);
    }
    auto p = std::make_unique<SitePlan>();
    p->key = key;
    plan_call_site(*this, site, *p);
    p->last_use = ++plan_clock;
    site.plans.push_back(std::move(p));
    return *site.plans.back();
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
        for (int st : p.stages) stage_stats[(size_t)st].ms += ms / (double)p.stages.size();
    }
    pending.clear();
    events_used = 0;
}

// Records a timed region on the stream around `body`, charged to `stages` (split evenly).
template <class F>
static void timed(Model &m, std::vector<int> stages, F &&body) {
    if (m.events_used > 4096) {  // long host loops: fold finished timings so the event pool stays small
        cuda_check(cudaStreamSynchronize(m.stream), "stage timing");
        m.collect_times();
    }
    auto ev = m.events();
    cuda_check(cudaEventRecord(ev.first, m.stream), "cudaEventRecord");
    body();
    cuda_check(cudaEventRecord(ev.second, m.stream), "cudaEventRecord");
    m.pending.push_back({std::move(stages), ev.first, ev.second});
}

void Model::launch_plan(SitePlan &p, int stage_index) {
    direct_launch = profiling || !profile_path.empty() || !use_graphs;
    timed(*this, {stage_index}, [&] {
        if (profiling || !profile_path.empty()) {  // each launch on its own, timed
            for (const auto &st : p.steps) {
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
                    profile_lines.push_back(prog.stages[(size_t)stage_index].name + "\t" + st.node + "\t" + st.kind + "\t" +
                                            std::to_string(ms));
            }
        } else if (use_graphs) {
            if (!p.graph) {
                cudaGraph_t g = nullptr;
                cuda_check(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
                try {
                    for (const auto &st : p.steps) st.run(stream);
                } catch (...) {
                    cudaStreamEndCapture(stream, &g);
                    if (g) cudaGraphDestroy(g);
                    throw;
                }
                cuda_check(cudaStreamEndCapture(stream, &g), "cudaStreamEndCapture");
                const cudaError_t e = cudaGraphInstantiate(&p.graph, g, 0);
                cudaGraphDestroy(g);
                cuda_check(e, "cudaGraphInstantiate");
            }
            cuda_check(cudaGraphLaunch(p.graph, stream), "cudaGraphLaunch");
        } else {
            for (const auto &st : p.steps) st.run(stream);
        }
    });
    stage_stats[(size_t)stage_index].calls++;
    last_calls++;
}

void Model::run_call(const DriverStep &d) {
    CallSite &site = calls[(size_t)d.call_site];
    launch_plan(plan_for(site), site.stage_index);
}

void Model::run_steps(const std::vector<DriverStep> &steps) {
    for (const DriverStep &d : steps) {
        if (d.is_loop) run_loop(*d.loop);
        else run_call(d);
    }
}

// ----------------------------------------------------------------------------------------- loops
//
// A loop runs on the device. Its per-iteration bookkeeping is two small kernels (gc_loop.cu) that
// take the iteration index from device memory, so the iterations between two changes of the
// symbol binding (a KV window growing by a block) are one CUDA graph: a guard kernel, then a
// conditional WHILE node whose body is loop_begin, the body's launches and loop_end, which
// decides whether the body runs again (no stop id seen, iterations left in the stretch). The host
// computes the binding of every iteration first (the counters' start values are read once), plans
// each stretch's calls before the loop starts, and launches one graph per stretch without waiting.
// A stop id ends the loop on the device; the remaining stretches' guards see it and run nothing.
// With graphs off, under profiling, for nested loops, or if the conditional graph cannot be made,
// the same kernels run iteration by iteration with the stop flag read back each time.

namespace {

void set_word(int32_t *p, int32_t v, cudaStream_t s) {
    set_i32_kernel<<<1, 1, 0, s>>>(p, v);
    cuda_check(cudaGetLastError(), "loop word");
}

}  // namespace

LoopRuntime &Model::loop_runtime(const LoopSpec &L) {
    auto &slot = loops[&L];
    if (slot) return *slot;
    if (L.counters.size() > (size_t)k::LOOP_MAX || L.masks.size() > (size_t)k::LOOP_MAX ||
        L.scalars.size() > (size_t)k::LOOP_MAX || L.slices.size() > (size_t)k::LOOP_MAX ||
        L.collect.size() > (size_t)k::LOOP_MAX || L.until.size() > (size_t)k::LOOP_MAX)
        throw std::runtime_error("loop has more than " + std::to_string(k::LOOP_MAX) +
                                 " counters, masks, scalars, slices, collects or stop values");
    for (const auto &u : L.until)
        if (u.ids.size() > (size_t)k::LOOP_MAX_IDS)
            throw std::runtime_error("loop stop value '" + u.value + "' has more than " + std::to_string(k::LOOP_MAX_IDS) + " ids");
    auto rt = std::make_unique<LoopRuntime>();
    rt->words.alloc((3 + k::LOOP_MAX) * sizeof(int32_t));
    int32_t *w = (int32_t *)rt->words.get();
    k::LoopDev &D = rt->dev;
    D.iter = w;
    D.stop = w + 1;
    D.end = w + 2;
    D.start = w + 3;
    if (!L.scalars.empty()) {
        std::vector<float> host;
        for (const auto &sc : L.scalars) host.insert(host.end(), sc.per_iteration.begin(), sc.per_iteration.end());
        rt->scalars.alloc(host.size() * sizeof(float));
        cuda_check(cudaMemcpy(rt->scalars.get(), host.data(), host.size() * sizeof(float), cudaMemcpyHostToDevice), "loop scalars");
    }
    slot = std::move(rt);
    return *slot;
}

// The value pointers of the loop's kernels at the current binding.
void Model::loop_bind(LoopRuntime &rt, const LoopSpec &L) {
    k::LoopDev &D = rt.dev;
    auto td = [&](const std::string &name) -> const TD & { return values.at(name).td; };
    D.n_counters = (int)L.counters.size();
    for (int k = 0; k < D.n_counters; k++) D.counter[k] = (int32_t *)td(L.counters[(size_t)k].value).data;
    D.n_masks = (int)L.masks.size();
    for (int k = 0; k < D.n_masks; k++) {
        const TD &m = td(L.masks[(size_t)k].value);
        D.mask[k] = (float *)m.data;
        D.mask_n[k] = m.nelements();
        D.mask_row[k] = m.ne[0];
        D.mask_counter[k] = L.masks[(size_t)k].counter;
    }
    D.n_scalars = (int)L.scalars.size();
    for (int k = 0; k < D.n_scalars; k++) {
        const TD &v = td(L.scalars[(size_t)k].value);
        D.scalar[k] = (float *)v.data;
        D.scalar_n[k] = v.nelements();
        D.scalar_vals[k] = (const float *)rt.scalars.get() + (size_t)k * (size_t)L.trips;
    }
    D.n_slices = (int)L.slices.size();
    for (int k = 0; k < D.n_slices; k++) {
        const TD &dst = td(L.slices[(size_t)k].dst);
        D.slice_dst[k] = dst.data;
        D.slice_src[k] = td(L.slices[(size_t)k].src).data;
        D.slice_bytes[k] = (int64_t)dst.nbytes();
    }
    D.n_collect = (int)L.collect.size();
    for (int k = 0; k < D.n_collect; k++) {
        const Value &src = values.at(L.collect[(size_t)k].src);
        D.collect_dst[k] = values.at(L.collect[(size_t)k].dst).buf.get();
        D.collect_src[k] = src.td.data;
        D.collect_bytes[k] = (int64_t)nbytes_of(*src.spec, binding);
    }
    D.n_until = (int)L.until.size();
    for (int k = 0; k < D.n_until; k++) {
        D.until_val[k] = (const int32_t *)td(L.until[(size_t)k].value).data;
        D.n_ids[k] = (int)L.until[(size_t)k].ids.size();
        for (int t = 0; t < D.n_ids[k]; t++) D.until_ids[k][t] = L.until[(size_t)k].ids[(size_t)t];
    }
}

// The stretch graph for the current binding: guard, then WHILE { loop_begin, body, loop_end }.
// Null if this loop cannot run as a conditional graph.
cudaGraphExec_t Model::loop_graph(LoopRuntime &rt, const LoopSpec &L, const std::vector<SitePlan *> &body) {
    for (auto &g : rt.graphs)
        if (g.key == binding) return g.exec;
    cudaGraph_t g = nullptr;
    cudaGraphExec_t exec = nullptr;
    cudaError_t e = cudaGraphCreate(&g, 0);
    auto fail = [&](const char *what) {
        if (std::getenv("GGML_COMPILER_B200_LOOP_DEBUG"))
            std::fprintf(stderr, "[ggml_compiler_b200] loop runs on the host: %s: %s\n", what, cudaGetErrorString(e));
        cudaGetLastError();
        if (g) cudaGraphDestroy(g);
        rt.device_ok = false;
        return (cudaGraphExec_t) nullptr;
    };
    if (e != cudaSuccess) return fail("cudaGraphCreate");
    cudaGraphConditionalHandle cond = 0;
    if ((e = cudaGraphConditionalHandleCreate(&cond, g, 0, 0)) != cudaSuccess) return fail("conditional handle");
    // the guard, captured into g, then the WHILE node after it
    if ((e = cudaStreamBeginCaptureToGraph(stream, g, nullptr, nullptr, 0, cudaStreamCaptureModeThreadLocal)) != cudaSuccess)
        return fail("capture of the guard");
    k::loop_guard(rt.dev, cond, stream);
    cudaGraph_t got = nullptr;
    if ((e = cudaStreamEndCapture(stream, &got)) != cudaSuccess) return fail("capture of the guard");
    cudaGraphNode_t guard = nullptr;
    size_t nn = 1;
    if ((e = cudaGraphGetNodes(g, &guard, &nn)) != cudaSuccess || nn != 1) return fail("guard node");
    cudaGraphNodeParams cp = {};
    cp.type = cudaGraphNodeTypeConditional;
    cp.conditional.handle = cond;
    cp.conditional.type = cudaGraphCondTypeWhile;
    cp.conditional.size = 1;
    cudaGraphNode_t wnode = nullptr;
    if ((e = cudaGraphAddNode(&wnode, g, &guard, 1, &cp)) != cudaSuccess) return fail("conditional node");
    cudaGraph_t bodyg = cp.conditional.phGraph_out[0];
    if ((e = cudaStreamBeginCaptureToGraph(stream, bodyg, nullptr, nullptr, 0, cudaStreamCaptureModeThreadLocal)) != cudaSuccess)
        return fail("capture of the body");
    try {
        k::loop_begin(rt.dev, stream);
        for (SitePlan *p : body)
            for (const auto &st : p->steps) st.run(stream);
        k::loop_end(rt.dev, cond, true, stream);
    } catch (...) {
        cudaGraph_t junk = nullptr;
        cudaStreamEndCapture(stream, &junk);
        e = cudaErrorUnknown;
        return fail("a launch of the body");
    }
    if ((e = cudaStreamEndCapture(stream, &got)) != cudaSuccess) return fail("capture of the body");
    if ((e = cudaGraphInstantiate(&exec, g, 0)) != cudaSuccess) return fail("instantiation");
    cudaGraphDestroy(g);
    rt.graphs.push_back({binding, exec});
    return exec;
}

void Model::run_loop(const LoopSpec &L) {
    LoopRuntime &rt = loop_runtime(L);
    const int64_t trips = L.trip_symbol >= 0 ? binding[(size_t)L.trip_symbol] : L.trips;
    for (const auto &c : L.carry) {
        const Value &src = values.at(c.src);
        cuda_check(cudaMemcpyAsync(values.at(c.dst).td.data, src.td.data, src.td.nbytes(), cudaMemcpyDeviceToDevice, stream),
                   "loop carry");
    }
    for (size_t k = 0; k < L.counters.size(); k++)
        cuda_check(cudaMemcpyAsync((int32_t *)rt.dev.start + k, values.at(L.counters[k].start).td.data, 4,
                                   cudaMemcpyDeviceToDevice, stream),
                   "loop counter start");
    cuda_check(cudaMemsetAsync(rt.dev.iter, 0, 2 * sizeof(int32_t), stream), "loop words");
    for (const auto &c : L.collect) {
        Value &dst = values.at(c.dst);
        cuda_check(cudaMemsetAsync(dst.buf.get(), 0, dst.buf.size(), stream), "loop collect");
    }
    if (trips <= 0) return;

    // the binding of every iteration: stretches of iterations that share one
    std::vector<int32_t> start(L.counters.size(), 0);
    if (!L.rebind.empty() && !L.counters.empty()) {
        cuda_check(cudaMemcpyAsync(start.data(), rt.dev.start, start.size() * 4, cudaMemcpyDeviceToHost, stream), "loop starts");
        cuda_check(cudaStreamSynchronize(stream), "loop starts");
    }
    struct Stretch {
        int64_t first, count;
        std::vector<int64_t> binding;
    };
    std::vector<Stretch> stretches;
    std::vector<int64_t> scope = binding;
    scope.resize(binding.size() + L.counters.size());
    for (int64_t i = 0; i < trips; i++) {
        std::vector<int64_t> b = binding;
        for (size_t k = 0; k < L.counters.size(); k++) scope[binding.size() + k] = (int64_t)start[k] + i;
        for (size_t k = 0; k < binding.size(); k++) scope[k] = stretches.empty() ? binding[k] : stretches.back().binding[k];
        for (const auto &rb : L.rebind) {
            const int64_t v = rb.value.eval(scope);
            const Symbol &sy = prog.symbols[(size_t)rb.symbol];
            if (v < sy.min || v > sy.max)
                throw std::runtime_error("loop sets " + sy.name + " to " + std::to_string(v) + " at iteration " +
                                         std::to_string(i) + ", outside [" + std::to_string(sy.min) + ", " +
                                         std::to_string(sy.max) + "]");
            b[(size_t)rb.symbol] = v;
            scope[(size_t)rb.symbol] = v;
        }
        if (stretches.empty() || stretches.back().binding != b) stretches.push_back({i, 0, b});
        stretches.back().count++;
    }

    bool device = use_graphs && use_device_loops && !profiling && profile_path.empty() && rt.device_ok;
    for (const auto &st : L.body) device = device && !st.is_loop;
    std::vector<int> body_stages;
    for (const auto &st : L.body)
        if (!st.is_loop) body_stages.push_back(st.stage);
    // every stretch's plans (and graphs) first: nothing is planned while the loop runs
    std::vector<std::vector<SitePlan *>> plans(stretches.size());
    std::vector<cudaGraphExec_t> graphs(stretches.size(), nullptr);
    for (size_t s = 0; s < stretches.size(); s++) {
        binding = stretches[s].binding;
        for (const auto &st : L.body)
            if (!st.is_loop) plans[s].push_back(&plan_for(calls[(size_t)st.call_site]));
        if (device) {
            loop_bind(rt, L);
            graphs[s] = loop_graph(rt, L, plans[s]);
            device = graphs[s] != nullptr;
        }
    }

    int64_t done = 0;
    if (device) {
        for (size_t s = 0; s < stretches.size(); s++) {
            set_word(rt.dev.end, (int32_t)(stretches[s].first + stretches[s].count), stream);
            timed(*this, body_stages, [&] { cuda_check(cudaGraphLaunch(graphs[s], stream), "loop graph"); });
        }
        int32_t ran = 0;
        cuda_check(cudaMemcpyAsync(&ran, rt.dev.iter, 4, cudaMemcpyDeviceToHost, stream), "loop iterations");
        cuda_check(cudaStreamSynchronize(stream), "loop");
        done = ran;
        for (int st : body_stages) stage_stats[(size_t)st].calls += (int)done;
        last_calls += (int)(done * (int64_t)body_stages.size());
    } else {
        for (size_t s = 0; s < stretches.size() && done == stretches[s].first; s++) {
            binding = stretches[s].binding;
            rebind();
            loop_bind(rt, L);
            for (int64_t i = 0; i < stretches[s].count; i++) {
                k::loop_begin(rt.dev, stream);
                run_steps(L.body);
                k::loop_end(rt.dev, 0, false, stream);
                int32_t stop = 0;
                cuda_check(cudaMemcpyAsync(&stop, rt.dev.stop, 4, cudaMemcpyDeviceToHost, stream), "loop stop");
                cuda_check(cudaStreamSynchronize(stream), "loop stop");
                done++;
                if (stop) break;
            }
        }
    }
    // the binding of the last iteration that ran stays in force, as after a host-driven loop
    for (const auto &st : stretches)
        if (done > st.first) binding = st.binding;
    rebind();
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
    run_steps(e->spec->driver);
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

// One line per CTA of every traced launch of every current plan, in plan order: stage, launch
// index, kind, node, CTA, then the stamps in ns relative to the earliest stamp of the file (-1:
// not recorded). A plan's stamps are those of its latest launch (a loop's last iteration).
void Model::write_trace() {
    FILE *f = std::fopen(trace_path.c_str(), "w");
    if (!f) return;
    std::vector<std::pair<std::string, const SitePlan *>> plans;  // every current plan with stamps
    for (const auto &c : calls)
        for (const auto &p : c.plans)
            if (p->trace.size()) plans.emplace_back(c.stage->name, p.get());
    if (batch)
        for (const auto &bp : batch->plans)
            if (bp.site->trace.size())
                plans.emplace_back("batch:" + bp.entry + "/" + std::to_string(bp.n) + "x" + std::to_string(bp.window), bp.site.get());
    std::vector<std::vector<uint64_t>> stamps;
    uint64_t t0 = ~0ull;
    for (const auto &pp : plans) {
        std::vector<uint64_t> h(pp.second->trace.size() / 8);
        cuda_check(cudaMemcpy(h.data(), pp.second->trace.get(), pp.second->trace.size(), cudaMemcpyDeviceToHost), "trace");
        for (uint64_t v : h)
            if (v) t0 = std::min(t0, v);
        stamps.push_back(std::move(h));
    }
    for (size_t k = 0; k < plans.size(); k++) {
        const SitePlan &p = *plans[k].second;
        const auto &h = stamps[k];
        for (size_t li = 0; li < p.trace_index.size(); li++) {
            const auto &e = p.trace_index[li];
            for (size_t cta = 0; cta < e.ctas; cta++) {
                const uint64_t *st = &h[e.offset + cta * 8];
                if (!st[0] && !st[2]) continue;  // a CTA the launch did not have
                std::fprintf(f, "%s\t%zu\t%s\t%s\t%zu", plans[k].first.c_str(), li, e.kind.c_str(), e.node.c_str(), cta);
                for (int s = 0; s < 8; s++) std::fprintf(f, "\t%lld", st[s] ? (long long)(st[s] - t0) : -1ll);
                std::fprintf(f, "\n");
            }
        }
    }
    std::fclose(f);
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
    // every plan is made again with this rank's share of the work and the exchanges
    cuda_check(cudaStreamSynchronize(stream), "tensor parallel");
    for (auto &c : calls) c.plans.clear();
    loops.clear();
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

}  // namespace gcb
