// The executor behind the C ABI: one loaded program on one B200.
//
// Counterpart of the reference's runtime core (runtime/src/ggml_compiler_rt.cpp:138-732): load
// (:250-281), weights (:445-479), driver values (:488-546), per-binding views (:548-568), call
// sites (:570-732) and the driver loop (:356-443). Instead of ggml graphs, each call site is
// planned into a list of kernel launches with every pointer resolved for the current binding, its
// intermediates packed into one arena by liveness, and replayed as a CUDA graph.
#pragma once

#include <cuda_runtime.h>

#include <functional>
#include <map>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "gc_gguf.h"
#include "gc_kernels.h"
#include "gc_program.h"

namespace gcb {

class DevBuf {
  public:
    DevBuf() = default;
    DevBuf(const DevBuf &) = delete;
    DevBuf &operator=(const DevBuf &) = delete;
    DevBuf(DevBuf &&o) noexcept : p_(o.p_), n_(o.n_) { o.p_ = nullptr, o.n_ = 0; }
    DevBuf &operator=(DevBuf &&o) noexcept;
    ~DevBuf() { release(); }
    void alloc(size_t n);  // frees any previous allocation; zero-filled
    void release();
    char *get() const { return (char *)p_; }
    size_t size() const { return n_; }

  private:
    void *p_ = nullptr;
    size_t n_ = 0;
};

struct Step {
    const char *kind = "";  // kernel family, for profiles
    std::string node;       // the node(s) it runs
    std::function<void(cudaStream_t)> run;
    double bytes = 0;       // algorithmic bytes moved (weights, activations, KV)
};

// One call site planned for one binding of the symbols its stage reads: its launches with every
// pointer resolved, the arena holding its intermediates, and the CUDA graph that replays them.
struct SitePlan {
    std::vector<int64_t> key;  // the stage's symbols, in symbol order, at this binding
    std::vector<Step> steps;
    DevBuf arena;
    cudaGraphExec_t graph = nullptr;
    uint64_t last_use = 0;
    // GGML_COMPILER_B200_TRACE: per-CTA stamps of the traced launches, [launch][CTA][8]
    struct TraceEntry {
        std::string kind, node;
        size_t offset, ctas;
    };
    DevBuf trace;
    std::vector<TraceEntry> trace_index;
    DevBuf act;  // Q8_0 activation rows handed between fused steps, and their counters
    SitePlan() = default;
    SitePlan(const SitePlan &) = delete;
    SitePlan &operator=(const SitePlan &) = delete;
    ~SitePlan() {
        if (graph) cudaGraphExecDestroy(graph);
    }
};

// A `call` step of an entry's driver. Its plans are kept per binding (up to kPlansPerSite, the
// least recently used is dropped), so a loop that moves between KV windows switches plans without
// planning again.
struct CallSite {
    static constexpr size_t kPlansPerSite = 4;
    const StageSpec *stage = nullptr;
    int stage_index = 0;
    const DriverStep *step = nullptr;
    std::vector<std::unique_ptr<SitePlan>> plans;
};

// The device state of one loop of the program (gc_model.cu, kernels/gc_loop.cu) and the stretch
// graphs made for it, one per binding.
struct LoopRuntime {
    DevBuf words;    // iter, stop, end, then the counters' start values
    DevBuf scalars;  // per-iteration scalar values, [scalar][trips]
    k::LoopDev dev;
    struct Graph {
        std::vector<int64_t> key;
        cudaGraphExec_t exec = nullptr;
    };
    std::vector<Graph> graphs;
    bool device_ok = true;  // false once a conditional graph could not be built
    LoopRuntime() = default;
    LoopRuntime(const LoopRuntime &) = delete;
    LoopRuntime &operator=(const LoopRuntime &) = delete;
    ~LoopRuntime() {
        for (auto &g : graphs)
            if (g.exec) cudaGraphExecDestroy(g.exec);
    }
};

// Batched decode (gc_batch.cpp; an extension: the reference decodes one sequence). Sequence slots
// hold copies of the program's state values (its KV caches); one batched step runs the decode
// stage's fused groups for n sequences at once, sequence i in slot i at its own position, so each
// weight stream serves up to 8 rows. Plans are kept per (entry, n, attention window).
struct BatchRuntime {
    static constexpr int kMaxSeq = 16;
    static constexpr size_t kMaxPlans = 8;
    int n_seq = 0;
    std::unordered_map<std::string, DevBuf> slots;  // state value -> n_seq copies, back to back
    DevBuf io;       // tok[16], pos[16], next[16], step, then the mask rows
    int32_t *tok = nullptr, *pos = nullptr, *next = nullptr, *step = nullptr;
    __half *mask = nullptr;   // [kMaxSeq][max_window]
    int64_t max_window = 0;   // rows of the smallest KV cache
    DevBuf logits_buf;        // [kMaxSeq][vocab] f32, made with the first plan
    int64_t vocab = 0;
    DevBuf gen;  // generated tokens, [steps][n]
    struct Plan {
        std::string entry;
        int n = 0;
        int64_t window = 0;
        std::unique_ptr<SitePlan> site;
        uint64_t last_use = 0;
    };
    std::vector<Plan> plans;
    uint64_t clock = 0;
};

struct Weight {
    TD td;
    DevBuf data, scales;
};

struct Value {
    const TensorSpec *spec = nullptr;
    DevBuf buf;  // room for the largest binding
    TD td;       // bound view (contiguous)
};

struct KernelStat {
    double ms = 0, bytes = 0;
    int launches = 0;
};

// Tensor parallelism: this process is rank `rank` of `world`, one GPU each. Decode GEMVs split
// their rows (attention its heads) over the ranks and exchange the slices through the ranks'
// windows (kernels/gc_tp.cu); everything else runs whole on every rank.
struct TpGroup {
    int rank = 0, world = 1;
    DevBuf window;  // flag words + two exchange slots, exported to the peers
    size_t slot_bytes = 0;
    DevBuf seq;                        // exchanges done (device word)
    DevBuf done;                       // CTAs of the running exchange that finished (device word)
    std::vector<char *> win;           // every rank's window as mapped here (own: window.get())
    bool connected = false;
    uint64_t timeout_ns = 60000000000ull;  // GGML_COMPILER_B200_TP_TIMEOUT_MS
    bool active() const { return connected && world > 1; }
};

struct Model {
    ProgramSpec prog;
    GgufFile gguf;
    int device = -1;
    std::string backend_name;
    cudaStream_t stream = nullptr;
    std::unordered_map<std::string, Weight> weights;
    std::unordered_map<std::string, Value> values;
    struct Entry {
        const EntrySpec *spec = nullptr;
        std::vector<const TensorSpec *> inputs, outputs;
    };
    std::vector<Entry> entries;
    std::map<std::string, bool> input_set;
    std::vector<CallSite> calls;
    std::vector<int64_t> binding;
    struct StageStat {
        double ms = 0;
        int calls = 0;
    };
    std::vector<StageStat> stage_stats;
    double last_ms = 0, last_device_ms = 0;
    int last_calls = 0;
    cudaEvent_t run_ev[2] = {nullptr, nullptr};
    int *d_err = nullptr;  // device error word (set_rows index out of range, ...)
    int64_t rope_positions = 4096;
    std::map<std::string, DevBuf> rope_tables;
    bool use_graphs = true;
    bool use_device_loops = true;  // GGML_COMPILER_B200_DEVICE_LOOPS=0: loops checked on the host every iteration
    bool profiling = false;
    int64_t l2_prefetch_bytes = 0;   // GCB_L2_PREFETCH_MB: what each fused GEMV prefetches of the next one's weights
    // GCB_ACT_HANDOFF: which producers hand the next GEMV its row quantized (bit 0: the attention
    // merge; bit 1: a residual GEMV's last CTA, normed; bit 2: the SwiGLU GEMV per block). Bit 1
    // measured slower (its serial tail), so the default is 5.
    int act_handoff = 5;
    int prologue_hold = 3;
    // GCB_PRODUCER_WAIT_AFTER_ATTN: the GEMV after attention streams only once attention completed
    // (1), or is launched without programmatic dependent launch at all (2)
    int producer_wait_after_attn = 0;    // GCB_PROLOGUE_HOLD: FusedArgs::hold_pieces of the single-row GEMVs
    // GCB_KV_PREFETCH=k: the GEMV k launches before a one-row attention prefetches its K/V into L2
    // (1: the QKV GEMV right before it; 2: the one before that, the previous layer's down GEMV)
    int kv_prefetch = 0;
    // GCB_ATTN_OVERLAP (default 1): one-row cluster attention over a cache a fused QKV GEMV writes
    // issues its K/V copies before the dependent-launch wait (re-reading the written row after it).
    // GCB_QKV_ONE_PER_SM=1: that QKV GEMV also runs one CTA per SM so the attention's CTAs can be
    // resident beside it (measured slower: the GEMV loses half its CTAs and the attention CTAs
    // still start only at its tail).
    bool attn_overlap = true;
    bool qkv_one_per_sm = false;
    // GGML_COMPILER_B200_PREFILL_ATTN=tc: prefill attention (16+ query rows) on the tensor cores,
    // within tolerance of the checker instead of bit-exact
    bool prefill_attn_tc = false;
    // Launches run one by one (profiling, graphs off) rather than as one graph: early K/V copies
    // are then off (consecutive steps' launches could overlap under programmatic dependent launch)
    bool direct_launch = false;
    bool stream_evict_first = true;  // GCB_STREAM_EVICT_FIRST=0: GEMV weight streams without the L2 evict-first policy
    std::map<std::string, KernelStat> kstats;
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> event_pool;
    size_t events_used = 0;
    struct PendingTime {
        std::vector<int> stages;  // the stages the timed region is charged to, evenly
        cudaEvent_t a, b;
    };
    std::vector<PendingTime> pending;
    std::string profile_path;  // GGML_COMPILER_PROFILE
    std::string trace_path;    // GGML_COMPILER_B200_TRACE: per-CTA stamps of the last run's launches
    std::vector<std::string> profile_lines;
    uint64_t plan_clock = 0;  // orders plan uses (least recently used plan of a site is dropped)
    TpGroup tp;
    std::unique_ptr<BatchRuntime> batch;

    // Batched decode (gc_batch.cpp). seq_slots allocates n zeroed slots (dropping earlier ones);
    // seq_copy copies the state between slots, -1 naming the model's own state (what the entries
    // read and write). decode_batch runs one step for sequences 0..n-1 (tok / pos host arrays):
    // logits [n][vocab] and greedy tokens [n] to host memory when non-null. generate_batch runs
    // `steps` greedy steps from first / start, with no host round trip between steps, and writes
    // the tokens [steps][n].
    void seq_slots(int n);
    void seq_copy(int dst, int src);
    void decode_batch(const std::string &entry, int n, const int32_t *tok, const int32_t *pos, float *logits, int32_t *next);
    void generate_batch(const std::string &entry, int n, const int32_t *first, const int32_t *start, int steps, int32_t *out);

    ~Model();
    // Tensor parallelism: allocate and export this rank's window (before any run), then map every
    // rank's window from the handles of all ranks in rank order; plans made before are redone.
    void tp_init(int rank, int world, size_t window_bytes, cudaIpcMemHandle_t *handle);
    void tp_connect(const cudaIpcMemHandle_t *handles);
    void load(const char *path, int backend, int device, bool allow_cpu_fallback);
    void rebind();  // the spec's dims and the values' views follow `binding`
    void run_entry(const std::string &name);
    void reset_state();
    size_t nbytes_of(const TensorSpec &v, const std::vector<int64_t> &b) const;
    const float *rope_table(int n_dims, float base, float scale, float attn, const std::string &ff_key,
                            const float *ff_host, int64_t *npos);
    // Zeroed device ints that persist across launches (arrival counters), one buffer per key.
    int *counters(const std::string &key, size_t n);
    std::map<std::string, DevBuf> counter_bufs;
    // The plan of `site` for the current binding, made if missing.
    SitePlan &plan_for(CallSite &site);

    std::pair<cudaEvent_t, cudaEvent_t> events();
    void collect_times();

  private:
    std::vector<int64_t> bound;  // the binding the spec and the value views were last bound to
    std::map<const LoopSpec *, std::unique_ptr<LoopRuntime>> loops;
    LoopRuntime &loop_runtime(const LoopSpec &L);
    void loop_bind(LoopRuntime &rt, const LoopSpec &L);
    cudaGraphExec_t loop_graph(LoopRuntime &rt, const LoopSpec &L, const std::vector<SitePlan *> &body);
    void load_weights();
    void alloc_values();
    void bind_values();
    void prepare(std::vector<DriverStep> &steps);  // call sites for every call, checks of every loop
    void run_steps(const std::vector<DriverStep> &steps);
    void run_call(const DriverStep &d);
    void launch_plan(SitePlan &p, int stage_index);
    void run_loop(const LoopSpec &loop);
    void write_trace();
    BatchRuntime::Plan &batch_plan(const std::string &entry, int n, int64_t window);
    void batch_launch(SitePlan &p);
    void batch_check_error(const char *what);
};

// Plans one stage call for the current binding into kernel launches (gc_plan.cpp).
void plan_call_site(Model &m, const CallSite &cs, SitePlan &plan);

void cuda_check(cudaError_t e, const char *what);

}  // namespace gcb
