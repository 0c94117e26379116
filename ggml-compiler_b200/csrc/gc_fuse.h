// Call-site planner state and the fusion pass that replaces node groups with fused kernels.
#pragma once

#include <functional>
#include <memory>
#include <set>
#include <string>
#include <unordered_map>
#include <vector>

#include "gc_fused.h"
#include "gc_model.h"

namespace gcb {

struct Storage {
    size_t bytes = 0;
    int first = 0, last = 0;  // node indices of the first write and the last read
    size_t offset = 0;
};

// Per-launch settings of a fused GEMV step that depend on the steps around it, filled once the
// whole call site is planned: L2 prefetch of a later launch's weights (FusedArgs::pf), the
// stream's cache policy, and the Q8_0 activation hand-off (FusedArgs::xq / act_*).
struct GemvExtras {
    const char *p[3] = {nullptr, nullptr, nullptr};
    int64_t n[3] = {0, 0, 0};
    int evict_first = 0;
    const char *xq = nullptr;  // non-null: the input row comes staged (PRO_Q8)
    int act_mode = 0;
    char *act_out = nullptr;
    const float *act_norm_w = nullptr;
    float act_eps = 0.0f;
    int *act_cnt = nullptr;
    int hold_pieces = 0;
    int producer_waits = 0;
    int max_ctas = 0;
};

struct PlanStep {
    const char *kind;
    std::string node;
    std::vector<TD> tds;  // arena TDs are resolved to pointers before the launch closure is made
    std::function<void(cudaStream_t, const std::vector<TD> &)> fn;
    double bytes;
    // Fused GEMV steps: their arguments from the resolved TDs, and the L2 prefetch ranges the
    // launch takes (filled once every step of the call site is planned).
    std::function<FusedArgs(const std::vector<TD> &)> gemv;
    std::shared_ptr<GemvExtras> pf;
    // A one-row split attention step: its output row (`attn_out`, H x D floats) and where its merge
    // writes that row's Q8_0 blocks for the GEMV that reads it (null: nowhere).
    std::shared_ptr<char *> attn_act;
    const float *attn_out = nullptr;
    int64_t attn_k = 0;
    bool attn_early = false;  // the attention loads its K/V before the dependent-launch wait
};

struct Planner {
    Planner(Model &m, SitePlan &plan, const CallSite &site);
    Model &m;
    SitePlan &plan;
    const DriverStep &d;
    const StageSpec &s;
    std::unordered_map<std::string, TD> env;  // node ids and stage params -> views
    std::vector<Storage> storages;
    std::vector<PlanStep> psteps;
    int cur = 0;
    bool copy_results = true;  // finish() copies the stage's results into their driver values
    std::set<int> head_sharded;  // tensor parallel: storages holding only this rank's query heads
    // K/V caches a fused QKV step of this plan writes, by their data pointer: the positions tensor
    // of the rows it writes (one-row attention over the cache then loads the other rows early)
    std::unordered_map<const char *, TD> kv_rows;
    // GGML_COMPILER_B200_TRACE: launches that record per-CTA stamps, and where (filled by finish)
    struct TraceReq {
        const char *kind;
        std::string node;
        size_t ctas;
        std::shared_ptr<uint64_t *> slot;
    };
    std::vector<TraceReq> traces;
    std::shared_ptr<uint64_t *> trace_slot(const char *kind, const std::string &node, size_t ctas);

    TD alloc(Type t, const int64_t *ne);          // a fresh arena tensor written at `cur`
    void *scratch_marker(size_t bytes, TD *out);  // scratch arena space for the launch at `cur`
    void use(const TD &t);                        // `t` is read at `cur`
    void add(const char *kind, const std::string &node, std::vector<TD> tds,
             std::function<void(cudaStream_t, const std::vector<TD> &)> fn, double bytes);
    // A fused GEMV step (gc_fused.h) that can also run as a decode-kernel phase. Under tensor
    // parallelism it computes this rank's rows and is followed by an exchange of its output (the
    // rope/QKV form: this rank's heads, no exchange; its query output is marked head_sharded).
    void add_gemv(const char *kind, const std::string &node, std::vector<TD> tds,
                  std::function<FusedArgs(const std::vector<TD> &)> build, double bytes);
    // Tensor parallel: after a step that wrote bytes [col[r], col[r + 1]) of each of `rows` rows of
    // `buf` on rank r, every rank gets the whole rows. False (nothing added) if the slices do not fit.
    bool add_exchange(const std::string &node, const TD &buf, int64_t rows, int64_t ld, const std::vector<int64_t> &col);
    bool exchange_fits(int64_t rows, int64_t ld, const std::vector<int64_t> &col) const;
    k::TpExchange exchange_args(int64_t rows, int64_t ld, const std::vector<int64_t> &col) const;
    TD src_of(const std::string &name);  // a node id, stage param or weight
    TD plan_node(const NodeSpec &n, const std::vector<TD> &src);
    void finish();
};

// What a matched group computes, by the names of what it reads and defines, independent of the
// token count it was matched at (the batched decode step re-plans groups for several sequences).
struct GroupDesc {
    enum Kind { QKV, GLU, HEAD, RESID } kind = RESID;
    std::string x;         // activation rows (a node id or stage parameter)
    std::string norm_w;    // QKV / GLU / HEAD: the rms_norm weight
    std::string w[3];      // weights: q, k, v / gate, up / the one matrix
    std::string res;       // RESID: the residual rows
    std::string pos;       // QKV: the positions parameter
    std::string kc, vc;    // QKV: the K and V cache parameters
    std::string out[3];    // QKV: rope(q), set_rows(k), set_rows(v); otherwise out[0]
    float eps = 0.0f, base = 0.0f;
    int64_t d = 0;         // input width
    int64_t N = 0;         // output width
    int64_t D = 0, H = 0, Hkv = 0;
};

// A set of node groups, each emitted as fused launches at its anchor (its last node).
struct FusionGroup {
    std::vector<size_t> nodes;
    size_t anchor = 0;
    std::function<void(Planner &)> emit;  // plans the launches and defines the group's visible outputs
    std::shared_ptr<GroupDesc> desc;
};

struct FusionPlan {
    std::vector<int> group_of;  // node index -> group, or -1
    std::vector<FusionGroup> groups;
    bool covered(size_t i) const { return i < group_of.size() && group_of[i] >= 0; }
    void emit_if_anchor(size_t i, Planner &p) {
        const FusionGroup &g = groups[(size_t)group_of[i]];
        if (g.anchor == i) g.emit(p);
    }
};

FusionPlan find_fusions(Model &m, const StageSpec &s, Planner &p);

}  // namespace gcb
