// Batched decode: one step of the decode stage for up to 16 sequences at once, sequence i in
// sequence slot i at its own position. An extension: the reference decodes one sequence per model
// (ggml_compiler/llm.py:64 builds the decode entry for batch 1; runtime/src/ggml_compiler_rt.cpp
// holds one copy of each state value).
//
// The decode stage of a program is written for one token, and its views are specialised to that
// (a [d, 1] row reshaped to [D, 1, Hkv] where a many-token stage permutes), so the batched step is
// not re-derived from the stage's shapes. It is planned from what the fusion pass recognised in
// the stage (gc_fuse.cpp GroupDesc: rms_norm + QKV + rope + KV rows, rms_norm + gate/up + SwiGLU,
// matmul + residual, rms_norm + output head), walking the stage's nodes in order:
//   - a fused group runs at n activation rows, 8 rows per launch (the GEMV's row limit): the
//     weight stream of a launch serves every row of it; the QKV group writes row i's K/V rows into
//     slot i's caches at position pos[i] (FusedArgs::cache_nb3);
//   - views are checked to be the identity on a token's row (or a cache's leading rows) and pass
//     the value through;
//   - get_rows reads the n token ids; clamp / cast of the mask input are dropped: each sequence's
//     mask row (0 up to its position, -inf after) is built on the device at the start of the step;
//   - flash_attn runs the split-KV kernel over the sequences as its batch dimension (ne[3]), K/V
//     of sequence i in slot i; argmax gives each row's greedy token.
// Anything else in the stage (a node outside these forms) fails the plan with its name.
//
// Each row's arithmetic is the single-sequence path's: the GEMV keeps one row's block order and
// butterfly whatever its row count (up to 8), and a key past a sequence's position weighs exactly
// 0 under either mask, so a chunk of 64 keys that lies wholly past it changes nothing in the merge.
// Logits of sequence i therefore equal, bit for bit, those of the decode entry run on that
// sequence alone.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <stdexcept>
#include <string>
#include <unordered_map>

#include "gc_fuse.h"
#include "gc_fused.h"
#include "gc_model.h"

namespace gcb {

namespace {

bool is_view(const std::string &op) { return op == "reshape" || op == "view" || op == "permute"; }

// Laid out as a contiguous tensor of its shape (dims of extent 1 take any stride).
bool dense(const TD &t) {
    int64_t want = (int64_t)t.elsize();
    for (int i = 0; i < 4; i++) {
        if (t.ne[i] == 1) continue;
        if (t.nb[i] != want) return false;
        want *= t.ne[i];
    }
    return true;
}

double qweight_bytes(const TD &w) { return (double)w.ne[1] * (double)(w.ne[0] / 32) * (quant_code_bytes(w.type) + 2); }

void put_weight(FusedArgs &a, int slot, const TD &w) {
    a.wc[slot] = w.data;
    a.ws[slot] = w.scales;
    a.wrows[slot] = w.ne[1];
    a.qtype = w.type;
}

// Bytes of M activation rows of K values in the GEMV's Q8_0 staging layout (codes, f32 block
// scales, 8 x code sums; rounded to 128), as kernels/gc_gemv_dev.cuh gemv_act_bytes lays them out.
size_t act_bytes(int64_t M, int64_t K) { return (size_t)((M * K + M * (K / 32) * 8 + 127) / 128 * 128); }

// A value of the decode stage as the batched step holds it.
struct BV {
    enum Kind { ROWS, CACHE, MASK, INDEX, TOKENS } kind = ROWS;
    TD td;              // ROWS: [width, n] f32; CACHE: slot 0's cache [D, rows, Hkv, 1]; TOKENS: [n] i32
    int64_t width = 0;  // ROWS
    int64_t slot = 0;   // CACHE: bytes from one slot to the next
    std::string param;  // INDEX: the stage parameter it views
};

struct BatchPlanner {
    Model &m;
    BatchRuntime &rt;
    Planner &p;
    const StageSpec &s;
    const DriverStep &d;
    int n;
    int64_t window;
    std::unordered_map<std::string, BV> bv;
    std::unordered_map<std::string, const std::array<int64_t, 4> *> spec_ne;
    std::unordered_map<std::string, Type> spec_type;
    std::string tok_param, pos_param;
    bool head_done = false;

    BatchPlanner(Model &m, BatchRuntime &rt, Planner &p, const StageSpec &s, const DriverStep &d, int n, int64_t window)
        : m(m), rt(rt), p(p), s(s), d(d), n(n), window(window) {}

    [[noreturn]] void fail(const NodeSpec &x, const std::string &msg) const {
        throw std::runtime_error("batched decode of stage '" + s.name + "': " + x.where() + ": " + msg);
    }
    // by value: the map may rehash when the caller then defines a value
    BV get(const NodeSpec &x, const std::string &name) const {
        auto it = bv.find(name);
        if (it == bv.end()) fail(x, "reads '" + name + "', which the batched step does not hold");
        return it->second;
    }
    BV rows(const NodeSpec &x, const std::string &name, int64_t width) const {
        const BV v = get(x, name);
        if (v.kind != BV::ROWS || (width > 0 && v.width != width))
            fail(x, "'" + name + "' is not one activation row of " + std::to_string(width) + " values per sequence");
        return v;
    }
    BV cache(const NodeSpec &x, const std::string &name) const {
        const BV v = get(x, name);
        if (v.kind != BV::CACHE) fail(x, "'" + name + "' is not a K/V cache held in sequence slots");
        return v;
    }
    void index_role(const NodeSpec &x, const std::string &name, std::string &role, const char *what) {
        const BV v = get(x, name);
        if (v.kind != BV::INDEX) fail(x, std::string("its ") + what + " '" + name + "' is not an i32 stage parameter");
        if (!role.empty() && role != v.param) fail(x, std::string("two different ") + what + " parameters");
        role = v.param;
    }
    // A fake contiguous descriptor of a stage value's one-token shape (views are replayed on it).
    TD fake(const std::string &name) const {
        TD t;
        t.type = spec_type.at(name);
        for (int i = 0; i < 4; i++) t.ne[i] = (*spec_ne.at(name))[(size_t)i];
        set_contiguous(t);
        return t;
    }
    TD alloc_rows(int64_t width) {
        const int64_t ne[4] = {width, n, 1, 1};
        return p.alloc(T_F32, ne);
    }
    BV as_rows(const TD &t, int64_t width) const {
        BV v;
        v.kind = BV::ROWS;
        v.td = t;
        v.width = width;
        return v;
    }

    void params() {
        for (size_t i = 0; i < s.params.size(); i++) {
            const TensorSpec &ps = s.params[i];
            spec_ne[ps.name] = &ps.ne;
            spec_type[ps.name] = ps.type;
            const std::string &arg = d.args[i];
            BV v;
            if (std::find(m.prog.state.begin(), m.prog.state.end(), arg) != m.prog.state.end()) {
                const Value &val = m.values.at(arg);
                if (val.td.type != T_F16 || !val.td.contiguous() || val.td.ne[3] != 1)
                    throw std::runtime_error("batched decode: state value '" + arg + "' is not an f16 cache [D, rows, heads]");
                v.kind = BV::CACHE;
                v.td = val.td;
                v.td.data = rt.slots.at(arg).get();
                v.slot = (int64_t)(rt.slots.at(arg).size() / (size_t)rt.n_seq);
            } else if (ps.type == T_I32) {
                v.kind = BV::INDEX;
                v.param = ps.name;
            } else {
                v.kind = BV::MASK;
            }
            bv[ps.name] = v;
        }
    }

    void view(const NodeSpec &x) {
        const BV src = get(x, x.src[0]);
        TD t;
        try {
            t = p.plan_node(x, {fake(x.src[0])});
        } catch (const std::exception &e) {
            fail(x, e.what());
        }
        const TD f = fake(x.src[0]);
        bool ok = true;
        switch (src.kind) {
            case BV::ROWS: ok = t.data == nullptr && dense(t) && t.nelements() == src.width; break;
            case BV::CACHE:
                ok = t.data == nullptr && t.ne[0] == f.ne[0] && t.ne[2] == f.ne[2] && t.nb[1] == f.nb[1] && t.nb[2] == f.nb[2];
                break;
            case BV::INDEX:
            case BV::TOKENS: ok = t.data == nullptr && t.nelements() == 1; break;
            case BV::MASK: break;
        }
        if (!ok) fail(x, "a view that is not the identity on one token's values");
        bv[x.id] = src;
    }

    void get_rows(const NodeSpec &x) {
        const TD tab = p.src_of(x.src[0]);
        if ((tab.type != T_F32 && tab.type != T_F16) || tab.ne[2] != 1 || tab.ne[3] != 1)
            fail(x, "needs an f32 / f16 embedding table");
        index_role(x, x.src[1], tok_param, "token");
        TD idx;
        idx.type = T_I32;
        idx.ne[0] = n;
        set_contiguous(idx);
        idx.data = (char *)rt.tok;
        TD y = alloc_rows(tab.ne[0]);
        p.add("get_rows", x.id, {tab, idx, y}, [](cudaStream_t st, const std::vector<TD> &t) { k::get_rows(t[0], t[1], t[2], st); },
              (double)(n * tab.ne[0] * 8));
        bv[x.id] = as_rows(y, tab.ne[0]);
    }

    void flash(const NodeSpec &x) {
        if (x.src.size() != 4 || get(x, x.src[3]).kind != BV::MASK)
            fail(x, "needs the stage's mask input (each sequence's causal row replaces it)");
        const auto &qn = *spec_ne.at(x.src[0]);
        const int64_t D = qn[0], H = qn[2];
        if (qn[1] != 1 || qn[3] != 1) fail(x, "needs one query row");
        const BV q = rows(x, x.src[0], D * H);
        const BV kc = cache(x, x.src[1]), vc = cache(x, x.src[2]);
        const int64_t Hkv = kc.td.ne[2];
        if (kc.td.ne[0] != D || vc.td.ne[0] != D || vc.td.ne[2] != Hkv || H % Hkv || kc.td.ne[1] < window)
            fail(x, "query and K/V heads do not line up");
        TD qt = q.td;
        qt.ne[0] = D, qt.ne[1] = 1, qt.ne[2] = H, qt.ne[3] = n;
        qt.nb[0] = 4, qt.nb[1] = 4 * D * H, qt.nb[2] = 4 * D, qt.nb[3] = 4 * D * H;
        auto kv = [&](const BV &c) {
            TD t = c.td;
            t.ne[1] = window;
            t.ne[3] = n;
            t.nb[3] = c.slot;
            return t;
        };
        TD kt = kv(kc), vt = kv(vc);
        TD mk;
        mk.type = T_F16;
        mk.ne[0] = window, mk.ne[3] = n;
        mk.nb[0] = 2, mk.nb[1] = mk.nb[2] = mk.nb[3] = 2 * window;
        mk.data = (char *)rt.mask;
        const int64_t ne[4] = {D, H, 1, n};
        TD y = p.alloc(T_F32, ne);
        if (!k::flash_split_ok(qt)) fail(x, "head size must be a multiple of 32 up to 256");
        TD scratch;
        p.scratch_marker(k::flash_split_scratch_bytes(qt, kt), &scratch);
        int *cnt = m.counters("batch/" + s.name + "/" + x.id + "/" + std::to_string(n) + "/" + std::to_string(window),
                              k::flash_split_counters(qt, kt));
        int *err = m.d_err;
        const float scale = x.pfloat("scale");
        const bool cluster = k::flash_split_prepare(qt, kt, vt, y);
        auto tr = p.trace_slot("flash_attn", x.id, cluster ? (size_t)(((window + 63) / 64) * Hkv * n) : k::flash_split_ctas(qt, kt));
        // the QKV launch before writes row pos[i] of slot i: the other rows are copied early
        const int32_t *kv_pos = cluster && m.attn_overlap ? rt.pos : nullptr;
        const bool *direct = &m.direct_launch;
        p.add("flash_attn", x.id, {qt, kt, vt, mk, y, scratch},
              [scale, cnt, err, tr, kv_pos, direct](cudaStream_t st, const std::vector<TD> &t) {
                  k::flash_attn_split(t[0], t[1], t[2], &t[3], t[4], scale, t[5].data, cnt, err, st, *tr, nullptr,
                                      *direct ? nullptr : kv_pos);
              },
              (double)n * ((double)window * Hkv * D * 4 + (double)D * H * 8));
        p.psteps.back().attn_early = kv_pos != nullptr;
        bv[x.id] = as_rows(y, D * H);
    }

    void argmax(const NodeSpec &x, const std::string &src) {
        const BV v = rows(x, src, 0);
        TD xt = v.td;
        xt.ne[0] = v.width, xt.ne[1] = n, xt.ne[2] = xt.ne[3] = 1;
        xt.nb[1] = 4 * v.width, xt.nb[2] = xt.nb[3] = 4 * v.width * n;
        TD y;
        y.type = T_I32;
        y.ne[0] = n;
        set_contiguous(y);
        y.data = (char *)rt.next;
        if (const int parts = k::argmax_split_parts(xt)) {
            TD scratch;
            p.scratch_marker((size_t)n * parts * 8, &scratch);
            int *cnt = m.counters("batch/argmax/" + std::to_string(n), (size_t)n);
            p.add("argmax", x.id, {xt, y, scratch},
                  [cnt](cudaStream_t st, const std::vector<TD> &t) { k::argmax_split(t[0], t[1], t[2].data, cnt, st); },
                  (double)(xt.nelements() * 4));
        } else {
            p.add("argmax", x.id, {xt, y}, [](cudaStream_t st, const std::vector<TD> &t) { k::argmax(t[0], t[1], st); },
                  (double)(xt.nelements() * 4));
        }
        BV r;
        r.kind = BV::TOKENS;
        r.td = y;
        bv[x.id] = r;
    }

    // Two or more rows: one launch quantizes them (normed for norm_w) into the staging layout the
    // GEMV then copies (PRO_Q8), instead of every CTA of the GEMV repeating that work. Returns the
    // staging buffer, or an empty descriptor for one row (the GEMV's own prologue does it).
    TD stage_rows(const std::string &node, const TD &x, const TD *nw, float eps, int64_t K, int r0, int r1) {
        TD act;
        if (r1 - r0 < 2) return act;
        p.scratch_marker(act_bytes(r1 - r0, K), &act);
        std::vector<TD> tds = {x, act};
        if (nw) tds.push_back(*nw);
        const bool norm = nw != nullptr;
        p.add("act_rows", node, tds,
              [=](cudaStream_t st, const std::vector<TD> &td) {
                  FusedArgs a;
                  a.pro = norm ? PRO_NORM : PRO_ACT;
                  a.x = (const float *)td[0].data + (int64_t)r0 * K;
                  a.ldx = K;
                  a.M = r1 - r0;
                  a.K = K;
                  if (norm) a.norm_w = (const float *)td[2].data;
                  a.eps = eps;
                  k::act_rows(a, td[1].data, st);
              },
              (double)(r1 - r0) * K * 5.25);
        return act;
    }

    // The row chunks of one fused GEMV: [r0, r1) with at most GEMV rows each.
    template <class F>
    void chunks(F &&f) {
        for (int r0 = 0; r0 < n; r0 += 8) f(r0, std::min(n, r0 + 8));
    }

    void group(const NodeSpec &x, const GroupDesc &g) {
        switch (g.kind) {
            case GroupDesc::QKV: {
                const BV xr = rows(x, g.x, g.d);
                const TD nw = p.src_of(g.norm_w), tq = p.src_of(g.w[0]), tk = p.src_of(g.w[1]), tv = p.src_of(g.w[2]);
                index_role(x, g.pos, pos_param, "position");
                const BV kc = cache(x, g.kc), vc = cache(x, g.vc);
                if (kc.td.nb[1] != vc.td.nb[1] || kc.td.nb[2] != vc.td.nb[2] || kc.td.ne[1] != vc.td.ne[1] || kc.slot != vc.slot)
                    fail(x, "K and V caches of different layouts");
                const int64_t D = g.D, H = g.H, Hkv = g.Hkv, d = g.d;
                TD qb = alloc_rows(H * D);
                int64_t npos = 0;
                const float *table = m.rope_table((int)D, g.base, 1.0f, 1.0f, "-", nullptr, &npos);
                const float theta_scale = ::powf(g.base, -2.0f / (float)D);
                const float eps = g.eps;
                int *err = m.d_err;
                const int32_t *pos = rt.pos;
                char *kb = kc.td.data, *vb = vc.td.data;
                const int64_t nb1 = kc.td.nb[1], nb2 = kc.td.nb[2], crows = kc.td.ne[1], slot = kc.slot;
                const char *kind = tq.type == T_Q4_0 ? "gemv_q4_0_qkv" : "gemv_q8_0_qkv";
                chunks([&](int r0, int r1) {
                    const double bytes = qweight_bytes(tq) + qweight_bytes(tk) + qweight_bytes(tv) + 4.0 * d * (r1 - r0);
                    const TD act = stage_rows(g.out[0], xr.td, &nw, eps, d, r0, r1);
                    const bool staged = act.sid >= 0;
                    p.add_gemv(kind, g.out[0], {xr.td, nw, tq, tk, tv, qb, act},
                               [=](const std::vector<TD> &td) {
                                   FusedArgs a;
                                   a.pro = staged ? PRO_Q8 : PRO_NORM;
                                   a.xq = staged ? td[6].data : nullptr;
                                   a.map = MAP_ROPE_QKV;
                                   a.x = (const float *)td[0].data + (int64_t)r0 * d;
                                   a.ldx = d;
                                   a.M = r1 - r0;
                                   a.K = d;
                                   a.norm_w = (const float *)td[1].data;
                                   a.eps = eps;
                                   put_weight(a, 0, td[2]);
                                   put_weight(a, 1, td[3]);
                                   put_weight(a, 2, td[4]);
                                   a.pos = pos + r0;
                                   a.kcache = kb + (int64_t)r0 * slot;
                                   a.vcache = vb + (int64_t)r0 * slot;
                                   a.cache_nb1 = nb1;
                                   a.cache_nb2 = nb2;
                                   a.cache_nb3 = slot;
                                   a.cache_rows = crows;
                                   a.q_out = (float *)td[5].data + (int64_t)r0 * H * D;
                                   a.ldq = H * D;
                                   a.D = D;
                                   a.H = H;
                                   a.Hkv = Hkv;
                                   a.table = table;
                                   a.npos = npos;
                                   a.theta_scale = theta_scale;
                                   a.err = err;
                                   return a;
                               },
                               bytes);
                });
                bv[g.out[0]] = as_rows(qb, H * D);
                bv[g.out[1]] = kc;
                bv[g.out[2]] = vc;
                break;
            }
            case GroupDesc::GLU:
            case GroupDesc::HEAD: {
                const BV xr = rows(x, g.x, g.d);
                const TD nw = p.src_of(g.norm_w), w0 = p.src_of(g.w[0]);
                const bool glu = g.kind == GroupDesc::GLU;
                const TD w1 = glu ? p.src_of(g.w[1]) : w0;
                const int64_t d = g.d, N = g.N;
                TD out;
                if (!glu) {  // the output head: its rows are the step's logits
                    if (head_done) fail(x, "a second output head");
                    head_done = true;
                    if (!rt.logits_buf.size()) {
                        rt.vocab = N;
                        rt.logits_buf.alloc((size_t)BatchRuntime::kMaxSeq * (size_t)N * 4);
                    }
                    if (rt.vocab != N) fail(x, "an output head of " + std::to_string(N) + " rows; the logits rows hold " +
                                                   std::to_string(rt.vocab));
                    out.type = T_F32;
                    out.ne[0] = N, out.ne[1] = n;
                    set_contiguous(out);
                    out.data = (char *)rt.logits_buf.get();
                } else {
                    out = alloc_rows(N);
                }
                const float eps = g.eps;
                const char *kind = glu ? (w0.type == T_Q4_0 ? "gemv_q4_0_glu" : "gemv_q8_0_glu")
                                       : (w0.type == T_Q4_0 ? "gemv_q4_0_head" : "gemv_q8_0_head");
                chunks([&](int r0, int r1) {
                    const double bytes = qweight_bytes(w0) + (glu ? qweight_bytes(w1) : 0.0) + 4.0 * (d + N) * (r1 - r0);
                    const TD act = stage_rows(g.out[0], xr.td, &nw, eps, d, r0, r1);
                    const bool staged = act.sid >= 0;
                    std::vector<TD> tds = {xr.td, nw, w0, glu ? w1 : w0, out, act};
                    p.add_gemv(kind, g.out[0], tds,
                               [=](const std::vector<TD> &td) {
                                   FusedArgs a;
                                   a.pro = staged ? PRO_Q8 : PRO_NORM;
                                   a.xq = staged ? td[5].data : nullptr;
                                   a.map = glu ? MAP_SWIGLU : MAP_SINGLE;
                                   a.x = (const float *)td[0].data + (int64_t)r0 * d;
                                   a.ldx = d;
                                   a.M = r1 - r0;
                                   a.K = d;
                                   a.norm_w = (const float *)td[1].data;
                                   a.eps = eps;
                                   put_weight(a, 0, td[2]);
                                   if (glu) put_weight(a, 1, td[3]);
                                   a.out = (float *)td[4].data + (int64_t)r0 * N;
                                   a.ldo = N;
                                   return a;
                               },
                               bytes);
                });
                bv[g.out[0]] = as_rows(out, N);
                break;
            }
            case GroupDesc::RESID: {
                const BV xr = rows(x, g.x, g.d), res = rows(x, g.res, g.N);
                const TD w = p.src_of(g.w[0]);
                const int64_t K = g.d, N = g.N;
                TD out = alloc_rows(N);
                const char *kind = w.type == T_Q4_0 ? "gemv_q4_0_res" : "gemv_q8_0_res";
                chunks([&](int r0, int r1) {
                    const TD act = stage_rows(g.out[0], xr.td, nullptr, 0.0f, K, r0, r1);
                    const bool staged = act.sid >= 0;
                    p.add_gemv(kind, g.out[0], {xr.td, res.td, w, out, act},
                               [=](const std::vector<TD> &td) {
                                   FusedArgs a;
                                   a.pro = staged ? PRO_Q8 : PRO_ACT;
                                   a.xq = staged ? td[4].data : nullptr;
                                   a.map = MAP_SINGLE;
                                   a.x = (const float *)td[0].data + (int64_t)r0 * K;
                                   a.ldx = K;
                                   a.M = r1 - r0;
                                   a.K = K;
                                   put_weight(a, 0, td[2]);
                                   a.res = (const float *)td[1].data + (int64_t)r0 * N;
                                   a.ldr = N;
                                   a.out = (float *)td[3].data + (int64_t)r0 * N;
                                   a.ldo = N;
                                   return a;
                               },
                               qweight_bytes(w) + 4.0 * (K + 2 * N) * (r1 - r0));
                });
                bv[g.out[0]] = as_rows(out, N);
                break;
            }
        }
    }

    void plan(const FusionPlan &fp) {
        params();
        for (const NodeSpec &x : s.nodes) {
            spec_ne[x.id] = &x.ne;
            spec_type[x.id] = x.type;
        }
        {
            BatchRuntime *r = &rt;
            const int nn = n;
            const int64_t w = window;
            p.cur = 0;
            p.add("batch_mask", "mask", {}, [r, nn, w](cudaStream_t st, const std::vector<TD> &) { k::batch_mask(r->mask, r->pos, nn, w, st); },
                  (double)(nn * w * 2));
        }
        for (size_t i = 0; i < s.nodes.size(); i++) {
            const NodeSpec &x = s.nodes[i];
            p.cur = (int)i;
            if (fp.covered(i)) {
                const FusionGroup &g = fp.groups[(size_t)fp.group_of[i]];
                if (g.anchor != i) continue;
                if (!g.desc) fail(x, "fused group without a batched form");
                group(x, *g.desc);
                continue;
            }
            if (is_view(x.op)) {
                view(x);
            } else if (x.op == "get_rows") {
                get_rows(x);
            } else if (x.op == "clamp" || x.op == "cast" || x.op == "scale") {
                if (get(x, x.src[0]).kind != BV::MASK) fail(x, "only the mask input's conversions are dropped in a batched step");
                const BV v = bv.at(x.src[0]);
                bv[x.id] = v;
            } else if (x.op == "flash_attn") {
                flash(x);
            } else if (x.op == "argmax") {
                argmax(x, x.src[0]);
            } else {
                fail(x, "not part of a fused group: the batched step runs only the fused decode layer");
            }
        }
        if (s.outputs.empty()) throw std::runtime_error("batched decode: stage '" + s.name + "' returns nothing");
        p.cur = (int)s.nodes.size();
        if (!bv.count(s.outputs[0])) throw std::runtime_error("batched decode: stage '" + s.name + "' has no result");
        const BV out0 = bv.at(s.outputs[0]);
        if (out0.kind == BV::ROWS) {
            if (out0.td.data != (char *)rt.logits_buf.get())
                throw std::runtime_error("batched decode: stage '" + s.name + "' returns rows other than the output head's");
            NodeSpec fake_node;
            fake_node.id = "next";
            fake_node.op = "argmax";
            argmax(fake_node, s.outputs[0]);
        } else if (out0.kind != BV::TOKENS) {
            throw std::runtime_error("batched decode: stage '" + s.name + "' returns neither logits nor a greedy token");
        }
        for (size_t i = 1; i < s.outputs.size(); i++)
            if (!bv.count(s.outputs[i]) || bv.at(s.outputs[i]).kind != BV::CACHE)
                throw std::runtime_error("batched decode: stage '" + s.name + "' returns a value other than its caches");
        if (tok_param.empty() || pos_param.empty())
            throw std::runtime_error("batched decode: stage '" + s.name + "' has no token or no position input");
    }
};

int64_t slot_bytes_of(const Value &v) { return (int64_t)((v.td.nbytes() + 255) / 256 * 256); }

}  // namespace

void Model::seq_slots(int n) {
    if (n < 1 || n > BatchRuntime::kMaxSeq)
        throw std::runtime_error("sequence slots: n must be 1.." + std::to_string(BatchRuntime::kMaxSeq));
    if (tp.active()) throw std::runtime_error("sequence slots: not with tensor parallelism");
    if (prog.state.empty()) throw std::runtime_error("sequence slots: the program has no state values");
    cuda_check(cudaSetDevice(device), "cudaSetDevice");
    cuda_check(cudaStreamSynchronize(stream), "sequence slots");
    batch.reset();  // plans point into the old slots
    auto rt = std::make_unique<BatchRuntime>();
    rt->n_seq = n;
    int64_t rows = 0;
    for (const auto &name : prog.state) {
        const Value &v = values.at(name);
        rt->slots[name].alloc((size_t)slot_bytes_of(v) * (size_t)n);
        const int64_t r = v.td.ne[1];
        rows = rows == 0 ? r : std::min(rows, r);
    }
    rt->max_window = rows;
    const size_t ints = 4 * BatchRuntime::kMaxSeq * sizeof(int32_t);
    rt->io.alloc(ints + (size_t)BatchRuntime::kMaxSeq * (size_t)rows * 2);
    rt->tok = (int32_t *)rt->io.get();
    rt->pos = rt->tok + BatchRuntime::kMaxSeq;
    rt->next = rt->pos + BatchRuntime::kMaxSeq;
    rt->step = rt->next + BatchRuntime::kMaxSeq;
    rt->mask = (__half *)(rt->io.get() + ints);
    batch = std::move(rt);
}

void Model::seq_copy(int dst, int src) {
    if (!batch) throw std::runtime_error("sequence slots: call seq_slots first");
    const int n = batch->n_seq;
    if (dst < -1 || dst >= n || src < -1 || src >= n)
        throw std::runtime_error("sequence slots: slot out of range (-1 is the model's own state, 0.." + std::to_string(n - 1) +
                                 " the slots)");
    if (dst == src) return;
    cuda_check(cudaSetDevice(device), "cudaSetDevice");
    for (const auto &name : prog.state) {
        Value &v = values.at(name);
        const size_t bytes = v.td.nbytes(), sb = (size_t)slot_bytes_of(v);
        char *slots = batch->slots.at(name).get();
        char *to = dst < 0 ? v.buf.get() : slots + sb * (size_t)dst;
        const char *from = src < 0 ? v.buf.get() : slots + sb * (size_t)src;
        cuda_check(cudaMemcpyAsync(to, from, bytes, cudaMemcpyDeviceToDevice, stream), "sequence slot copy");
    }
    cuda_check(cudaStreamSynchronize(stream), "sequence slot copy");
}

BatchRuntime::Plan &Model::batch_plan(const std::string &entry, int n, int64_t window) {
    BatchRuntime &rt = *batch;
    rt.clock++;
    for (auto &pl : rt.plans)
        if (pl.entry == entry && pl.n == n && pl.window == window) {
            pl.last_use = rt.clock;
            return pl;
        }
    // the entry's single stage call
    const Entry *e = nullptr;
    for (const auto &en : entries)
        if (en.spec->name == entry) e = &en;
    if (!e) throw std::runtime_error("no entry point named '" + entry + "'");
    if (e->spec->driver.size() != 1 || e->spec->driver[0].is_loop)
        throw std::runtime_error("batched decode: entry '" + entry + "' is not a single stage call");
    const DriverStep &d = e->spec->driver[0];
    const CallSite &site = calls[(size_t)d.call_site];
    const StageSpec &s = *site.stage;
    rebind();
    if (rt.plans.size() >= BatchRuntime::kMaxPlans) {
        auto lru = std::min_element(rt.plans.begin(), rt.plans.end(),
                                    [](const BatchRuntime::Plan &a, const BatchRuntime::Plan &b) { return a.last_use < b.last_use; });
        cuda_check(cudaStreamSynchronize(stream), "batched plan");
        rt.plans.erase(lru);
    }
    BatchRuntime::Plan pl;
    pl.entry = entry;
    pl.n = n;
    pl.window = window;
    pl.site = std::make_unique<SitePlan>();
    Planner p(*this, *pl.site, site);
    p.copy_results = false;
    const FusionPlan fp = find_fusions(*this, s, p);
    BatchPlanner bp(*this, rt, p, s, d, n, window);
    bp.plan(fp);
    p.finish();
    pl.last_use = rt.clock;
    rt.plans.push_back(std::move(pl));
    return rt.plans.back();
}

void Model::batch_launch(SitePlan &p) {
    direct_launch = profiling || !use_graphs;
    if (profiling) {  // each launch on its own, timed (ggml_compiler_b200_set_profiling)
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
            KernelStat &ks = kstats[std::string("batch_") + st.kind];
            ks.ms += ms;
            ks.bytes += st.bytes;
            ks.launches++;
        }
        return;
    }
    if (!use_graphs) {
        for (const auto &st : p.steps) st.run(stream);
        return;
    }
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
}

void Model::batch_check_error(const char *what) {
    int err = 0;
    cuda_check(cudaMemcpy(&err, d_err, sizeof err, cudaMemcpyDeviceToHost), "error word");
    if (!err) return;
    cudaMemset(d_err, 0, sizeof(int));
    if (err == 2) throw std::runtime_error(std::string(what) + ": a kernel's pipeline wait timed out (results are invalid)");
    throw std::runtime_error(std::string(what) + ": a K/V row index was outside its cache (row skipped)");
}

namespace {

// The attention window of a step whose largest position is `top`: keys up to `top`, in steps of 256
// rows (so a plan serves 256 positions), at most the cache's rows.
int64_t window_for(int64_t top, int64_t max_window) { return std::min(max_window, (top + 1 + 255) / 256 * 256); }

void check_positions(const BatchRuntime &rt, int n, const int32_t *pos, int extra) {
    for (int i = 0; i < n; i++)
        if (pos[i] < 0 || (int64_t)pos[i] + extra >= rt.max_window)
            throw std::runtime_error("batched decode: position " + std::to_string((int64_t)pos[i] + extra) + " of sequence " +
                                     std::to_string(i) + " is outside the KV cache (" + std::to_string(rt.max_window) + " rows)");
}

}  // namespace

void Model::decode_batch(const std::string &entry, int n, const int32_t *tok, const int32_t *pos, float *logits, int32_t *next) {
    if (!batch) throw std::runtime_error("batched decode: call seq_slots first");
    if (n < 1 || n > batch->n_seq) throw std::runtime_error("batched decode: n must be 1.." + std::to_string(batch->n_seq));
    if (!tok || !pos) throw std::runtime_error("batched decode: NULL tokens or positions");
    check_positions(*batch, n, pos, 0);
    cuda_check(cudaSetDevice(device), "cudaSetDevice");
    const int64_t top = *std::max_element(pos, pos + n);
    BatchRuntime::Plan &pl = batch_plan(entry, n, window_for(top, batch->max_window));
    BatchRuntime &rt = *batch;
    if (!run_ev[0]) {
        cuda_check(cudaEventCreate(&run_ev[0]), "cudaEventCreate");
        cuda_check(cudaEventCreate(&run_ev[1]), "cudaEventCreate");
    }
    const auto t0 = std::chrono::steady_clock::now();
    cuda_check(cudaEventRecord(run_ev[0], stream), "cudaEventRecord");
    cuda_check(cudaMemcpyAsync(rt.tok, tok, sizeof(int32_t) * n, cudaMemcpyHostToDevice, stream), "tokens");
    cuda_check(cudaMemcpyAsync(rt.pos, pos, sizeof(int32_t) * n, cudaMemcpyHostToDevice, stream), "positions");
    batch_launch(*pl.site);
    if (logits)
        cuda_check(cudaMemcpyAsync(logits, rt.logits_buf.get(), sizeof(float) * (size_t)n * (size_t)rt.vocab,
                                   cudaMemcpyDeviceToHost, stream),
                   "logits");
    if (next) cuda_check(cudaMemcpyAsync(next, rt.next, sizeof(int32_t) * n, cudaMemcpyDeviceToHost, stream), "tokens");
    cuda_check(cudaEventRecord(run_ev[1], stream), "cudaEventRecord");
    cuda_check(cudaStreamSynchronize(stream), "batched decode");
    last_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    float dms = 0;
    cuda_check(cudaEventElapsedTime(&dms, run_ev[0], run_ev[1]), "cudaEventElapsedTime");
    last_device_ms = dms;
    batch_check_error("batched decode");
    if (!trace_path.empty()) write_trace();
}

void Model::generate_batch(const std::string &entry, int n, const int32_t *first, const int32_t *start, int steps,
                           int32_t *out) {
    if (!batch) throw std::runtime_error("batched decode: call seq_slots first");
    if (n < 1 || n > batch->n_seq) throw std::runtime_error("batched decode: n must be 1.." + std::to_string(batch->n_seq));
    if (!first || !start || steps < 1) throw std::runtime_error("batched decode: NULL inputs or no steps");
    check_positions(*batch, n, start, steps - 1);
    cuda_check(cudaSetDevice(device), "cudaSetDevice");
    BatchRuntime &rt = *batch;
    const int64_t top = *std::max_element(start, start + n);
    // plans for every window the steps reach, made before the timed region
    if (window_for(top + steps - 1, rt.max_window) / 256 - window_for(top, rt.max_window) / 256 >= (int64_t)BatchRuntime::kMaxPlans)
        throw std::runtime_error("batched decode: the steps cross more attention windows than plans are kept; run fewer steps per call");
    std::vector<SitePlan *> plan_of((size_t)steps);
    for (int s = 0; s < steps; s++) {
        const int64_t w = window_for(top + s, rt.max_window);
        plan_of[(size_t)s] = s > 0 && window_for(top + s - 1, rt.max_window) == w ? plan_of[(size_t)s - 1]
                                                                                  : batch_plan(entry, n, w).site.get();
    }
    const size_t gen_bytes = sizeof(int32_t) * (size_t)steps * (size_t)n;
    if (rt.gen.size() < gen_bytes) {
        cuda_check(cudaStreamSynchronize(stream), "generated tokens");
        rt.gen.alloc(gen_bytes);
    }
    if (!run_ev[0]) {
        cuda_check(cudaEventCreate(&run_ev[0]), "cudaEventCreate");
        cuda_check(cudaEventCreate(&run_ev[1]), "cudaEventCreate");
    }
    const auto t0 = std::chrono::steady_clock::now();
    cuda_check(cudaEventRecord(run_ev[0], stream), "cudaEventRecord");
    cuda_check(cudaMemcpyAsync(rt.tok, first, sizeof(int32_t) * n, cudaMemcpyHostToDevice, stream), "tokens");
    cuda_check(cudaMemcpyAsync(rt.pos, start, sizeof(int32_t) * n, cudaMemcpyHostToDevice, stream), "positions");
    cuda_check(cudaMemsetAsync(rt.step, 0, sizeof(int32_t), stream), "step");
    for (int s = 0; s < steps; s++) {
        batch_launch(*plan_of[(size_t)s]);
        k::batch_advance(rt.tok, rt.pos, rt.next, (int32_t *)rt.gen.get(), rt.step, n, stream);
    }
    if (out) cuda_check(cudaMemcpyAsync(out, rt.gen.get(), gen_bytes, cudaMemcpyDeviceToHost, stream), "generated tokens");
    cuda_check(cudaEventRecord(run_ev[1], stream), "cudaEventRecord");
    cuda_check(cudaStreamSynchronize(stream), "batched generate");
    last_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    float dms = 0;
    cuda_check(cudaEventElapsedTime(&dms, run_ev[0], run_ev[1]), "cudaEventElapsedTime");
    last_device_ms = dms;
    batch_check_error("batched generate");
    if (!trace_path.empty()) write_trace();
}

}  // namespace gcb
