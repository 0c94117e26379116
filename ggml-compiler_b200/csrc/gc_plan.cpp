// Call-site planning: a stage's node list -> kernel launches for the current binding.
//
// The op table mirrors the reference's dispatcher (runtime/src/ops.cpp:74-351) for the ops that
// language-model programs use, with the same preconditions and the same "produced shape / type"
// check per node (ops.cpp:355-378). Views (view, reshape, permute) are pure stride arithmetic, as
// the reference's ggml views are (runtime/include/ggml_compiler_ops.h:69-107). Every other node gets
// a kernel; its output lives in the call site's arena, packed by liveness. Stage results are
// copied into their driver values after every other launch, except a result that already is that
// value's memory (set_rows into a state value: the reference skips that copy too,
// ggml_compiler_rt.cpp:703-708).
//
// Fused decode/prefill kernels replace node groups here as well (gc_fuse.cpp).
#include <algorithm>
#include <cstring>
#include <map>
#include <set>
#include <sstream>
#include <stdexcept>
#include <unordered_map>

#include "gc_fuse.h"
#include "gc_fused.h"
#include "gc_model.h"
#include "kernels/gc_qweight.cuh"

namespace gcb {

namespace {

std::string shape_str(const int64_t *ne) {
    std::ostringstream os;
    os << "[" << ne[0] << ", " << ne[1] << ", " << ne[2] << ", " << ne[3] << "]";
    return os.str();
}

[[noreturn]] void fail(const NodeSpec &n, const std::string &msg) { throw std::runtime_error(n.where() + ": " + msg); }

void need_src(const NodeSpec &n, const std::vector<TD> &s, size_t lo, size_t hi) {
    if (s.size() < lo || s.size() > hi)
        fail(n, "expected " + std::to_string(lo) + (lo == hi ? "" : "-" + std::to_string(hi)) + " inputs, got " +
                    std::to_string(s.size()));
}

bool can_repeat(const TD &b, const TD &a) {
    for (int i = 0; i < 4; i++)
        if (b.ne[i] == 0 || a.ne[i] % b.ne[i] != 0) return false;
    return true;
}

bool same_shape(const TD &a, const TD &b) {
    for (int i = 0; i < 4; i++)
        if (a.ne[i] != b.ne[i]) return false;
    return true;
}

bool is_quant(Type t) { return t == T_Q4_0 || t == T_Q8_0; }

const std::map<std::string, int> &unary_ops() {
    static const std::map<std::string, int> m = {
        {"silu", k::SILU}, {"neg", k::NEG},   {"abs", k::ABS},         {"sqr", k::SQR},           {"sqrt", k::SQRT},
        {"exp", k::EXP},   {"log", k::LOG},   {"relu", k::RELU},       {"tanh", k::TANH},         {"sigmoid", k::SIGMOID},
        {"step", k::STEP}, {"sin", k::SIN},   {"cos", k::COS},         {"softplus", k::SOFTPLUS}, {"gelu", k::GELU_TANH},
        {"gelu_tanh", k::GELU_TANH},          {"gelu_erf", k::GELU_ERF},
    };
    return m;
}

}  // namespace

Planner::Planner(Model &m, SitePlan &plan, const CallSite &site) : m(m), plan(plan), d(*site.step), s(*site.stage) {}

TD Planner::alloc(Type t, const int64_t *ne) {
    TD o;
    o.type = t;
    for (int i = 0; i < 4; i++) o.ne[i] = ne[i];
    set_contiguous(o);
    Storage st;
    st.bytes = std::max<size_t>(o.nbytes(), 4);
    st.first = st.last = cur;
    storages.push_back(st);
    o.sid = (int)storages.size() - 1;
    return o;
}

void *Planner::scratch_marker(size_t bytes, TD *out) {
    int64_t ne[4] = {(int64_t)((bytes + 3) / 4), 1, 1, 1};
    *out = alloc(T_F32, ne);
    return nullptr;
}

void Planner::use(const TD &t) {
    if (t.sid >= 0) storages[(size_t)t.sid].last = std::max(storages[(size_t)t.sid].last, cur);
}

void Planner::add(const char *kind, const std::string &node, std::vector<TD> tds,
                  std::function<void(cudaStream_t, const std::vector<TD> &)> fn, double bytes) {
    for (const auto &t : tds) use(t);
    psteps.push_back(PlanStep{kind, node, std::move(tds), std::move(fn), bytes});
}

void Planner::add_gemv(const char *kind, const std::string &node, std::vector<TD> tds,
                       std::function<FusedArgs(const std::vector<TD> &)> build, double bytes) {
    int shard = 0, nshard = 1;
    std::vector<int64_t> col;
    TD out;
    int64_t rows = 0, ld = 0;
    if (m.tp.active()) {
        // the geometry of the arguments does not depend on where the arena puts the tensors
        const FusedArgs g = build(tds);
        const int W = m.tp.world;
        if (g.map == MAP_ROPE_QKV) {
            if (g.H % W == 0 && g.Hkv % W == 0) {
                shard = m.tp.rank, nshard = W;
                head_sharded.insert(tds.back().sid);
                bytes /= W;
            }
        } else {
            const int64_t N = g.wrows[0], tiles = (N + QTR - 1) / QTR;
            out = tds.back();
            rows = g.M, ld = g.ldo * 4;
            col.resize((size_t)W + 1);
            for (int r = 0; r <= W; r++) col[(size_t)r] = std::min<int64_t>(N, tiles * r / W * QTR) * 4;
            if (tiles >= W && exchange_fits(rows, ld, col) && out.off % 16 == 0) {
                shard = m.tp.rank, nshard = W;
                bytes *= (double)(col[(size_t)shard + 1] - col[(size_t)shard]) / (double)col.back();
            }
        }
    }
    auto b2 = [build, shard, nshard](const std::vector<TD> &t) {
        FusedArgs a = build(t);
        a.shard = shard;
        a.nshard = nshard;
        return a;
    };
    auto pf = std::make_shared<GemvExtras>();
    auto tr = trace_slot(kind, node, (size_t)(2 * k::num_sms()));
    add(kind, node, std::move(tds),
        [b2, pf, tr](cudaStream_t st, const std::vector<TD> &t) {
            FusedArgs a = b2(t);
            for (int r = 0; r < 3; r++) {
                a.pf[r] = pf->p[r];
                a.pf_bytes[r] = pf->n[r];
            }
            a.stream_evict_first = pf->evict_first;
            a.trace = *tr;
            if (pf->xq) {
                a.pro = PRO_Q8;
                a.xq = pf->xq;
            }
            a.act_mode = pf->act_mode;
            a.act_out = pf->act_out;
            a.act_norm_w = pf->act_norm_w;
            a.act_eps = pf->act_eps;
            a.act_cnt = pf->act_cnt;
            a.hold_pieces = pf->hold_pieces;
            a.producer_waits = pf->producer_waits;
            if (pf->max_ctas) a.max_ctas = pf->max_ctas;
            k::fused_gemv(a, st, pf->producer_waits < 2);
        },
        bytes);
    psteps.back().gemv = b2;
    psteps.back().pf = pf;
    if (nshard > 1 && !col.empty()) add_exchange(node, out, rows, ld, col);
}

std::shared_ptr<uint64_t *> Planner::trace_slot(const char *kind, const std::string &node, size_t ctas) {
    auto slot = std::make_shared<uint64_t *>(nullptr);
    if (!m.trace_path.empty()) traces.push_back({kind, node, ctas, slot});
    return slot;
}

k::TpExchange Planner::exchange_args(int64_t rows, int64_t ld, const std::vector<int64_t> &col) const {
    k::TpExchange x;
    x.rank = m.tp.rank;
    x.world = m.tp.world;
    x.rows = rows;
    x.ld = ld;
    x.row_bytes = col.back();
    for (size_t r = 0; r < col.size() && r <= (size_t)k::TP_MAX; r++) x.col[r] = col[r];
    for (int r = 0; r < x.world; r++) x.win[r] = m.tp.win[(size_t)r];
    x.slot_bytes = (int64_t)m.tp.slot_bytes;
    x.seq = (unsigned *)m.tp.seq.get();
    x.done = (unsigned *)m.tp.done.get();
    x.err = m.d_err;
    x.timeout_ns = m.tp.timeout_ns;
    return x;
}

bool Planner::exchange_fits(int64_t rows, int64_t ld, const std::vector<int64_t> &col) const {
    return (int)col.size() == m.tp.world + 1 && k::tp_exchange_ok(exchange_args(rows, ld, col));
}

bool Planner::add_exchange(const std::string &node, const TD &buf, int64_t rows, int64_t ld, const std::vector<int64_t> &col) {
    if (!exchange_fits(rows, ld, col) || (buf.sid >= 0 ? buf.off : (size_t)(uintptr_t)buf.data) % 16) return false;
    const k::TpExchange x = exchange_args(rows, ld, col);
    add("tp_exchange", node, {buf}, [x](cudaStream_t st, const std::vector<TD> &t) {
            k::TpExchange y = x;
            y.buf = t[0].data;
            k::tp_exchange(y, st);
        },
        (double)(rows * x.row_bytes));
    return true;
}

TD Planner::src_of(const std::string &name) {
    auto it = env.find(name);
    if (it != env.end()) return it->second;
    auto w = m.weights.find(name);
    if (w == m.weights.end()) throw std::runtime_error("stage '" + s.name + "' reads unknown tensor '" + name + "'");
    return w->second.td;
}

// ------------------------------------------------------------------------------------------------

TD Planner::plan_node(const NodeSpec &n, const std::vector<TD> &sv) {
    const std::string &op = n.op;
    auto out_like = [&](Type t, const int64_t *ne) { return alloc(t, ne); };

    if (op == "reshape") {
        need_src(n, sv, 1, 1);
        const TD &x = sv[0];
        if (x.nelements() != n.ne[0] * n.ne[1] * n.ne[2] * n.ne[3])
            fail(n, "cannot reshape " + shape_str(x.ne) + " to " + shape_str(n.ne.data()));
        TD y = x;
        for (int i = 0; i < 4; i++) y.ne[i] = n.ne[i];
        if (is_quant(x.type)) {
            if (n.ne[0] != x.ne[0] || !x.contiguous()) fail(n, "a quantized tensor can only be reshaped row for row");
            set_contiguous(y);
            return y;
        }
        if (x.contiguous()) {
            set_contiguous(y);
            return y;
        }
        // a strided view may only gain or lose size-1 dims (ggml_compiler_ops.h:85-107)
        int64_t nb[4] = {x.nb[0], 0, 0, 0};
        int k = 0;
        for (int i = 0; i < 4; i++) {
            if (n.ne[i] == 1) {
                if (i > 0) nb[i] = nb[i - 1] * n.ne[i - 1];
                continue;
            }
            while (k < 4 && x.ne[k] == 1) k++;
            if (k == 4 || x.ne[k] != n.ne[i])
                fail(n, "input is a strided view and the reshape does more than add or drop size-1 dims; it needs a cont first");
            nb[i] = x.nb[k++];
        }
        while (k < 4 && x.ne[k] == 1) k++;
        if (k != 4 || nb[0] != x.nb[0])
            fail(n, "input is a strided view and the reshape does more than add or drop size-1 dims; it needs a cont first");
        for (int i = 0; i < 4; i++) y.nb[i] = nb[i];
        return y;
    }
    if (op == "view") {
        need_src(n, sv, 1, 1);
        const TD &x = sv[0];
        const int dim = (int)n.pint("dim");
        const int64_t start = n.pint("start");
        if (dim < 0 || dim > 3 || start < 0 || start + n.ne[(size_t)dim] > x.ne[dim]) fail(n, "slice out of range of " + shape_str(x.ne));
        if (is_quant(x.type)) fail(n, "views of quantized tensors are not supported");
        TD y = x;
        for (int i = 0; i < 4; i++) y.ne[i] = n.ne[i];
        for (int i = 1; i < 4; i++)
            if (y.ne[i] == 1) y.nb[i] = y.nb[i - 1] * y.ne[i - 1];
        const size_t delta = (size_t)(start * x.nb[dim]);
        if (y.sid >= 0) y.off += delta;
        else y.data += delta;
        return y;
    }
    if (op == "permute") {
        need_src(n, sv, 1, 1);
        const Json &ax = n.p.at("axes");
        if (!ax.is_array() || ax.size() != 4) fail(n, "'axes' must have 4 entries");
        const TD &x = sv[0];
        TD y = x;
        for (int i = 0; i < 4; i++) {
            const int a = (int)ax[(size_t)i].as_int();
            if (a < 0 || a > 3) fail(n, "bad permute axes");
            y.ne[a] = x.ne[i];
            y.nb[a] = x.nb[i];
        }
        return y;
    }
    if (op == "cont" || op == "cast") {
        need_src(n, sv, 1, 1);
        const TD &x = sv[0];
        if (is_quant(x.type)) fail(n, "cannot copy a quantized tensor");
        const Type t = op == "cast" ? n.type : x.type;
        TD y = out_like(t, op == "cast" ? x.ne : n.ne.data());
        if (op == "cont" && x.nelements() != y.nelements()) fail(n, "cont changes the element count");
        add("copy", n.id, {x, y}, [](cudaStream_t st, const std::vector<TD> &t) { k::copy(t[0], t[1], st); },
            (double)(x.nelements() * (x.elsize() + y.elsize())));
        return y;
    }
    if (op == "add" || op == "sub" || op == "mul" || op == "div") {
        need_src(n, sv, 2, 2);
        const TD &a = sv[0], &b = sv[1];
        if (!can_repeat(b, a)) fail(n, "cannot broadcast " + shape_str(b.ne) + " into " + shape_str(a.ne));
        if (is_quant(a.type) || is_quant(b.type)) fail(n, "quantized operand");
        const int bop = op == "add" ? k::ADD : op == "sub" ? k::SUB : op == "mul" ? k::MUL : k::DIV;
        TD y = out_like(a.type, a.ne);
        add("binary", n.id, {a, b, y}, [bop](cudaStream_t st, const std::vector<TD> &t) { k::binary(bop, t[0], t[1], t[2], st); },
            (double)(a.nelements() * 12));
        return y;
    }
    auto un = unary_ops().find(op);
    if (un != unary_ops().end() || op == "scale" || op == "clamp") {
        need_src(n, sv, 1, 1);
        const TD &x = sv[0];
        if (is_quant(x.type)) fail(n, "quantized operand");
        int uop;
        float p0 = 0, p1 = 0;
        if (op == "scale") {
            uop = k::SCALE;
            p0 = n.pfloat("s");
            p1 = n.has("b") ? n.pfloat("b") : 0.0f;
        } else if (op == "clamp") {
            uop = k::CLAMP;
            p0 = n.pfloat("min");
            p1 = n.pfloat("max");
        } else {
            uop = un->second;
        }
        TD y = out_like(x.type, x.ne);
        add("unary", n.id, {x, y}, [uop, p0, p1](cudaStream_t st, const std::vector<TD> &t) { k::unary(uop, t[0], t[1], p0, p1, st); },
            (double)(x.nelements() * 8));
        return y;
    }
    if (op == "rms_norm" || op == "norm") {
        need_src(n, sv, 1, 1);
        const TD &x = sv[0];
        if (x.type != T_F32 || x.nb[0] != 4) fail(n, "needs an f32 input with contiguous rows");
        const float eps = n.pfloat("eps");
        TD y = out_like(T_F32, x.ne);
        if (op == "rms_norm")
            add("rms_norm", n.id, {x, y}, [eps](cudaStream_t st, const std::vector<TD> &t) { k::rms_norm(t[0], t[1], eps, st); },
                (double)(x.nelements() * 8));
        else
            add("norm", n.id, {x, y}, [eps](cudaStream_t st, const std::vector<TD> &t) { k::norm(t[0], t[1], eps, st); },
                (double)(x.nelements() * 8));
        return y;
    }
    if (op == "soft_max") {
        need_src(n, sv, 1, 2);
        const TD &x = sv[0];
        const float scale = n.has("scale") ? n.pfloat("scale") : 1.0f;
        if (n.has("max_bias") && n.pfloat("max_bias") != 0.0f) fail(n, "ALiBi (max_bias != 0) is not supported");
        if (x.type != T_F32 || x.nb[0] != 4) fail(n, "needs an f32 input with contiguous rows");
        TD y = out_like(T_F32, x.ne);
        if (sv.size() > 1) {
            const TD &mk = sv[1];
            if (mk.ne[0] != x.ne[0] || mk.ne[1] < x.ne[1] || x.ne[2] % mk.ne[2] || x.ne[3] % mk.ne[3])
                fail(n, "mask " + shape_str(mk.ne) + " does not fit " + shape_str(x.ne));
            add("soft_max", n.id, {x, mk, y},
                [scale](cudaStream_t st, const std::vector<TD> &t) { k::soft_max(t[0], &t[1], t[2], scale, st); },
                (double)(x.nelements() * 12));
        } else {
            add("soft_max", n.id, {x, y}, [scale](cudaStream_t st, const std::vector<TD> &t) { k::soft_max(t[0], nullptr, t[1], scale, st); },
                (double)(x.nelements() * 8));
        }
        return y;
    }
    if (op == "mul_mat") {
        need_src(n, sv, 2, 2);
        const TD &a = sv[0], &b = sv[1];
        if (a.ne[0] != b.ne[0] || b.ne[2] % a.ne[2] != 0 || b.ne[3] % a.ne[3] != 0)
            fail(n, "cannot multiply " + shape_str(a.ne) + " by " + shape_str(b.ne));
        if (a.ne[0] > 1 && a.nb[0] > a.nb[1] && !is_quant(a.type)) fail(n, "weight operand is transposed; it needs a cont first");
        const bool raw_q = k::raw_block_type(a.type);
        if ((is_quant(a.type) || raw_q) && !a.contiguous()) fail(n, "quantized weight must be contiguous");
        if (!is_quant(a.type) && !raw_q && a.type != T_F32 && a.type != T_F16 && a.type != T_BF16)
            fail(n, std::string("weight type ") + type_name(a.type) +
                        " is not supported by this backend (q4_0, q4_1, q5_0, q5_1, q8_0, iq4_nl, q4_K, q5_K, q6_K, f16, bf16, f32 are)");
        if (b.type != T_F32) fail(n, "activation operand must be f32");
        int64_t ne[4] = {a.ne[1], b.ne[1], b.ne[2], b.ne[3]};
        TD y = out_like(T_F32, ne);
        const double bytes = (double)(is_quant(a.type) ? (double)a.nrows() * (a.ne[0] / 32) * (quant_code_bytes(a.type) + 2)
                                      : raw_q           ? (double)a.nrows() * (double)row_size(a.type, a.ne[0])
                                                        : (double)a.nelements() * a.elsize()) +
                             (double)b.nelements() * 4 + (double)y.nelements() * 4;
        // 2-8 rows whose staged form is too large for the CUDA-core GEMV's shared memory (K = 14336 at
        // 8 rows) still take the tensor-core GEMV, which stages them itself
        auto mma_takes = [&]() {
            if (b.ne[1] < 2 || b.ne[1] > 8 || m.tp.active()) return false;
            FusedArgs fa;
            fa.qtype = a.type;
            fa.pro = PRO_Q8;
            fa.xq = b.data ? b.data : (const char *)&fa;  // only its presence matters here
            fa.map = MAP_SINGLE;
            fa.M = (int)b.ne[1];
            fa.K = a.ne[0];
            fa.wrows[0] = a.ne[1];
            return k::gemv_mma_ok(fa);
        };
        if (is_quant(a.type) && a.ne[2] == 1 && a.ne[3] == 1 && b.ne[2] == 1 && b.ne[3] == 1 && b.nb[0] == 4 &&
            (b.ne[1] == 1 || b.nb[1] == 4 * b.ne[0]) &&
            (k::fused_gemv_supported(a.ne[0], b.ne[1], MAP_SINGLE) || mma_takes())) {
            const int64_t K = a.ne[0], N = a.ne[1], M = b.ne[1];
            // 2-8 rows: quantized once into the staging layout by act_rows, so the GEMV (the
            // tensor-core one where it takes the shape) reads them instead of quantizing per CTA
            TD act;
            if (M >= 2 && !m.tp.active()) {
                scratch_marker((size_t)((M * K + M * (K / 32) * 8 + 127) / 128 * 128), &act);
                add("act_rows", n.id, {b, act},
                    [K, M](cudaStream_t st, const std::vector<TD> &t) {
                        FusedArgs fa;
                        fa.pro = PRO_ACT;
                        fa.x = (const float *)t[0].data;
                        fa.ldx = K;
                        fa.M = (int)M;
                        fa.K = K;
                        k::act_rows(fa, t[1].data, st);
                    },
                    (double)M * K * 5.25);
            }
            const bool staged = act.sid >= 0;
            add_gemv(a.type == T_Q4_0 ? "gemv_q4_0" : "gemv_q8_0", n.id, {a, b, y, act},
                     [K, N, M, staged](const std::vector<TD> &t) {
                         FusedArgs fa;
                         fa.qtype = t[0].type;
                         fa.pro = staged ? PRO_Q8 : PRO_ACT;
                         fa.xq = staged ? t[3].data : nullptr;
                         fa.map = MAP_SINGLE;
                         fa.x = (const float *)t[1].data;
                         fa.ldx = K;
                         fa.M = (int)M;
                         fa.K = K;
                         fa.wc[0] = t[0].data;
                         fa.wrows[0] = N;
                         fa.out = (float *)t[2].data;
                         fa.ldo = N;
                         return fa;
                     },
                     bytes);
            return y;
        }
        const size_t sb = k::mul_mat_scratch_bytes(a, b);
        TD scratch;
        if (sb) scratch_marker(sb, &scratch);
        if (sb)
            add("mul_mat", n.id, {a, b, y, scratch},
                [](cudaStream_t st, const std::vector<TD> &t) { k::mul_mat(t[0], t[1], t[2], t[3].data, st); }, bytes);
        else
            add("mul_mat", n.id, {a, b, y}, [](cudaStream_t st, const std::vector<TD> &t) { k::mul_mat(t[0], t[1], t[2], nullptr, st); },
                bytes);
        return y;
    }
    if (op == "flash_attn") {
        need_src(n, sv, 3, 4);
        const TD &q = sv[0], &kk = sv[1], &v = sv[2];
        if (kk.ne[0] != q.ne[0] || kk.ne[1] != v.ne[1] || q.ne[3] != kk.ne[3] || q.ne[3] != v.ne[3] || q.ne[2] % kk.ne[2] != 0 ||
            v.ne[0] != q.ne[0])
            fail(n, "q " + shape_str(q.ne) + ", k " + shape_str(kk.ne) + ", v " + shape_str(v.ne) + " do not line up");
        if (q.type != T_F32 || kk.type != T_F16 || v.type != T_F16) fail(n, "needs an f32 query and f16 K/V");
        if (kk.nb[0] != 2 || v.nb[0] != 2) fail(n, "K/V rows must be contiguous");
        if (q.ne[0] > 512) fail(n, "head size above 512");
        const float scale = n.pfloat("scale");
        int64_t ne[4] = {q.ne[0], q.ne[2], q.ne[1], q.ne[3]};
        TD y = out_like(T_F32, ne);
        const double bytes = (double)(kk.ne[1] * kk.ne[2] * kk.ne[3]) * kk.ne[0] * 4 + (double)q.nelements() * 8;
        if (q.sid >= 0 && head_sharded.count(q.sid)) {
            // tensor parallel: this rank's query heads (and their K/V heads, the only ones its
            // cache holds), then an exchange of the output rows' head slices
            const int W = m.tp.world, r = m.tp.rank;
            const int64_t D = q.ne[0], H = q.ne[2], Hkv = kk.ne[2], hw = H / W, kw = Hkv / W;
            const TD *mk = sv.size() > 3 ? &sv[3] : nullptr;
            if (!k::flash_split_ok(q) || H % W || Hkv % W || (mk && (mk->type != T_F16 || !mk->contiguous() || mk->ne[2] != 1 ||
                                                                     mk->ne[0] != kk.ne[1] || mk->ne[1] < q.ne[1])))
                fail(n, "tensor parallel: attention over this rank's query heads needs the split-KV kernel, head counts "
                        "divisible by the ranks and one mask for all heads");
            auto shift = [](TD t, int64_t bytes) {
                if (t.sid >= 0) t.off += (size_t)bytes;
                else t.data += bytes;
                return t;
            };
            TD qs = shift(q, hw * r * q.nb[2]), ks = shift(kk, kw * r * kk.nb[2]), vs = shift(v, kw * r * v.nb[2]);
            TD ys = shift(y, hw * r * D * 4);
            qs.ne[2] = hw;
            ks.ne[2] = vs.ne[2] = kw;
            ys.ne[1] = hw;
            TD scratch;
            scratch_marker(k::flash_split_scratch_bytes(qs, ks), &scratch);
            int *cnt = m.counters(s.name + "/" + n.id, k::flash_split_counters(qs, ks));
            int *err = m.d_err;
            const double sbytes = bytes / W;
            if (mk)
                add("flash_attn", n.id, {qs, ks, vs, *mk, ys, scratch},
                    [scale, cnt, err](cudaStream_t st, const std::vector<TD> &t) {
                        k::flash_attn_split(t[0], t[1], t[2], &t[3], t[4], scale, t[5].data, cnt, err, st);
                    },
                    sbytes);
            else
                add("flash_attn", n.id, {qs, ks, vs, ys, scratch},
                    [scale, cnt, err](cudaStream_t st, const std::vector<TD> &t) {
                        k::flash_attn_split(t[0], t[1], t[2], nullptr, t[3], scale, t[4].data, cnt, err, st);
                    },
                    sbytes);
            std::vector<int64_t> col((size_t)W + 1);
            for (int i = 0; i <= W; i++) col[(size_t)i] = hw * i * D * 4;
            if (!add_exchange(n.id, y, q.ne[1] * q.ne[3], H * D * 4, col))
                fail(n, "tensor parallel: the attention output does not fit the exchange window");
            return y;
        }
        if (sv.size() > 3) {
            const TD &mk = sv[3];
            if (mk.type != T_F16 || !mk.contiguous() || q.ne[2] % mk.ne[2] != 0 || mk.ne[0] != kk.ne[1] || mk.ne[1] < q.ne[1])
                fail(n, "mask must be a contiguous f16 tensor broadcastable over heads");
            if (k::flash_split_ok(q)) {
                TD scratch;
                scratch_marker(k::flash_split_scratch_bytes(q, kk), &scratch);
                int *cnt = m.counters(s.name + "/" + n.id, k::flash_split_counters(q, kk));
                int *err = m.d_err;
                const bool cluster = k::flash_split_prepare(q, kk, v, y);
                auto tr = trace_slot("flash_attn", n.id, cluster ? (size_t)(((kk.ne[1] + 63) / 64) * kk.ne[2] * q.ne[3])
                                                                  : k::flash_split_ctas(q, kk));
                auto act = std::make_shared<char *>(nullptr);
                // a fused QKV step of this plan writes the caches' rows at its positions: the cluster
                // kernel copies the other rows before its dependent-launch wait
                TD pos;
                auto kr = kv_rows.find(kk.data), vr = kv_rows.find(v.data);
                const bool early = cluster && m.attn_overlap && kk.sid < 0 && v.sid < 0 && kr != kv_rows.end() &&
                                   vr != kv_rows.end() && kr->second.data == vr->second.data && q.ne[3] == 1;
                if (early) pos = kr->second;
                const bool *direct = &m.direct_launch;
                const bool tc = m.prefill_attn_tc;
                add("flash_attn", n.id, {q, kk, v, mk, y, scratch, pos},
                    [scale, cnt, err, tr, act, early, direct, tc](cudaStream_t st, const std::vector<TD> &t) {
                        k::flash_attn_split(t[0], t[1], t[2], &t[3], t[4], scale, t[5].data, cnt, err, st, *tr, *act,
                                            early && !*direct ? (const int32_t *)t[6].data : nullptr, tc);
                    },
                    bytes);
                psteps.back().attn_early = early;
                if (q.ne[1] == 1 && q.ne[3] == 1) {
                    psteps.back().attn_act = act;
                    psteps.back().attn_k = q.ne[0] * q.ne[2];
                }
                return y;
            }
            add("flash_attn", n.id, {q, kk, v, mk, y},
                [scale](cudaStream_t st, const std::vector<TD> &t) { k::flash_attn(t[0], t[1], t[2], &t[3], t[4], scale, st); },
                bytes);
        } else if (k::flash_split_ok(q)) {
            TD scratch;
            scratch_marker(k::flash_split_scratch_bytes(q, kk), &scratch);
            int *cnt = m.counters(s.name + "/" + n.id, k::flash_split_counters(q, kk));
            int *err = m.d_err;
            const bool cluster = k::flash_split_prepare(q, kk, v, y);
            auto tr = trace_slot("flash_attn", n.id, cluster ? (size_t)(((kk.ne[1] + 63) / 64) * kk.ne[2] * q.ne[3])
                                                              : k::flash_split_ctas(q, kk));
            const bool tc = m.prefill_attn_tc;
            add("flash_attn", n.id, {q, kk, v, y, scratch},
                [scale, cnt, err, tr, tc](cudaStream_t st, const std::vector<TD> &t) {
                    k::flash_attn_split(t[0], t[1], t[2], nullptr, t[3], scale, t[4].data, cnt, err, st, *tr, nullptr,
                                        nullptr, tc);
                },
                bytes);
        } else {
            add("flash_attn", n.id, {q, kk, v, y},
                [scale](cudaStream_t st, const std::vector<TD> &t) { k::flash_attn(t[0], t[1], t[2], nullptr, t[3], scale, st); },
                bytes);
        }
        return y;
    }
    if (op == "swiglu") {
        need_src(n, sv, 2, 2);
        const TD &g = sv[0], &u = sv[1];
        if (!same_shape(g, u) || !g.contiguous() || !u.contiguous()) fail(n, "swiglu needs a gate and an up of one shape, both contiguous");
        TD y = out_like(T_F32, g.ne);
        add("swiglu", n.id, {g, u, y}, [](cudaStream_t st, const std::vector<TD> &t) { k::swiglu(t[0], t[1], t[2], st); },
            (double)(g.nelements() * 12));
        return y;
    }
    if (op == "set_rows") {
        need_src(n, sv, 3, 3);
        const TD &dst = sv[0], &src = sv[1], &idx = sv[2];
        if (dst.ne[0] != src.ne[0] || dst.ne[2] != src.ne[2] || dst.ne[3] != src.ne[3] || src.ne[1] != idx.ne[0] ||
            idx.ne[1] != 1 || idx.type != T_I32 || (src.type != T_F32 && src.type != T_F16))
            fail(n, "cannot write rows " + shape_str(src.ne) + " at indices " + shape_str(idx.ne) + " into " + shape_str(dst.ne));
        if (dst.nb[0] != (int64_t)dst.elsize() || src.nb[0] != (int64_t)src.elsize()) fail(n, "set_rows needs rows that are contiguous");
        int *err = m.d_err;
        add("set_rows", n.id, {dst, src, idx},
            [err](cudaStream_t st, const std::vector<TD> &t) { k::set_rows(t[0], t[1], t[2], err, st); },
            (double)(src.nelements() * (src.elsize() + dst.elsize())));
        return dst;  // written in place
    }
    if (op == "rope") {
        need_src(n, sv, 2, 3);
        const TD &x = sv[0], &pos = sv[1];
        const int n_dims = (int)n.pint("n_dims");
        const int mode = (int)n.pint("mode");
        if (x.type != T_F32 || x.nb[0] != 4 || pos.type != T_I32 || pos.ne[0] != x.ne[2] || pos.nrows() != 1 || n_dims % 2 ||
            n_dims > x.ne[0] || (sv.size() > 2 && (sv[2].type != T_F32 || sv[2].ne[0] < n_dims / 2)))
            fail(n, "cannot rotate " + shape_str(x.ne) + " at positions " + shape_str(pos.ne));
        if (mode != 0 && mode != 2) fail(n, "rope mode " + std::to_string(mode) + " is not supported (0 and 2 (NEOX) are)");
        const float base = n.pfloat("freq_base"), fs = n.pfloat("freq_scale"), af = n.pfloat("attn_factor");
        std::vector<float> ff;
        std::string ff_key = "-";
        if (sv.size() > 2) {
            if (sv[2].sid >= 0) fail(n, "rope frequency factors must be a weight");
            ff.resize((size_t)(n_dims / 2));
            cuda_check(cudaMemcpy(ff.data(), sv[2].data, ff.size() * 4, cudaMemcpyDeviceToHost), "rope factors");
            ff_key = n.src[2];
        }
        int64_t npos = 0;
        const float *table = m.rope_table(n_dims, base, fs, af, ff_key, ff.empty() ? nullptr : ff.data(), &npos);
        const float theta_scale = ::powf(base, -2.0f / (float)n_dims);
        const float *ffd = sv.size() > 2 ? (const float *)sv[2].data : nullptr;
        TD y = out_like(T_F32, x.ne);
        add("rope", n.id, {x, pos, y},
            [=](cudaStream_t st, const std::vector<TD> &t) {
                if (mode == 2)
                    k::rope_neox(t[0], t[1], t[2], n_dims, table, npos, theta_scale, fs, af, ffd, st);
                else
                    k::rope_norm(t[0], t[1], t[2], n_dims, table, npos, theta_scale, fs, af, ffd, st);
            },
            (double)(x.nelements() * 8));
        return y;
    }
    if (op == "argmax") {
        need_src(n, sv, 1, 1);
        const TD &x = sv[0];
        if (x.ne[2] != 1 || x.ne[3] != 1) fail(n, "argmax needs a matrix, got " + shape_str(x.ne));
        int64_t ne[4] = {x.ne[1], 1, 1, 1};
        TD y = out_like(T_I32, ne);
        if (const int parts = k::argmax_split_parts(x)) {
            TD scratch;
            scratch_marker((size_t)x.nrows() * parts * 8, &scratch);
            int *cnt = m.counters(s.name + "/" + n.id, (size_t)x.nrows());
            add("argmax", n.id, {x, y, scratch},
                [cnt](cudaStream_t st, const std::vector<TD> &t) { k::argmax_split(t[0], t[1], t[2].data, cnt, st); },
                (double)(x.nelements() * 4));
            return y;
        }
        add("argmax", n.id, {x, y}, [](cudaStream_t st, const std::vector<TD> &t) { k::argmax(t[0], t[1], st); },
            (double)(x.nelements() * 4));
        return y;
    }
    if (op == "get_rows") {
        need_src(n, sv, 2, 2);
        const TD &tab = sv[0], &idx = sv[1];
        if (idx.type != T_I32) fail(n, "row indices must be i32");
        if ((is_quant(tab.type) || k::raw_block_type(tab.type)) && !tab.contiguous()) fail(n, "quantized table must be contiguous");
        if (is_quantized(tab.type) && !is_quant(tab.type) && !k::raw_block_type(tab.type))
            fail(n, std::string("table type ") + type_name(tab.type) + " is not supported by this backend");
        int64_t ne[4] = {tab.ne[0], idx.ne[0], idx.ne[1], idx.ne[2]};
        TD y = out_like(T_F32, ne);
        add("get_rows", n.id, {tab, idx, y}, [](cudaStream_t st, const std::vector<TD> &t) { k::get_rows(t[0], t[1], t[2], st); },
            (double)(y.nelements() * 8));
        return y;
    }
    if (op == "sum_rows" || op == "mean") {
        need_src(n, sv, 1, 1);
        const TD &x = sv[0];
        int64_t ne[4] = {1, x.ne[1], x.ne[2], x.ne[3]};
        TD y = out_like(T_F32, ne);
        const float scale = op == "mean" ? 1.0f / (float)x.ne[0] : 1.0f;
        add("sum_rows", n.id, {x, y}, [scale](cudaStream_t st, const std::vector<TD> &t) { k::sum_rows(t[0], t[1], scale, st); },
            (double)(x.nelements() * 4));
        return y;
    }
    if (op == "repeat") {
        need_src(n, sv, 1, 1);
        for (int i = 0; i < 4; i++)
            if (n.ne[(size_t)i] % sv[0].ne[i] != 0) fail(n, "cannot repeat " + shape_str(sv[0].ne) + " to " + shape_str(n.ne.data()));
        TD y = out_like(sv[0].type, n.ne.data());
        add("repeat", n.id, {sv[0], y}, [](cudaStream_t st, const std::vector<TD> &t) { k::repeat(t[0], t[1], st); },
            (double)(y.nelements() * 8));
        return y;
    }
    if (op == "concat") {
        need_src(n, sv, 2, 2);
        const int dim = (int)n.pint("dim");
        if (dim < 0 || dim > 3) fail(n, "bad concat dim");
        for (int i = 0; i < 4; i++)
            if (i != dim && sv[0].ne[i] != sv[1].ne[i])
                fail(n, "cannot concat " + shape_str(sv[0].ne) + " and " + shape_str(sv[1].ne) + " along ggml dim " + std::to_string(dim));
        int64_t ne[4] = {sv[0].ne[0], sv[0].ne[1], sv[0].ne[2], sv[0].ne[3]};
        ne[dim] += sv[1].ne[dim];
        TD y = out_like(sv[0].type, ne);
        add("concat", n.id, {sv[0], sv[1], y}, [dim](cudaStream_t st, const std::vector<TD> &t) { k::concat(t[0], t[1], t[2], dim, st); },
            (double)(y.nelements() * 8));
        return y;
    }
    if (op == "arange") {
        need_src(n, sv, 0, 0);
        const float start = n.pfloat("start"), step = n.pfloat("step");
        TD y = out_like(T_F32, n.ne.data());
        add("arange", n.id, {y}, [start, step](cudaStream_t st, const std::vector<TD> &t) { k::arange(t[0], start, step, st); },
            (double)(y.nelements() * 4));
        return y;
    }
    fail(n, "op is not supported by this backend");
}

void Planner::finish() {
    // stage results into their driver values, after every other launch
    cur = (int)s.nodes.size();
    for (size_t i = 0; copy_results && i < s.outputs.size(); i++) {
        auto it = env.find(s.outputs[i]);
        if (it == env.end()) throw std::runtime_error("stage '" + s.name + "' returns unknown value '" + s.outputs[i] + "'");
        const TD r = it->second;
        auto vit = m.values.find(d.out[i]);
        if (vit == m.values.end()) throw std::runtime_error("driver value '" + d.out[i] + "' is not declared");
        const TD dst = vit->second.td;
        use(r);
        if (r.sid < 0 && r.data == dst.data && r.type == dst.type && same_shape(r, dst) && r.contiguous()) continue;
        if (r.nelements() != dst.nelements() || r.type != dst.type)
            throw std::runtime_error("stage '" + s.name + "' result " + std::to_string(i) + " does not match value '" + d.out[i] + "'");
        add("copy", "out." + std::to_string(i), {r, dst}, [](cudaStream_t st, const std::vector<TD> &t) { k::copy(t[0], t[1], st); },
            (double)(r.nelements() * r.elsize() * 2));
    }

    // pack storages: best fit over a free list, freed after their last use
    std::vector<std::vector<int>> starts(s.nodes.size() + 2), ends(s.nodes.size() + 2);
    for (size_t i = 0; i < storages.size(); i++) {
        starts[(size_t)storages[i].first].push_back((int)i);
        ends[(size_t)storages[i].last].push_back((int)i);
    }
    std::map<size_t, size_t> free_blocks;  // offset -> size
    size_t top = 0;
    auto take = [&](size_t bytes) {
        bytes = (bytes + 255) / 256 * 256;
        auto best = free_blocks.end();
        for (auto it = free_blocks.begin(); it != free_blocks.end(); ++it)
            if (it->second >= bytes && (best == free_blocks.end() || it->second < best->second)) best = it;
        if (best == free_blocks.end()) {
            const size_t o = top;
            top += bytes;
            return o;
        }
        const size_t o = best->first, sz = best->second;
        free_blocks.erase(best);
        if (sz > bytes) free_blocks[o + bytes] = sz - bytes;
        return o;
    };
    auto give = [&](size_t off, size_t bytes) {
        bytes = (bytes + 255) / 256 * 256;
        auto it = free_blocks.emplace(off, bytes).first;
        auto nx = std::next(it);
        if (nx != free_blocks.end() && it->first + it->second == nx->first) {
            it->second += nx->second;
            free_blocks.erase(nx);
        }
        if (it != free_blocks.begin()) {
            auto pv = std::prev(it);
            if (pv->first + pv->second == it->first) {
                pv->second += it->second;
                free_blocks.erase(it);
            }
        }
    };
    for (size_t i = 0; i < starts.size(); i++) {
        for (int sid : starts[i]) storages[(size_t)sid].offset = take(storages[(size_t)sid].bytes);
        for (int sid : ends[i]) give(storages[(size_t)sid].offset, storages[(size_t)sid].bytes);
    }
    if (plan.arena.size() < top) {
        cuda_check(cudaStreamSynchronize(m.stream), "arena");
        plan.arena.alloc(top);
    }
    char *base = plan.arena.get();
    for (auto &ps : psteps)
        for (auto &t : ps.tds)
            if (t.sid >= 0) {
                t.data = base + storages[(size_t)t.sid].offset + t.off;
                t.sid = -1;
                t.off = 0;
            }

    // Each fused GEMV prefetches into L2 the leading bytes of the next fused GEMV's matrices (the
    // last one those of the first: the next decode step starts there), up to m.l2_prefetch_bytes
    // in all, split over the matrices by size. In the tiled layout those leading tiles are exactly
    // the first pieces every CTA of the next launch streams.
    std::vector<size_t> gi;
    for (size_t i = 0; i < psteps.size(); i++)
        if (psteps[i].pf) gi.push_back(i);
    for (size_t x = 0; x < gi.size(); x++) {
        GemvExtras &pf = *psteps[gi[x]].pf;
        pf = GemvExtras{};
        pf.evict_first = m.stream_evict_first ? 1 : 0;
        pf.hold_pieces = m.prologue_hold;
        if (gi[x] > 0 && std::string(psteps[gi[x] - 1].kind) == "flash_attn") pf.producer_waits = m.producer_wait_after_attn;
        // a one-row attention that loads its K/V early right after: one CTA per SM, so that the
        // attention's CTAs fit beside this GEMV's
        if (m.qkv_one_per_sm && gi[x] + 1 < psteps.size() && psteps[gi[x] + 1].attn_early) pf.max_ctas = k::num_sms();
        // a one-row attention step m.kv_prefetch launches later: its K and V cache rows into L2
        // while this GEMV streams (the attention's bulk copies then read L2)
        const size_t ahead = (size_t)std::max(0, m.kv_prefetch);
        if (ahead && gi[x] + ahead < psteps.size() && psteps[gi[x] + ahead].attn_act) {
            const PlanStep &at = psteps[gi[x] + ahead];
            for (int r = 0; r < 2; r++) {
                const TD &kv = at.tds[(size_t)(1 + r)];
                pf.p[r] = kv.data;
                pf.n[r] = (int64_t)((kv.ne[2] - 1) * kv.nb[2] + kv.ne[1] * kv.nb[1]) & ~(int64_t)255;
            }
            continue;
        }
        if (m.l2_prefetch_bytes <= 0 || gi.size() < 2) continue;
        const PlanStep &nx = psteps[gi[(x + 1) % gi.size()]];
        const FusedArgs na = nx.gemv(nx.tds);
        if (na.nshard > 1) continue;
        const int nm = na.map == MAP_SINGLE ? 1 : na.map == MAP_SWIGLU ? 2 : 3;
        int64_t tot[3] = {0, 0, 0}, sum = 0;
        for (int r = 0; r < nm; r++) {
            tot[r] = qw_total_bytes(na.wrows[r], na.K / 32, na.qtype == T_Q4_0 ? 16 : 32);
            sum += tot[r];
        }
        for (int r = 0; r < nm && sum > 0; r++) {
            const int64_t take = std::min<int64_t>(tot[r], (int64_t)((double)m.l2_prefetch_bytes * (double)tot[r] / (double)sum));
            pf.p[r] = na.wc[r];
            pf.n[r] = take & ~(int64_t)255;
        }
    }

    // Q8_0 activation hand-off (one activation row, one GPU). A fused GEMV whose input row is the
    // whole output of the step right before it takes the row already quantized, in its staging
    // layout (PRO_Q8), and that step writes it: a split attention step from its merge; a residual
    // GEMV from its last CTA, with the rms_norm x weight the next GEMV applies; the SwiGLU GEMV per
    // 32-row block. The quantization rule is the prologue's, so results do not change; the
    // consumers' prologue shrinks to one copy into shared memory.
    if (m.act_handoff) {
        struct Link {
            size_t from, to;
            int mode;  // 0: attention merge, else an ACT8_* mode
            int64_t K;
        };
        std::vector<Link> links;
        for (size_t i = 1; i < psteps.size(); i++) {
            const PlanStep &B = psteps[i], &A = psteps[i - 1];
            if (!B.pf) continue;
            const FusedArgs b = B.gemv(B.tds);
            if (b.M != 1 || b.nshard != 1 || b.K % 32 || b.pro == PRO_Q8) continue;
            if (A.attn_act && b.pro == PRO_ACT && (const char *)b.x == A.tds[4].data && b.K == A.attn_k) {
                if (m.act_handoff & 1) links.push_back({i - 1, i, 0, b.K});
            } else if (A.pf) {
                const FusedArgs a = A.gemv(A.tds);
                if (a.M != 1 || a.nshard != 1 || (const float *)a.out != b.x || a.wrows[0] != b.K) continue;
                if (a.map == MAP_SINGLE && b.pro == PRO_NORM && (m.act_handoff & 2))
                    links.push_back({i - 1, i, ACT8_NORM, b.K});
                else if (a.map == MAP_SWIGLU && b.pro == PRO_ACT && (m.act_handoff & 4))
                    links.push_back({i - 1, i, ACT8_BLOCKS, b.K});
            }
        }
        auto staged = [](int64_t K) { return (size_t)((K + K / 32 * 8 + 127) / 128 * 128); };
        size_t bytes = 0;
        for (const Link &l : links) bytes += staged(l.K) + (size_t)((l.K / 32 + 32) * 4 + 127) / 128 * 128;
        if (bytes) {
            cuda_check(cudaStreamSynchronize(m.stream), "activation hand-off");
            plan.act.alloc(bytes);  // zero-filled: the counters start at zero
            char *p = plan.act.get();
            for (const Link &l : links) {
                char *act = p;
                int *cnt = (int *)(p + staged(l.K));
                p += staged(l.K) + (size_t)((l.K / 32 + 32) * 4 + 127) / 128 * 128;
                GemvExtras &to = *psteps[l.to].pf;
                to.xq = act;
                if (l.mode == 0) {
                    *psteps[l.from].attn_act = act;
                    continue;
                }
                const FusedArgs b = psteps[l.to].gemv(psteps[l.to].tds);
                GemvExtras &from = *psteps[l.from].pf;
                from.act_mode = l.mode;
                from.act_out = act;
                from.act_cnt = cnt;
                from.act_norm_w = b.norm_w;
                from.act_eps = b.eps;
            }
        }
    }

    if (!traces.empty()) {
        size_t words = 0;
        for (const auto &t : traces) words += t.ctas * 8;
        cuda_check(cudaStreamSynchronize(m.stream), "trace");
        plan.trace.alloc(words * sizeof(uint64_t));
        size_t off = 0;
        plan.trace_index.clear();
        for (auto &t : traces) {
            *t.slot = (uint64_t *)plan.trace.get() + off;
            plan.trace_index.push_back({t.kind, t.node, off, t.ctas});
            off += t.ctas * 8;
        }
    }
    plan.steps.clear();
    for (PlanStep &ps : psteps) {
        Step st;
        st.kind = ps.kind;
        st.node = ps.node;
        st.bytes = ps.bytes;
        auto fn = std::move(ps.fn);
        auto tds = std::move(ps.tds);
        st.run = [fn, tds](cudaStream_t stream) { fn(stream, tds); };
        plan.steps.push_back(std::move(st));
    }
}

void plan_call_site(Model &m, const CallSite &site, SitePlan &plan) {
    const StageSpec &s = *site.stage;
    const DriverStep &d = *site.step;
    if (d.args.size() != s.params.size() || d.out.size() != s.outputs.size())
        throw std::runtime_error("call to stage '" + s.name + "' has the wrong number of arguments or results");
    Planner p(m, plan, site);
    for (size_t i = 0; i < s.params.size(); i++) {
        auto it = m.values.find(d.args[i]);
        if (it == m.values.end()) throw std::runtime_error("driver value '" + d.args[i] + "' is not declared");
        const TD &arg = it->second.td;
        const TensorSpec &ps = s.params[i];
        for (int k = 0; k < 4; k++)
            if (arg.ne[k] != ps.ne[(size_t)k] || arg.type != ps.type)
                throw std::runtime_error("stage '" + s.name + "' parameter " + ps.name + " does not match value '" + d.args[i] + "'");
        p.env[ps.name] = arg;
    }
    std::vector<TD> sv;
    FusionPlan fp = find_fusions(m, s, p);

    // Nodes that read only weights and stage parameters that no node writes (the mask conversion
    // that every layer of a decode stage repeats) are planned first, and identical ones once, so
    // the launches that remain, the fused groups, are adjacent. `cur` counts plan positions.
    std::set<std::string> params, written;
    for (const auto &ps : s.params) params.insert(ps.name);
    for (const auto &n : s.nodes)
        if (n.op == "set_rows" && !n.src.empty()) written.insert(n.src[0]);
    std::unordered_map<std::string, size_t> index_of;
    std::unordered_map<std::string, std::string> same_as;  // node id -> an earlier identical node
    std::map<std::string, std::string> seen;
    std::vector<char> hoisted(s.nodes.size(), 0);
    for (size_t i = 0; i < s.nodes.size(); i++) {
        const NodeSpec &n = s.nodes[i];
        index_of[n.id] = i;
        if (fp.covered(i) || n.op == "set_rows") continue;
        bool ok = true;
        std::string key = n.op + "|" + std::to_string((int)n.type);
        for (int k = 0; k < 4; k++) key += "," + std::to_string(n.ne[(size_t)k]);
        for (const auto &name : n.src) {
            auto it = index_of.find(name);
            if (params.count(name)) ok = ok && !written.count(name);
            else if (it != index_of.end()) ok = ok && hoisted[it->second];
            auto al = same_as.find(name);
            key += "|" + (al == same_as.end() ? name : al->second);
        }
        if (!ok) continue;
        hoisted[i] = 1;
        key += "|" + n.p.dump();
        for (const auto &pb : n.p_bound) key += "|" + pb.first + "=" + std::to_string(pb.second);
        auto it = seen.find(key);
        if (it != seen.end()) same_as[n.id] = it->second;
        else seen.emplace(key, n.id);
    }
    std::vector<size_t> order;
    for (size_t i = 0; i < s.nodes.size(); i++)
        if (hoisted[i]) order.push_back(i);
    for (size_t i = 0; i < s.nodes.size(); i++)
        if (!hoisted[i]) order.push_back(i);

    for (size_t pos = 0; pos < order.size(); pos++) {
        const size_t i = order[pos];
        const NodeSpec &n = s.nodes[i];
        p.cur = (int)pos;
        auto al = same_as.find(n.id);
        if (al != same_as.end()) {
            p.env[n.id] = p.env.at(al->second);
            continue;
        }
        if (fp.covered(i)) {
            fp.emit_if_anchor(i, p);
            continue;
        }
        sv.clear();
        for (const auto &name : n.src) {
            sv.push_back(p.src_of(name));
            p.use(sv.back());
        }
        TD t = p.plan_node(n, sv);
        if (t.type != n.type) fail(n, std::string("produced type ") + type_name(t.type) + ", program expects " + type_name(n.type));
        for (int k = 0; k < 4; k++)
            if (t.ne[k] != n.ne[(size_t)k]) fail(n, "produced shape " + shape_str(t.ne) + ", program expects " + shape_str(n.ne.data()));
        p.env[n.id] = t;
    }
    p.finish();
}

}  // namespace gcb
