// Fusion pass: finds the language-model layer patterns the reference compiler emits (O2/O3:
// fuse_rms_norm, fuse_glu, fuse_rope, fuse_attention, f16 KV cache) and plans fused decode kernels
// for them (kernels/gc_fused.cu). Patterns, by the nodes they replace:
//
//   QKV    rms_norm -> mul(w) -> views -> 3 x mul_mat(Q4_0/Q8_0) -> views -> rope(q), rope(k) ->
//          views -> set_rows(k cache), views -> set_rows(v cache)          => one ROPE_QKV GEMV
//   GLU    rms_norm -> mul(w) -> views -> 2 x mul_mat -> views -> swiglu  => one SWIGLU GEMV
//   HEAD   rms_norm -> mul(w) -> views -> 1 x mul_mat                     => one NORM GEMV
//   RESID  mul_mat -> views -> add(residual, .)                           => one GEMV + residual
//
// A group is matched only if every value inside it has no reader outside it (other than the
// outputs it defines), every view chain is the stride arithmetic the fused kernel assumes (checked
// by replaying the views on the planner's descriptors), and the token count fits the GEMV (<= 8).
// The group is emitted at its first node; nodes between its members that are not in it only read
// values defined before it or the group's outputs.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <stdexcept>
#include <map>
#include <set>
#include <unordered_map>

#include "gc_fuse.h"
#include "gc_fused.h"

namespace gcb {

namespace {

bool is_view_op(const std::string &op) { return op == "reshape" || op == "view" || op == "permute"; }

struct Graph {
    const StageSpec &s;
    std::unordered_map<std::string, int> idx;
    std::vector<std::vector<int>> readers;
    std::set<std::string> outputs;

    explicit Graph(const StageSpec &st) : s(st), readers(st.nodes.size()) {
        for (size_t i = 0; i < s.nodes.size(); i++) idx[s.nodes[i].id] = (int)i;
        for (size_t i = 0; i < s.nodes.size(); i++)
            for (const auto &src : s.nodes[i].src) {
                auto it = idx.find(src);
                if (it != idx.end()) readers[(size_t)it->second].push_back((int)i);
            }
        for (const auto &o : s.outputs) outputs.insert(o);
    }
    const NodeSpec &n(int i) const { return s.nodes[(size_t)i]; }
    int node(const std::string &id) const {
        auto it = idx.find(id);
        return it == idx.end() ? -1 : it->second;
    }
    // Non-view consumers reached from node i through view nodes; the views passed on the way.
    void reach(int i, std::vector<int> &views, std::vector<int> &terms) const {
        for (int r : readers[(size_t)i]) {
            if (is_view_op(n(r).op)) {
                views.push_back(r);
                reach(r, views, terms);
            } else {
                terms.push_back(r);
            }
        }
    }
    // The view nodes from `from` to the value `id` (id is `from` itself or a chain of views of it).
    bool chain(int from, const std::string &id, std::vector<int> &out) const {
        out.clear();
        int cur = node(id);
        while (cur != from) {
            if (cur < 0 || !is_view_op(n(cur).op)) return false;
            out.push_back(cur);
            cur = node(n(cur).src[0]);
        }
        std::reverse(out.begin(), out.end());
        return true;
    }
};

bool quant_weight(const Model &m, const std::string &name, Type *t) {
    auto it = m.weights.find(name);
    if (it == m.weights.end()) return false;
    const TD &w = it->second.td;
    if ((w.type != T_Q4_0 && w.type != T_Q8_0) || w.ne[2] != 1 || w.ne[3] != 1) return false;
    *t = w.type;
    return true;
}

bool f32_vector(const Model &m, const std::string &name, int64_t n) {
    auto it = m.weights.find(name);
    if (it == m.weights.end()) return false;
    const TD &w = it->second.td;
    return w.type == T_F32 && w.ne[0] == n && w.ne[1] == 1 && w.ne[2] == 1 && w.ne[3] == 1;
}

// Replay a view chain on a descriptor (views only: no launches, no allocations).
bool replay(Planner &p, const Graph &g, TD t, const std::vector<int> &views, TD *out) {
    for (int v : views) {
        std::vector<TD> sv{t};
        try {
            t = p.plan_node(g.n(v), sv);
        } catch (...) {
            return false;
        }
    }
    *out = t;
    return true;
}

TD fake_contig(int64_t ne0, int64_t ne1, int64_t ne2) {
    TD t;
    t.type = T_F32;
    t.ne[0] = ne0;
    t.ne[1] = ne1;
    t.ne[2] = ne2;
    t.ne[3] = 1;
    set_contiguous(t);
    return t;  // data = nullptr: offsets show up as data pointers
}

bool strides_are(const TD &t, int64_t ne0, int64_t ne1, int64_t ne2, int64_t nb1, int64_t nb2) {
    return t.ne[0] == ne0 && t.ne[1] == ne1 && t.ne[2] == ne2 && t.ne[3] == 1 && t.nb[0] == 4 &&
           (ne1 == 1 || t.nb[1] == nb1) && (ne2 == 1 || t.nb[2] == nb2) && t.data == nullptr;
}

struct NormIn {
    int norm = -1, mul = -1;
    std::vector<int> mm;        // the matmuls reading the normalized activation
    std::vector<int> in_views;  // views between mul and the matmuls
    int64_t d = 0, M = 0, row0 = 0;  // width, token rows read, first row
};

// rms_norm -> mul(f32 [d] weight) -> views -> matmuls on quantized weights; the matmuls' activation
// must be consecutive rows of the normalized tensor.
bool match_norm_in(Model &m, Planner &p, const Graph &g, int i, NormIn *r) {
    const NodeSpec &nn = g.n(i);
    if (nn.op != "rms_norm" || g.outputs.count(nn.id) || g.readers[(size_t)i].size() != 1) return false;
    const int j = g.readers[(size_t)i][0];
    const NodeSpec &mul = g.n(j);
    if (mul.op != "mul" || mul.src[0] != nn.id || g.outputs.count(mul.id)) return false;
    const int64_t d = nn.ne[0];
    if (!f32_vector(m, mul.src[1], d) || nn.ne[2] != 1 || nn.ne[3] != 1) return false;
    std::vector<int> views, terms;
    g.reach(j, views, terms);
    if (terms.empty()) return false;
    for (int v : views)
        if (g.outputs.count(g.n(v).id)) return false;
    TD act;
    bool first = true;
    Type qt = T_F32;
    for (int t : terms) {
        const NodeSpec &mm = g.n(t);
        Type wt;
        if (mm.op != "mul_mat" || !quant_weight(m, mm.src[0], &wt)) return false;
        if (first) qt = wt;
        if (wt != qt) return false;
        std::vector<int> ch;
        if (!g.chain(j, mm.src[1], ch)) return false;
        TD a;
        if (!replay(p, g, fake_contig(d, nn.ne[1], 1), ch, &a)) return false;
        if (a.ne[0] != d || a.nb[0] != 4 || a.ne[2] != 1 || a.ne[3] != 1 || (a.ne[1] > 1 && a.nb[1] != 4 * d)) return false;
        if (!first && (a.data != act.data || a.ne[1] != act.ne[1])) return false;
        act = a;
        first = false;
        if (m.weights.at(mm.src[0]).td.ne[0] != d) return false;
    }
    r->norm = i;
    r->mul = j;
    r->mm = terms;
    r->in_views = views;
    r->d = d;
    r->M = act.ne[1];
    r->row0 = (int64_t)(size_t)act.data / (4 * d);
    return k::fused_gemv_supported(d, r->M, MAP_SINGLE);
}

void fill_weight(FusedArgs &a, int slot, const TD &w) {
    a.wc[slot] = w.data;
    a.ws[slot] = w.scales;
    a.wrows[slot] = w.ne[1];
    a.qtype = w.type;
}

double weight_bytes(const TD &w) { return (double)w.ne[1] * (double)(w.ne[0] / 32) * (quant_code_bytes(w.type) + 2); }

}  // namespace

FusionPlan find_fusions(Model &m, const StageSpec &s, Planner &p) {
    FusionPlan fp;
    fp.group_of.assign(s.nodes.size(), -1);
    if (std::getenv("GGML_COMPILER_B200_NOFUSE")) return fp;
    Graph g(s);
    // Emitter marks: a stage whose nodes carry "fuse" marks fuses exactly the groups it marked (a
    // matched group whose nodes are one whole mark of the matched kind); other matches run unfused.
    // A stage without marks (a program from an emitter that writes none) is matched as a whole.
    std::map<std::string, size_t> mark_size;
    for (const auto &n : s.nodes)
        if (!n.fuse.empty()) mark_size[n.fuse]++;
    static const char *kind_mark[] = {"qkv.", "glu.", "head.", "resid."};
    auto claim = [&](std::vector<int> nodes, std::function<void(Planner &)> emit, std::shared_ptr<GroupDesc> desc) {
        for (int x : nodes)
            if (fp.group_of[(size_t)x] >= 0) return false;
        FusionGroup grp;
        std::sort(nodes.begin(), nodes.end());
        nodes.erase(std::unique(nodes.begin(), nodes.end()), nodes.end());
        if (!mark_size.empty()) {
            const std::string &mk = g.n(nodes.front()).fuse;
            if (mk.empty() || mk.rfind(kind_mark[desc->kind], 0) != 0 || mark_size[mk] != nodes.size()) return false;
            for (int x : nodes)
                if (g.n(x).fuse != mk) return false;
        }
        for (int x : nodes) grp.nodes.push_back((size_t)x);
        grp.anchor = (size_t)nodes.front();
        grp.emit = std::move(emit);
        grp.desc = std::move(desc);
        const int gid = (int)fp.groups.size();
        for (int x : nodes) fp.group_of[(size_t)x] = gid;
        fp.groups.push_back(std::move(grp));
        return true;
    };
    // every node of a group must be read only inside the group, except the listed outputs
    auto closed = [&](const std::vector<int> &nodes, const std::set<int> &outs) {
        std::set<int> in(nodes.begin(), nodes.end());
        for (int x : nodes) {
            if (outs.count(x)) continue;
            if (g.outputs.count(g.n(x).id)) return false;
            for (int r : g.readers[(size_t)x])
                if (!in.count(r)) return false;
        }
        return true;
    };

    for (size_t i = 0; i < s.nodes.size(); i++) {
        if (fp.group_of[i] >= 0) continue;
        NormIn ni;
        if (s.nodes[i].op != "rms_norm" || !match_norm_in(m, p, g, (int)i, &ni)) continue;
        const NodeSpec &rms = g.n(ni.norm), &mul = g.n(ni.mul);
        const float eps = rms.pfloat("eps");
        const std::string xname = rms.src[0], wname = mul.src[1];
        const int64_t d = ni.d, M = ni.M, row0 = ni.row0;

        if (ni.mm.size() == 3) {  // ---- QKV + rope + KV cache
            int q = -1, kk = -1, v = -1, rq = -1, rk = -1, sk = -1, sv = -1;
            std::vector<int> group = {ni.norm, ni.mul};
            group.insert(group.end(), ni.in_views.begin(), ni.in_views.end());
            std::vector<int> qviews_out;
            bool ok = true;
            for (int mmi : ni.mm) {
                std::vector<int> views, terms;
                g.reach(mmi, views, terms);
                if (terms.size() != 1) {
                    ok = false;
                    break;
                }
                const NodeSpec &t = g.n(terms[0]);
                if (t.op == "set_rows") {
                    v = mmi;
                    sv = terms[0];
                    group.insert(group.end(), views.begin(), views.end());
                } else if (t.op == "rope") {
                    std::vector<int> v2, t2;
                    g.reach(terms[0], v2, t2);
                    if (t2.size() != 1) {
                        ok = false;
                        break;
                    }
                    if (g.n(t2[0]).op == "set_rows") {
                        kk = mmi;
                        rk = terms[0];
                        sk = t2[0];
                        group.insert(group.end(), v2.begin(), v2.end());
                    } else if (g.n(t2[0]).op == "flash_attn") {
                        q = mmi;
                        rq = terms[0];
                        qviews_out = v2;
                    } else {
                        ok = false;
                        break;
                    }
                    group.insert(group.end(), views.begin(), views.end());
                } else {
                    ok = false;
                    break;
                }
                group.push_back(mmi);
            }
            if (!ok || q < 0 || kk < 0 || v < 0) continue;
            group.insert(group.end(), {rq, rk, sk, sv});
            const NodeSpec &ropeq = g.n(rq), &ropek = g.n(rk), &setk = g.n(sk), &setv = g.n(sv);
            const int64_t D = ropeq.ne[0], H = ropeq.ne[1];
            const int64_t Hkv = ropek.ne[1];
            const std::string pos = ropeq.src[1];
            if (ropeq.src.size() != 2 || ropek.src.size() != 2 || ropek.src[1] != pos || setk.src[2] != pos ||
                setv.src[2] != pos || ropeq.pint("mode") != 2 || ropek.pint("mode") != 2 || ropeq.pint("n_dims") != D ||
                ropek.pint("n_dims") != D || ropek.ne[0] != D || ropeq.pfloat("freq_scale") != 1.0f ||
                ropeq.pfloat("attn_factor") != 1.0f || ropek.pfloat("freq_base") != ropeq.pfloat("freq_base") ||
                ropek.pfloat("freq_scale") != 1.0f || ropek.pfloat("attn_factor") != 1.0f || ropeq.ne[2] != M ||
                ropek.ne[2] != M || D % 2)
                continue;
            if (!k::fused_gemv_supported(d, M, MAP_ROPE_QKV)) continue;
            const TD &wq = m.weights.at(g.n(q).src[0]).td, &wk = m.weights.at(g.n(kk).src[0]).td,
                     &wv = m.weights.at(g.n(v).src[0]).td;
            if (wq.ne[1] != H * D || wk.ne[1] != Hkv * D || wv.ne[1] != Hkv * D || H % Hkv) continue;
            // the ropes read [D, heads, M] views of the matmul outputs; the set_rows read [D, M, heads]
            std::vector<int> ch;
            TD t;
            if (!g.chain(q, ropeq.src[0], ch) || !replay(p, g, fake_contig(H * D, M, 1), ch, &t) ||
                !strides_are(t, D, H, M, 4 * D, 4 * D * H))
                continue;
            if (!g.chain(kk, ropek.src[0], ch) || !replay(p, g, fake_contig(Hkv * D, M, 1), ch, &t) ||
                !strides_are(t, D, Hkv, M, 4 * D, 4 * D * Hkv))
                continue;
            if (!g.chain(rk, setk.src[1], ch) || !replay(p, g, fake_contig(D, Hkv, M), ch, &t) ||
                !strides_are(t, D, M, Hkv, 4 * D * Hkv, 4 * D))
                continue;
            if (!g.chain(v, setv.src[1], ch) || !replay(p, g, fake_contig(Hkv * D, M, 1), ch, &t) ||
                !strides_are(t, D, M, Hkv, 4 * D * Hkv, 4 * D))
                continue;
            if (!closed(group, {rq, sk, sv})) continue;
            // rope q's readers are the views to flash attention: outside the group, read after it
            const std::string qid = ropeq.id, kid = setk.id, vid = setv.id;
            const std::string kc = setk.src[0], vc = setv.src[0];
            const std::string wqn = g.n(q).src[0], wkn = g.n(kk).src[0], wvn = g.n(v).src[0];
            const float base = ropeq.pfloat("freq_base");
            claim(group, [=, &m](Planner &pl) {
                TD x = pl.src_of(xname), nw = pl.src_of(wname), tq = pl.src_of(wqn), tk = pl.src_of(wkn),
                   tv = pl.src_of(wvn), tp = pl.src_of(pos), tkc = pl.src_of(kc), tvc = pl.src_of(vc);
                const int64_t ne[4] = {D, H, M, 1};
                TD qb = pl.alloc(T_F32, ne);
                int64_t npos = 0;
                const float *table = m.rope_table((int)D, base, 1.0f, 1.0f, "-", nullptr, &npos);
                const float theta_scale = ::powf(base, -2.0f / (float)D);
                int *err = m.d_err;
                const double bytes = weight_bytes(tq) + weight_bytes(tk) + weight_bytes(tv) + 4.0 * d * M;
                pl.add_gemv(tq.type == T_Q4_0 ? "gemv_q4_0_qkv" : "gemv_q8_0_qkv", qid, {x, nw, tq, tk, tv, tp, tkc, tvc, qb},
                       [=](const std::vector<TD> &td) {
                           FusedArgs a;
                           a.pro = PRO_NORM;
                           a.map = MAP_ROPE_QKV;
                           a.x = (const float *)td[0].data + row0 * (td[0].nb[1] / 4);
                           a.ldx = td[0].nb[1] / 4;
                           a.M = (int)M;
                           a.K = d;
                           a.norm_w = (const float *)td[1].data;
                           a.eps = eps;
                           fill_weight(a, 0, td[2]);
                           fill_weight(a, 1, td[3]);
                           fill_weight(a, 2, td[4]);
                           a.pos = (const int32_t *)td[5].data;
                           a.kcache = td[6].data;
                           a.vcache = td[7].data;
                           a.cache_nb1 = td[6].nb[1];
                           a.cache_nb2 = td[6].nb[2];
                           a.cache_rows = td[6].ne[1];
                           a.q_out = (float *)td[8].data;
                           a.ldq = D * H;
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
                pl.env[qid] = qb;
                pl.env[kid] = tkc;
                pl.env[vid] = tvc;
                pl.kv_rows[tkc.data] = tp;
                pl.kv_rows[tvc.data] = tp;
            }, [&] {
                auto ds = std::make_shared<GroupDesc>();
                ds->kind = GroupDesc::QKV;
                ds->x = xname;
                ds->norm_w = wname;
                ds->w[0] = wqn, ds->w[1] = wkn, ds->w[2] = wvn;
                ds->pos = pos;
                ds->kc = kc, ds->vc = vc;
                ds->out[0] = qid, ds->out[1] = kid, ds->out[2] = vid;
                ds->eps = eps, ds->base = base;
                ds->d = d, ds->N = (H + 2 * Hkv) * D;
                ds->D = D, ds->H = H, ds->Hkv = Hkv;
                return ds;
            }());
            continue;
        }

        if (ni.mm.size() == 2) {  // ---- gate / up + swiglu
            std::vector<int> group = {ni.norm, ni.mul};
            group.insert(group.end(), ni.in_views.begin(), ni.in_views.end());
            int sw = -1;
            bool ok = true;
            for (int mmi : ni.mm) {
                std::vector<int> views, terms;
                g.reach(mmi, views, terms);
                if (terms.size() != 1 || g.n(terms[0]).op != "swiglu" || (sw >= 0 && terms[0] != sw)) {
                    ok = false;
                    break;
                }
                sw = terms[0];
                group.insert(group.end(), views.begin(), views.end());
                group.push_back(mmi);
            }
            if (!ok || sw < 0) continue;
            const NodeSpec &swn = g.n(sw);
            // which matmul feeds the gate (src 0) and which the up (src 1)
            int mg = -1, mu = -1;
            std::vector<int> ch;
            for (int mmi : ni.mm) {
                if (g.chain(mmi, swn.src[0], ch)) mg = mmi;
                else if (g.chain(mmi, swn.src[1], ch)) mu = mmi;
            }
            if (mg < 0 || mu < 0) continue;
            const int64_t F = swn.ne[0];
            const TD &wg = m.weights.at(g.n(mg).src[0]).td, &wu = m.weights.at(g.n(mu).src[0]).td;
            if (wg.ne[1] != F || wu.ne[1] != F || swn.ne[1] != M || swn.ne[2] != 1) continue;
            TD t;
            if (!g.chain(mg, swn.src[0], ch) || !replay(p, g, fake_contig(F, M, 1), ch, &t) || !strides_are(t, F, M, 1, 4 * F, 0))
                continue;
            if (!g.chain(mu, swn.src[1], ch) || !replay(p, g, fake_contig(F, M, 1), ch, &t) || !strides_are(t, F, M, 1, 4 * F, 0))
                continue;
            group.push_back(sw);
            if (!closed(group, {sw})) continue;
            if (!k::fused_gemv_supported(d, M, MAP_SWIGLU)) continue;
            const std::string swid = swn.id, wgn = g.n(mg).src[0], wun = g.n(mu).src[0];
            claim(group, [=](Planner &pl) {
                TD x = pl.src_of(xname), nw = pl.src_of(wname), tg = pl.src_of(wgn), tu = pl.src_of(wun);
                const int64_t ne[4] = {F, M, 1, 1};
                TD hb = pl.alloc(T_F32, ne);
                const double bytes = weight_bytes(tg) + weight_bytes(tu) + 4.0 * d * M + 4.0 * F * M;
                pl.add_gemv(tg.type == T_Q4_0 ? "gemv_q4_0_glu" : "gemv_q8_0_glu", swid, {x, nw, tg, tu, hb},
                       [=](const std::vector<TD> &td) {
                           FusedArgs a;
                           a.pro = PRO_NORM;
                           a.map = MAP_SWIGLU;
                           a.x = (const float *)td[0].data + row0 * (td[0].nb[1] / 4);
                           a.ldx = td[0].nb[1] / 4;
                           a.M = (int)M;
                           a.K = d;
                           a.norm_w = (const float *)td[1].data;
                           a.eps = eps;
                           fill_weight(a, 0, td[2]);
                           fill_weight(a, 1, td[3]);
                           a.out = (float *)td[4].data;
                           a.ldo = F;
                           return a;
                       },
                       bytes);
                pl.env[swid] = hb;
            }, [&] {
                auto ds = std::make_shared<GroupDesc>();
                ds->kind = GroupDesc::GLU;
                ds->x = xname;
                ds->norm_w = wname;
                ds->w[0] = wgn, ds->w[1] = wun;
                ds->out[0] = swid;
                ds->eps = eps;
                ds->d = d, ds->N = F;
                return ds;
            }());
            continue;
        }

        if (ni.mm.size() == 1) {  // ---- norm + one matmul (the output head)
            const int mmi = ni.mm[0];
            std::vector<int> group = {ni.norm, ni.mul, mmi};
            group.insert(group.end(), ni.in_views.begin(), ni.in_views.end());
            if (!closed(group, {mmi})) continue;
            const NodeSpec &mm = g.n(mmi);
            const std::string mid = mm.id, wn = mm.src[0];
            const int64_t N = mm.ne[0];
            claim(group, [=](Planner &pl) {
                TD x = pl.src_of(xname), nw = pl.src_of(wname), tw = pl.src_of(wn);
                const int64_t ne[4] = {N, M, 1, 1};
                TD yb = pl.alloc(T_F32, ne);
                const double bytes = weight_bytes(tw) + 4.0 * d * M + 4.0 * N * M;
                pl.add_gemv(tw.type == T_Q4_0 ? "gemv_q4_0_head" : "gemv_q8_0_head", mid, {x, nw, tw, yb},
                       [=](const std::vector<TD> &td) {
                           FusedArgs a;
                           a.pro = PRO_NORM;
                           a.map = MAP_SINGLE;
                           a.x = (const float *)td[0].data + row0 * (td[0].nb[1] / 4);
                           a.ldx = td[0].nb[1] / 4;
                           a.M = (int)M;
                           a.K = d;
                           a.norm_w = (const float *)td[1].data;
                           a.eps = eps;
                           fill_weight(a, 0, td[2]);
                           a.out = (float *)td[3].data;
                           a.ldo = N;
                           return a;
                       },
                       bytes);
                pl.env[mid] = yb;
            }, [&] {
                auto ds = std::make_shared<GroupDesc>();
                ds->kind = GroupDesc::HEAD;
                ds->x = xname;
                ds->norm_w = wname;
                ds->w[0] = wn;
                ds->out[0] = mid;
                ds->eps = eps;
                ds->d = d, ds->N = N;
                return ds;
            }());
        }
    }

    // ---- matmul + residual add (o_proj, down): mul_mat(W, x) -> views -> add(res, .)
    for (size_t i = 0; i < s.nodes.size(); i++) {
        if (fp.group_of[i] >= 0 || s.nodes[i].op != "mul_mat") continue;
        const NodeSpec &mm = s.nodes[i];
        Type wt;
        if (!quant_weight(m, mm.src[0], &wt)) continue;
        std::vector<int> views, terms;
        g.reach((int)i, views, terms);
        if (terms.size() != 1 || g.n(terms[0]).op != "add") continue;
        const NodeSpec &add = g.n(terms[0]);
        std::vector<int> ch;
        if (!g.chain((int)i, add.src[1], ch) || g.chain((int)i, add.src[0], ch)) continue;
        const int64_t N = mm.ne[0], M = mm.ne[1], K = m.weights.at(mm.src[0]).td.ne[0];
        if (mm.ne[2] != 1 || mm.ne[3] != 1 || add.ne[0] != N || add.ne[1] != M || add.ne[2] != 1) continue;
        TD t;
        g.chain((int)i, add.src[1], ch);
        if (!replay(p, g, fake_contig(N, M, 1), ch, &t) || !strides_are(t, N, M, 1, 4 * N, 0)) continue;
        if (!k::fused_gemv_supported(K, M, MAP_SINGLE)) continue;
        std::vector<int> group = {(int)i, terms[0]};
        group.insert(group.end(), views.begin(), views.end());
        if (!closed(group, {terms[0]})) continue;
        if (g.node(add.src[0]) >= (int)i) continue;  // the residual must exist when the group runs
        const std::string aid = add.id, resn = add.src[0], xn = mm.src[1], wn = mm.src[0];
        claim(group, [=](Planner &pl) {
            TD x = pl.src_of(xn), res = pl.src_of(resn), tw = pl.src_of(wn);
            if (x.type != T_F32 || x.nb[0] != 4 || (M > 1 && x.nb[1] != 4 * K) || res.type != T_F32 || res.nb[0] != 4 ||
                (M > 1 && res.nb[1] != 4 * N))
                throw std::runtime_error("fused residual GEMV: unexpected strides at " + aid);
            const int64_t ne[4] = {N, M, 1, 1};
            TD yb = pl.alloc(T_F32, ne);
            const double bytes = weight_bytes(tw) + 4.0 * K * M + 8.0 * N * M;
            pl.add_gemv(tw.type == T_Q4_0 ? "gemv_q4_0_res" : "gemv_q8_0_res", aid, {x, res, tw, yb},
                   [=](const std::vector<TD> &td) {
                       FusedArgs a;
                       a.pro = PRO_ACT;
                       a.map = MAP_SINGLE;
                       a.x = (const float *)td[0].data;
                       a.ldx = K;
                       a.M = (int)M;
                       a.K = K;
                       fill_weight(a, 0, td[2]);
                       a.res = (const float *)td[1].data;
                       a.ldr = N;
                       a.out = (float *)td[3].data;
                       a.ldo = N;
                       return a;
                   },
                   bytes);
            pl.env[aid] = yb;
        }, [&] {
            auto ds = std::make_shared<GroupDesc>();
            ds->kind = GroupDesc::RESID;
            ds->x = xn;
            ds->res = resn;
            ds->w[0] = wn;
            ds->out[0] = aid;
            ds->d = K, ds->N = N;
            return ds;
        }());
    }
    return fp;
}

}  // namespace gcb
