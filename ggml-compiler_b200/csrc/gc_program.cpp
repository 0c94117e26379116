#include "gc_program.h"

#include <algorithm>
#include <climits>
#include <stdexcept>

namespace gcb {

int64_t floor_div(int64_t a, int64_t b) {
    const int64_t q = a / b, r = a % b;
    return (r != 0 && ((r < 0) != (b < 0))) ? q - 1 : q;
}

int64_t floor_mod(int64_t a, int64_t b) {
    const int64_t r = a % b;
    return (r != 0 && ((r < 0) != (b < 0))) ? r + b : r;
}

Type parse_type(const std::string &name) {
    const TypeTraits *t = type_by_name(name);
    if (!t) throw std::runtime_error("unknown tensor type '" + name + "'");
    return t->type;
}

// ---------------------------------------------------------------------------------------- DimExpr

void DimExpr::emit(const Json &j, const std::vector<std::string> &names, std::vector<Ins> &out, int depth) {
    if (depth > 64) throw std::runtime_error("dim expression nests too deeply");
    if (j.is_int()) {
        out.push_back({K, 0, j.as_int()});
        return;
    }
    if (j.is_string()) {
        const auto it = std::find(names.begin(), names.end(), j.as_string());
        if (it == names.end()) throw std::runtime_error("dim refers to unknown symbol '" + j.as_string() + "'");
        out.push_back({SYM, 0, (int64_t)(it - names.begin())});
        return;
    }
    if (!j.is_array() || j.size() < 2 || !j[0].is_string()) throw std::runtime_error("malformed dim " + j.dump());
    static const std::pair<const char *, Op> ops[] = {{"+", ADD},  {"*", MUL},    {"//", FDIV},
                                                      {"%", MOD},  {"max", MAX}, {"min", MIN}};
    const std::string &name = j[0].as_string();
    const auto *op = std::find_if(std::begin(ops), std::end(ops), [&](const auto &o) { return name == o.first; });
    if (op == std::end(ops)) throw std::runtime_error("unknown dim operator '" + name + "'");
    for (size_t i = 1; i < j.size(); i++) emit(j[i], names, out, depth + 1);
    out.push_back({op->second, (uint16_t)(j.size() - 1), 0});
}

DimExpr DimExpr::parse(const Json &j, const std::vector<std::string> &names) {
    DimExpr e;
    e.code_.clear();
    emit(j, names, e.code_, 0);
    return e;
}

int64_t DimExpr::eval(const std::vector<int64_t> &vals) const {
    if (is_const()) return code_[0].x;
    int64_t stack[80];  // an operator's operands sit on top; depth <= nesting + arity
    int top = 0;
    for (const Ins &in : code_) {
        if (in.op == K || in.op == SYM) {
            if (top == 80) throw std::runtime_error("dim expression too large");
            if (in.op == SYM && (size_t)in.x >= vals.size()) throw std::runtime_error("dim reads an unbound symbol");
            stack[top++] = in.op == K ? in.x : vals[(size_t)in.x];
            continue;
        }
        int64_t *arg = stack + (top - in.argc), acc = arg[0];
        for (int k = 1; k < in.argc; k++) {
            const int64_t v = arg[k];
            if ((in.op == FDIV || in.op == MOD) && v == 0)
                throw std::runtime_error(std::string(in.op == FDIV ? "division" : "modulo") + " by zero in a symbolic dim");
            switch (in.op) {
                case ADD: acc += v; break;
                case MUL: acc *= v; break;
                case FDIV: acc = floor_div(acc, v); break;
                case MOD: acc = floor_mod(acc, v); break;
                case MAX: acc = std::max(acc, v); break;
                default: acc = std::min(acc, v); break;
            }
        }
        top -= in.argc;
        stack[top++] = acc;
    }
    return stack[0];
}

uint64_t DimExpr::reads() const {
    uint64_t m = 0;
    for (const Ins &in : code_)
        if (in.op == SYM) m |= 1ull << in.x;
    return m;
}

// ------------------------------------------------------------------------------ declarations, nodes

std::array<int64_t, 4> TensorSpec::ne_at(const std::vector<int64_t> &b) const {
    return {ne_expr[0].eval(b), ne_expr[1].eval(b), ne_expr[2].eval(b), ne_expr[3].eval(b)};
}

std::vector<int64_t> TensorSpec::shape_at(const std::vector<int64_t> &b) const {
    std::vector<int64_t> s(shape_expr.size());
    for (size_t i = 0; i < s.size(); i++) s[i] = shape_expr[i].eval(b);
    return s;
}

bool NodeSpec::has(const char *key) const {
    for (const auto &kv : dim_params)
        if (kv.first == key) return true;
    return p.contains(key);
}

double NodeSpec::pnum(const char *key) const { return (double)pint_or_num(key, true); }

int64_t NodeSpec::pint(const char *key) const { return (int64_t)pint_or_num(key, false); }

double NodeSpec::pint_or_num(const char *key, bool as_double) const {
    for (const auto &kv : p_bound)
        if (kv.first == key) return (double)kv.second;
    const Json *j = p.find(key);
    if (!j) throw std::runtime_error(where() + ": missing parameter '" + key + "'");
    return as_double ? j->as_double() : (double)j->as_int();
}

void ProgramSpec::bind(const std::vector<int64_t> &b) {
    if (b.size() != symbols.size()) throw std::runtime_error("binding has the wrong number of symbols");
    for (size_t k = 0; k < b.size(); k++)
        if (b[k] < symbols[k].min || b[k] > symbols[k].max)
            throw std::runtime_error("symbol '" + symbols[k].name + "' = " + std::to_string(b[k]) + " is outside [" +
                                     std::to_string(symbols[k].min) + ", " + std::to_string(symbols[k].max) + "]");
    auto bind_decl = [&](TensorSpec &t) {
        t.ne = t.ne_at(b);
        t.shape = t.shape_at(b);
        if (*std::min_element(t.ne.begin(), t.ne.end()) < 1)
            throw std::runtime_error("value '" + t.name + "' gets a dim below 1 at this binding");
    };
    for (auto &v : values) bind_decl(v);
    for (auto &st : stages) {
        for (auto &prm : st.params) bind_decl(prm);
        for (auto &n : st.nodes) {
            for (int i = 0; i < 4; i++) n.ne[i] = n.ne_expr[i].eval(b);
            n.p_bound.clear();
            for (const auto &dp : n.dim_params) n.p_bound.emplace_back(dp.first, dp.second.eval(b));
        }
    }
}

int ProgramSpec::symbol_index(const std::string &name) const {
    for (size_t k = 0; k < symbols.size(); k++)
        if (symbols[k].name == name) return (int)k;
    return -1;
}

// ----------------------------------------------------------------------------------------- reader

namespace {

// Walks the document once, building the specs; `names` are the symbol names dims may use.
class Reader {
  public:
    explicit Reader(const Json &root) : root_(root) {}

    ProgramSpec read() {
        ProgramSpec prog;
        prog.format_version = (int)root_.at("format_version").as_int();
        if (prog.format_version < kMinFormatVersion || prog.format_version > kFormatVersion)
            throw std::runtime_error("program format_version " + std::to_string(prog.format_version) +
                                     " is not supported (this runtime reads " + std::to_string(kMinFormatVersion) +
                                     " to " + std::to_string(kFormatVersion) + ")");
        for (const Json &s : list(root_, "symbols")) {
            prog.symbols.push_back({s.at("name").as_string(), s.at("min").as_int(), s.at("max").as_int()});
            names_.push_back(prog.symbols.back().name);
        }
        if (names_.size() > (size_t)kMaxSymbols) throw std::runtime_error("program has more than 64 symbols");
        for (const Json &v : root_.at("values").items()) prog.values.push_back(decl(v));
        for (const Json &s : root_.at("stages").items()) prog.stages.push_back(stage(s));
        stages_ = &prog.stages;
        symbols_ = &prog.symbols;
        if (const Json *es = root_.find("entries")) {
            for (const Json &e : es->items()) prog.entries.push_back(entry(e, e.at("name").as_string()));
        } else {  // format 1-2: the document itself is the one entry point
            prog.entries.push_back(entry(root_, "main"));
        }
        if (prog.entries.empty()) throw std::runtime_error("program has no entry point");
        for (const Json &s : list(root_, "state")) prog.state.push_back(s.as_string());
        std::vector<int64_t> lows;
        for (const Symbol &s : prog.symbols) lows.push_back(s.min);
        prog.bind(lows);  // every dim evaluates at the smallest binding, or the program is refused
        return prog;
    }

  private:
    const Json &root_;
    std::vector<std::string> names_;
    const std::vector<StageSpec> *stages_ = nullptr;
    const std::vector<Symbol> *symbols_ = nullptr;

    static const std::vector<Json> &list(const Json &j, const char *key) {
        static const Json none = Json::parse("[]");
        const Json *v = j.find(key);
        return (v ? *v : none).items();
    }

    static std::vector<std::string> strings(const Json &j) {
        std::vector<std::string> out;
        for (const Json &x : j.items()) out.push_back(x.as_string());
        return out;
    }

    std::array<DimExpr, 4> dims4(const Json &j, uint64_t &reads) const {
        if (!j.is_array() || j.size() != 4) throw std::runtime_error("'ne' must be an array of 4 dims");
        std::array<DimExpr, 4> ne;
        for (int i = 0; i < 4; i++) {
            ne[i] = DimExpr::parse(j[i], names_);
            reads |= ne[i].reads();
        }
        return ne;
    }

    TensorSpec decl(const Json &j) const {
        TensorSpec t;
        t.name = j.at("name").as_string();
        t.type = parse_type(j.at("type").as_string());
        t.ne_expr = dims4(j.at("ne"), t.reads);
        for (const Json &d : j.at("shape").items()) t.shape_expr.push_back(DimExpr::parse(d, names_));
        return t;
    }

    StageSpec stage(const Json &j) const {
        StageSpec s;
        s.name = j.at("name").as_string();
        for (const Json &p : j.at("params").items()) {
            s.params.push_back(decl(p));
            s.reads |= s.params.back().reads;
        }
        s.outputs = strings(j.at("outputs"));
        for (const Json &jn : j.at("nodes").items()) {
            NodeSpec n;
            n.id = jn.at("id").as_string();
            n.op = jn.at("op").as_string();
            n.src = strings(jn.at("src"));
            n.type = parse_type(jn.at("type").as_string());
            n.ne_expr = dims4(jn.at("ne"), s.reads);
            if (const Json *p = jn.find("p")) n.p = *p;
            if (const Json *l = jn.find("loc"); l && l->is_string()) n.loc = l->as_string();
            if (const Json *f = jn.find("fuse"); f && f->is_string()) n.fuse = f->as_string();
            // a view's start and an arange's bounds may be dims too (format 3)
            for (const char *key : {"start", "stop"})
                if (const Json *v = n.p.find(key); v && !v->is_number()) {
                    n.dim_params.emplace_back(key, DimExpr::parse(*v, names_));
                    s.reads |= n.dim_params.back().second.reads();
                }
            s.nodes.push_back(std::move(n));
        }
        return s;
    }

    EntrySpec entry(const Json &j, const std::string &name) const {
        EntrySpec e;
        e.name = name;
        e.inputs = strings(j.at("inputs"));
        e.outputs = strings(j.at("outputs"));
        for (const Json &d : j.at("driver").items()) e.driver.push_back(step(d));
        return e;
    }

    DriverStep step(const Json &j) const {
        DriverStep d;
        const std::string &op = j.at("op").as_string();
        if (op == "call") {
            const std::string &st = j.at("stage").as_string();
            for (size_t i = 0; i < stages_->size() && d.stage < 0; i++)
                if ((*stages_)[i].name == st) d.stage = (int)i;
            if (d.stage < 0) throw std::runtime_error("driver calls unknown stage '" + st + "'");
            d.args = strings(j.at("args"));
            d.out = strings(j.at("out"));
            return d;
        }
        if (op != "loop") throw std::runtime_error("driver op '" + op + "' is not supported by this runtime");
        d.is_loop = true;
        d.loop = std::make_shared<LoopSpec>(loop(j));
        return d;
    }

    int symbol(const std::string &name, const char *what) const {
        const auto it = std::find(names_.begin(), names_.end(), name);
        if (it == names_.end()) throw std::runtime_error(std::string(what) + " unknown symbol '" + name + "'");
        return (int)(it - names_.begin());
    }

    LoopSpec loop(const Json &j) const {
        LoopSpec L;
        const Json &n = j.at("n");
        if (n.is_string()) {
            L.trip_symbol = symbol(n.as_string(), "loop count refers to");
            L.trips = (*symbols_)[(size_t)L.trip_symbol].max;
        } else {
            L.trips = n.as_int();
        }
        std::vector<std::string> scope = names_;  // re-bind expressions see the counters after the symbols
        for (const Json &c : list(j, "counters")) {
            L.counters.push_back({c[0].as_string(), c[1].as_string()});
            scope.push_back(c[0].as_string());
        }
        if (scope.size() > (size_t)kMaxSymbols) throw std::runtime_error("loop has too many counters");
        for (const Json &b : list(j, "bind"))
            L.rebind.push_back({symbol(b[0].as_string(), "loop binds"), DimExpr::parse(b[1], scope)});
        for (const Json &m : list(j, "masks")) {
            int k = -1;
            for (size_t i = 0; i < L.counters.size() && k < 0; i++)
                if (L.counters[i].value == m[1].as_string()) k = (int)i;
            if (k < 0) throw std::runtime_error("loop mask uses unknown counter '" + m[1].as_string() + "'");
            L.masks.push_back({m[0].as_string(), k});
        }
        for (const Json &u : list(j, "until")) {
            LoopSpec::StopIds s{u[0].as_string(), {}};
            for (const Json &x : u[1].items()) s.ids.push_back((int32_t)x.as_int());
            L.until.push_back(std::move(s));
        }
        for (const Json &c : list(j, "collect")) L.collect.push_back({c[0].as_string(), c[1].as_string()});
        for (const Json &c : j.at("carry").items()) L.carry.push_back({c[0].as_string(), c[1].as_string()});
        for (const Json &s : j.at("scalars").items()) {
            LoopSpec::Scalar sc{s.at("value").as_string(), {}};
            for (const Json &x : s.at("values").items()) sc.per_iteration.push_back(x.as_float());
            if ((int64_t)sc.per_iteration.size() != L.trips)
                throw std::runtime_error("loop scalar has " + std::to_string(sc.per_iteration.size()) + " entries for " +
                                         std::to_string(L.trips) + " iterations");
            L.scalars.push_back(std::move(sc));
        }
        for (const Json &s : list(j, "slices")) L.slices.push_back({s[0].as_string(), s[1].as_string()});
        for (const Json &b : j.at("body").items()) L.body.push_back(step(b));
        return L;
    }
};

// Messages that already say what is wrong with the program pass through; anything else (a missing
// key, a wrong JSON kind) is reported as a malformed program.
bool self_explaining(const std::string &m) {
    for (const char *p : {"program ", "symbol ", "value ", "dim ", "loop ", "driver ", "unknown ", "'ne' "})
        if (m.rfind(p, 0) == 0) return true;
    return false;
}

}  // namespace

ProgramSpec parse_program(const std::string &text) {
    Json root;
    try {
        root = Json::parse(text);
    } catch (const std::exception &e) {
        throw std::runtime_error(std::string("program JSON does not parse: ") + e.what());
    }
    try {
        return Reader(root).read();
    } catch (const std::runtime_error &e) {
        if (self_explaining(e.what())) throw;
        throw std::runtime_error(std::string("malformed program: ") + e.what());
    }
}

}  // namespace gcb
