#include "gc_program.h"

#include <algorithm>
#include <climits>
#include <stdexcept>

namespace gcb {

int64_t floordiv(int64_t a, int64_t b) {
    const int64_t q = a / b;
    return (a % b != 0 && ((a < 0) != (b < 0))) ? q - 1 : q;
}

int64_t pymod(int64_t a, int64_t b) {
    const int64_t r = a % b;
    return (r != 0 && ((r < 0) != (b < 0))) ? r + b : r;
}

Type parse_type(const std::string &name) {
    const TypeTraits *t = type_by_name(name);
    if (!t) throw std::runtime_error("unknown tensor type '" + name + "'");
    return t->type;
}

int64_t Expr::eval(const std::vector<int64_t> &b) const {
    if (kind == Kind::Const) return value;
    if (kind == Kind::Sym) {
        if (value < 0 || (size_t)value >= b.size()) throw std::runtime_error("symbol index out of range");
        return b[(size_t)value];
    }
    int64_t acc = args.at(0).eval(b);
    for (size_t i = 1; i < args.size(); i++) {
        const int64_t x = args[i].eval(b);
        switch (kind) {
            case Kind::Add: acc += x; break;
            case Kind::Mul: acc *= x; break;
            case Kind::FloorDiv:
                if (x == 0) throw std::runtime_error("division by zero in a symbolic dim");
                acc = floordiv(acc, x);
                break;
            case Kind::Mod:
                if (x == 0) throw std::runtime_error("modulo by zero in a symbolic dim");
                acc = pymod(acc, x);
                break;
            case Kind::Max: acc = std::max(acc, x); break;
            case Kind::Min: acc = std::min(acc, x); break;
            default: break;
        }
    }
    return acc;
}

void Expr::symbols(std::vector<bool> &used) const {
    if (kind == Kind::Sym) used.at((size_t)value) = true;
    for (const auto &a : args) a.symbols(used);
}

int ProgramSpec::symbol_index(const std::string &name) const {
    for (size_t i = 0; i < symbols.size(); i++)
        if (symbols[i].name == name) return (int)i;
    return -1;
}

bool NodeSpec::has(const char *key) const {
    for (const auto &kv : p_bound)
        if (kv.first == key) return true;
    return p.contains(key);
}

double NodeSpec::pnum(const char *key) const {
    for (const auto &kv : p_bound)
        if (kv.first == key) return (double)kv.second;
    const Json *j = p.find(key);
    if (!j) throw std::runtime_error(where() + ": missing parameter '" + key + "'");
    return j->as_double();
}

int64_t NodeSpec::pint(const char *key) const {
    for (const auto &kv : p_bound)
        if (kv.first == key) return kv.second;
    const Json *j = p.find(key);
    if (!j) throw std::runtime_error(where() + ": missing parameter '" + key + "'");
    return j->as_int();
}

namespace {

Expr parse_dim(const Json &j, const std::vector<Symbol> &symbols) {
    Expr e;
    if (j.is_int()) {
        e.value = j.as_int();
        return e;
    }
    if (j.is_string()) {
        const std::string &name = j.as_string();
        for (size_t i = 0; i < symbols.size(); i++) {
            if (symbols[i].name == name) {
                e.kind = Expr::Kind::Sym;
                e.value = (int64_t)i;
                return e;
            }
        }
        throw std::runtime_error("dim refers to unknown symbol '" + name + "'");
    }
    if (!j.is_array() || j.size() < 2 || !j[0].is_string()) throw std::runtime_error("malformed dim " + j.dump());
    const std::string &op = j[0].as_string();
    if (op == "+") e.kind = Expr::Kind::Add;
    else if (op == "*") e.kind = Expr::Kind::Mul;
    else if (op == "//") e.kind = Expr::Kind::FloorDiv;
    else if (op == "%") e.kind = Expr::Kind::Mod;
    else if (op == "max") e.kind = Expr::Kind::Max;
    else if (op == "min") e.kind = Expr::Kind::Min;
    else throw std::runtime_error("unknown dim operator '" + op + "'");
    for (size_t i = 1; i < j.size(); i++) e.args.push_back(parse_dim(j[i], symbols));
    return e;
}

std::array<Expr, 4> parse_ne(const Json &j, const std::vector<Symbol> &symbols) {
    if (!j.is_array() || j.size() != 4) throw std::runtime_error("'ne' must be an array of 4 dims");
    std::array<Expr, 4> ne{};
    for (int i = 0; i < 4; i++) ne[i] = parse_dim(j[i], symbols);
    return ne;
}

TensorSpec parse_tensor(const Json &j, const std::vector<Symbol> &symbols) {
    TensorSpec t;
    t.name = j.at("name").as_string();
    t.type = parse_type(j.at("type").as_string());
    t.ne_x = parse_ne(j.at("ne"), symbols);
    for (const auto &d : j.at("shape").items()) t.shape_x.push_back(parse_dim(d, symbols));
    return t;
}

void bind_tensor(TensorSpec &t, const std::vector<int64_t> &b) {
    t.ne = eval_ne(t, b);
    t.shape = eval_shape(t, b);
    for (int64_t d : t.ne)
        if (d < 1) throw std::runtime_error("value '" + t.name + "' gets a dim of " + std::to_string(d));
}

std::vector<std::string> strings(const Json &j) {
    std::vector<std::string> out;
    for (const auto &x : j.items()) out.push_back(x.as_string());
    return out;
}

const Json &empty_array() {
    static const Json e = Json::parse("[]");
    return e;
}

const Json &opt_array(const Json &j, const char *key) {
    const Json *v = j.find(key);
    return v ? *v : empty_array();
}

DriverOp parse_driver_op(const Json &jd, const std::vector<Symbol> &symbols) {
    DriverOp d;
    const std::string &kind = jd.at("op").as_string();
    if (kind == "call") {
        d.kind = DriverOp::Kind::Call;
        d.stage = jd.at("stage").as_string();
        d.args = strings(jd.at("args"));
        d.out = strings(jd.at("out"));
        return d;
    }
    if (kind != "loop") throw std::runtime_error("driver op '" + kind + "' is not supported by this runtime");
    d.kind = DriverOp::Kind::Loop;
    const Json &jn = jd.at("n");
    if (jn.is_string()) {
        for (size_t i = 0; i < symbols.size(); i++)
            if (symbols[i].name == jn.as_string()) d.n_symbol = (int)i;
        if (d.n_symbol < 0) throw std::runtime_error("loop count refers to unknown symbol '" + jn.as_string() + "'");
        d.n = (int)symbols[(size_t)d.n_symbol].max;
    } else {
        d.n = (int)jn.as_int();
    }
    std::vector<Symbol> ext = symbols;  // counters extend the symbols the bind expressions see
    for (const auto &c : opt_array(jd, "counters").items()) {
        d.counters.emplace_back(c[0].as_string(), c[1].as_string());
        ext.push_back({c[0].as_string(), 0, INT64_MAX});
    }
    for (const auto &b : opt_array(jd, "bind").items()) {
        const std::string &name = b[0].as_string();
        int k = -1;
        for (size_t i = 0; i < symbols.size(); i++)
            if (symbols[i].name == name) k = (int)i;
        if (k < 0) throw std::runtime_error("loop binds unknown symbol '" + name + "'");
        d.bind.emplace_back(k, parse_dim(b[1], ext));
    }
    for (const auto &m : opt_array(jd, "masks").items()) {
        const std::string &counter = m[1].as_string();
        int k = -1;
        for (size_t i = 0; i < d.counters.size(); i++)
            if (d.counters[i].first == counter) k = (int)i;
        if (k < 0) throw std::runtime_error("loop mask uses unknown counter '" + counter + "'");
        d.masks.emplace_back(m[0].as_string(), k);
    }
    for (const auto &u : opt_array(jd, "until").items()) {
        std::vector<int> ids;
        for (const auto &x : u[1].items()) ids.push_back((int)x.as_int());
        d.until.emplace_back(u[0].as_string(), ids);
    }
    for (const auto &c : opt_array(jd, "collect").items()) d.collect.emplace_back(c[0].as_string(), c[1].as_string());
    for (const auto &c : jd.at("carry").items()) d.carry.emplace_back(c[0].as_string(), c[1].as_string());
    for (const auto &sc : jd.at("scalars").items()) {
        std::vector<float> vals;
        for (const auto &x : sc.at("values").items()) vals.push_back(x.as_float());
        if ((int)vals.size() != d.n)
            throw std::runtime_error("loop scalar has " + std::to_string(vals.size()) + " entries for " +
                                     std::to_string(d.n) + " iterations");
        d.scalars.emplace_back(sc.at("value").as_string(), std::move(vals));
    }
    for (const auto &sl : opt_array(jd, "slices").items()) d.slices.emplace_back(sl[0].as_string(), sl[1].as_string());
    for (const auto &b : jd.at("body").items()) d.body.push_back(parse_driver_op(b, symbols));
    return d;
}

}  // namespace

std::array<int64_t, 4> eval_ne(const TensorSpec &t, const std::vector<int64_t> &b) {
    std::array<int64_t, 4> ne{};
    for (int i = 0; i < 4; i++) ne[i] = t.ne_x[i].eval(b);
    return ne;
}

std::vector<int64_t> eval_shape(const TensorSpec &t, const std::vector<int64_t> &b) {
    std::vector<int64_t> s;
    for (const auto &d : t.shape_x) s.push_back(d.eval(b));
    return s;
}

void ProgramSpec::bind(const std::vector<int64_t> &b) {
    if (b.size() != symbols.size()) throw std::runtime_error("binding has the wrong number of symbols");
    for (size_t i = 0; i < symbols.size(); i++) {
        if (b[i] < symbols[i].min || b[i] > symbols[i].max)
            throw std::runtime_error("symbol '" + symbols[i].name + "' = " + std::to_string(b[i]) + " is outside [" +
                                     std::to_string(symbols[i].min) + ", " + std::to_string(symbols[i].max) + "]");
    }
    for (auto &v : values) bind_tensor(v, b);
    for (auto &s : stages) {
        for (auto &p : s.params) bind_tensor(p, b);
        for (auto &n : s.nodes) {
            for (int i = 0; i < 4; i++) n.ne[i] = n.ne_x[i].eval(b);
            n.p_bound.clear();
            for (const auto &kv : n.p_x) n.p_bound.emplace_back(kv.first, kv.second.eval(b));
        }
    }
}

ProgramSpec parse_program(const std::string &text) {
    Json j;
    try {
        j = Json::parse(text);
    } catch (const std::exception &e) {
        throw std::runtime_error(std::string("program JSON does not parse: ") + e.what());
    }
    ProgramSpec prog;
    try {
        prog.format_version = (int)j.at("format_version").as_int();
        if (prog.format_version < kMinFormatVersion || prog.format_version > kFormatVersion)
            throw std::runtime_error("program format_version " + std::to_string(prog.format_version) +
                                     " is not supported (this runtime reads " + std::to_string(kMinFormatVersion) +
                                     " to " + std::to_string(kFormatVersion) + ")");
        for (const auto &js : opt_array(j, "symbols").items())
            prog.symbols.push_back({js.at("name").as_string(), js.at("min").as_int(), js.at("max").as_int()});
        for (const auto &v : j.at("values").items()) prog.values.push_back(parse_tensor(v, prog.symbols));
        for (const auto &js : j.at("stages").items()) {
            StageSpec s;
            s.name = js.at("name").as_string();
            s.uses.assign(prog.symbols.size(), false);
            for (const auto &p : js.at("params").items()) {
                s.params.push_back(parse_tensor(p, prog.symbols));
                for (const auto &d : s.params.back().ne_x) d.symbols(s.uses);
            }
            s.outputs = strings(js.at("outputs"));
            for (const auto &jn : js.at("nodes").items()) {
                NodeSpec n;
                n.id = jn.at("id").as_string();
                n.op = jn.at("op").as_string();
                n.src = strings(jn.at("src"));
                n.type = parse_type(jn.at("type").as_string());
                n.ne_x = parse_ne(jn.at("ne"), prog.symbols);
                if (const Json *p = jn.find("p")) n.p = *p;
                if (const Json *l = jn.find("loc"))
                    if (l->is_string()) n.loc = l->as_string();
                for (const auto &d : n.ne_x) d.symbols(s.uses);
                for (const char *key : {"start", "stop"}) {  // symbolic parameters
                    const Json *v = n.p.find(key);
                    if (v && !v->is_number()) {
                        n.p_x.emplace_back(key, parse_dim(*v, prog.symbols));
                        n.p_x.back().second.symbols(s.uses);
                    }
                }
                s.nodes.push_back(std::move(n));
            }
            prog.stages.push_back(std::move(s));
        }
        auto parse_entry = [&](const Json &je, const std::string &name) {
            EntrySpec e;
            e.name = name;
            e.inputs = strings(je.at("inputs"));
            e.outputs = strings(je.at("outputs"));
            for (const auto &jd : je.at("driver").items()) e.driver.push_back(parse_driver_op(jd, prog.symbols));
            return e;
        };
        if (const Json *es = j.find("entries")) {
            for (const auto &je : es->items()) prog.entries.push_back(parse_entry(je, je.at("name").as_string()));
        } else {
            prog.entries.push_back(parse_entry(j, "main"));
        }
        if (prog.entries.empty()) throw std::runtime_error("program has no entry point");
        if (const Json *st = j.find("state")) prog.state = strings(*st);
        std::vector<int64_t> lo;
        for (const auto &sy : prog.symbols) lo.push_back(sy.min);
        prog.bind(lo);
    } catch (const std::runtime_error &e) {
        const std::string m = e.what();
        if (m.rfind("program ", 0) == 0 || m.rfind("symbol ", 0) == 0 || m.rfind("value ", 0) == 0 ||
            m.rfind("dim ", 0) == 0 || m.rfind("loop ", 0) == 0 || m.rfind("driver op", 0) == 0 ||
            m.rfind("unknown ", 0) == 0)
            throw;
        throw std::runtime_error("malformed program: " + m);
    }
    return prog;
}

}  // namespace gcb
