// The `ggml_compiler.program` JSON (formats 1-3) as specs the executor plans kernels from.
//
// Same document and semantics as the reference's runtime/src/program.h:21-125 and
// runtime/src/program.cpp:22-302: `ne` is innermost-first, a dim may be an integer, a symbol name or
// [op, operand...] with op in + * // % max min (Python floor semantics), and ProgramSpec::bind
// evaluates every symbolic dim and parameter for one binding (every symbol in its range).
#pragma once

#include <array>
#include <cstdint>
#include <string>
#include <utility>
#include <vector>

#include "gc_json.h"
#include "gc_types.h"

namespace gcb {

constexpr int kFormatVersion = 3;
constexpr int kMinFormatVersion = 1;

struct Expr {
    enum class Kind { Const, Sym, Add, Mul, FloorDiv, Mod, Max, Min };
    Kind kind = Kind::Const;
    int64_t value = 0;  // Const: the value; Sym: the symbol index
    std::vector<Expr> args;

    bool is_const() const { return kind == Kind::Const; }
    int64_t eval(const std::vector<int64_t> &binding) const;
    void symbols(std::vector<bool> &used) const;
};

int64_t floordiv(int64_t a, int64_t b);
int64_t pymod(int64_t a, int64_t b);

struct Symbol {
    std::string name;
    int64_t min = 1, max = 1;
};

struct TensorSpec {
    std::string name;
    Type type = T_F32;
    std::array<int64_t, 4> ne{1, 1, 1, 1};  // for the bound symbols
    std::vector<int64_t> shape;             // PyTorch order, for the bound symbols
    std::array<Expr, 4> ne_x;
    std::vector<Expr> shape_x;
};

struct NodeSpec {
    std::string id;   // "%N"
    std::string op;
    std::vector<std::string> src;  // node ids, stage params "a.N", or GGUF tensors
    Type type = T_F32;
    std::array<int64_t, 4> ne{1, 1, 1, 1};
    std::array<Expr, 4> ne_x;
    Json p;                                            // op parameters as written
    std::vector<std::pair<std::string, Expr>> p_x;     // symbolic parameters (view start, arange)
    std::vector<std::pair<std::string, int64_t>> p_bound;  // their values for the binding
    std::string loc;

    bool has(const char *key) const;
    double pnum(const char *key) const;  // bound value of a parameter; throws if missing
    int64_t pint(const char *key) const;
    float pfloat(const char *key) const { return (float)pnum(key); }
    std::string where() const { return id + " (" + op + ")" + (loc.empty() ? "" : " at " + loc); }
};

struct StageSpec {
    std::string name;
    std::vector<TensorSpec> params;  // "a.0", "a.1", ...
    std::vector<std::string> outputs;
    std::vector<NodeSpec> nodes;     // topological order
    std::vector<bool> uses;          // per symbol: does any shape in the stage read it
    bool symbolic() const {
        for (bool u : uses)
            if (u) return true;
        return false;
    }
};

struct DriverOp {
    enum class Kind { Call, Loop };
    Kind kind = Kind::Call;
    // Call
    std::string stage;
    std::vector<std::string> args, out;
    int call_site = -1;
    // Loop (reference program.h:83-97): carries copied in, then per iteration: scalars, slices,
    // counters, bound symbols, masks, body, collect, until.
    int n = 0;
    int n_symbol = -1;
    std::vector<std::pair<std::string, std::string>> counters;   // (loop value, i32 start value)
    std::vector<std::pair<int, Expr>> bind;                       // (symbol, over symbols + counters)
    std::vector<std::pair<std::string, int>> masks;               // (loop value, counter index)
    std::vector<std::pair<std::string, std::vector<int>>> until;  // (loop value, stop ids)
    std::vector<std::pair<std::string, std::string>> collect;     // (driver value, loop value)
    std::vector<std::pair<std::string, std::string>> carry;       // (loop value, initial value)
    std::vector<std::pair<std::string, std::vector<float>>> scalars;
    std::vector<std::pair<std::string, std::string>> slices;      // (loop value, source [n, ...])
    std::vector<DriverOp> body;
};

struct EntrySpec {
    std::string name;
    std::vector<std::string> inputs, outputs;
    std::vector<DriverOp> driver;
};

struct ProgramSpec {
    int format_version = 0;
    std::vector<Symbol> symbols;
    std::vector<TensorSpec> values;
    std::vector<StageSpec> stages;
    std::vector<EntrySpec> entries;
    std::vector<std::string> state;

    void bind(const std::vector<int64_t> &binding);
    int symbol_index(const std::string &name) const;
};

std::array<int64_t, 4> eval_ne(const TensorSpec &t, const std::vector<int64_t> &binding);
std::vector<int64_t> eval_shape(const TensorSpec &t, const std::vector<int64_t> &binding);
ProgramSpec parse_program(const std::string &json_text);  // throws std::runtime_error
Type parse_type(const std::string &name);

}  // namespace gcb
