// The program a ggml-compiler GGUF carries (metadata key `ggml_compiler.program`, JSON, format
// versions 1 to 3), held the way this executor uses it.
//
// The document's content is fixed by its writer, the reference's emitter
// (ggml_compiler/emit/gguf_runtime.py:117-202; described in docs/ARCHITECTURE.md:227-246): symbols
// with their ranges; driver values with a type, ggml dims `ne` (innermost first) and a PyTorch
// shape; stages whose nodes are ggml ops in topological order; entry points whose drivers call
// stages and run loops; and the names of the state values. Here:
//  - a dim is a DimExpr, a postfix program over the symbol values (an integer, a symbol, or
//    + * // % max min over operands, with Python's floor semantics), so evaluating one binding is a
//    straight pass with no recursion;
//  - each declaration keeps its expressions and, after ProgramSpec::bind, their values for the binding
//    in force, which is all the planner reads;
//  - what the driver names is resolved while reading: a call's stage by index, a loop's trip
//    count, re-bound symbols and mask counters by index, so the executor never looks names up.
#pragma once

#include <array>
#include <cstdint>
#include <memory>
#include <string>
#include <utility>
#include <vector>

#include "gc_json.h"
#include "gc_types.h"

namespace gcb {

constexpr int kFormatVersion = 3;     // symbolic dims, entry points, state
constexpr int kMinFormatVersion = 1;  // 2 added loop slices
constexpr int kMaxSymbols = 64;       // symbols (plus a loop's counters) a dim may read

int64_t floor_div(int64_t a, int64_t b);  // Python's //
int64_t floor_mod(int64_t a, int64_t b);  // Python's %

class DimExpr {
  public:
    DimExpr() : code_{{K, 0, 0}} {}
    explicit DimExpr(int64_t k) : code_{{K, 0, k}} {}
    // From the document: an int, a name among `names` (symbols, then a loop's counters), or
    // [op, operand, ...]. Throws on an unknown name or operator.
    static DimExpr parse(const Json &j, const std::vector<std::string> &names);

    bool is_const() const { return code_.size() == 1 && code_[0].op == K; }
    int64_t eval(const std::vector<int64_t> &vals) const;
    uint64_t reads() const;  // bit k: the expression reads name k

  private:
    enum Op : uint8_t { K, SYM, ADD, MUL, FDIV, MOD, MAX, MIN };
    struct Ins {
        Op op;
        uint16_t argc;  // operands an operator folds (left to right)
        int64_t x;      // K: the constant; SYM: the name's index
    };
    std::vector<Ins> code_;
    static void emit(const Json &j, const std::vector<std::string> &names, std::vector<Ins> &out, int depth);
};

struct Symbol {
    std::string name;
    int64_t min = 1, max = 1;
};

// A driver value or a stage parameter.
struct TensorSpec {
    std::string name;
    Type type = T_F32;
    std::array<DimExpr, 4> ne_expr;
    std::vector<DimExpr> shape_expr;
    uint64_t reads = 0;                     // symbols its dims read
    std::array<int64_t, 4> ne{1, 1, 1, 1};  // at the bound symbols
    std::vector<int64_t> shape;             // PyTorch order, at the bound symbols

    std::array<int64_t, 4> ne_at(const std::vector<int64_t> &binding) const;
    std::vector<int64_t> shape_at(const std::vector<int64_t> &binding) const;
};

struct NodeSpec {
    std::string id;  // "%N"
    std::string op;
    std::vector<std::string> src;  // node ids, stage params "a.N", or GGUF tensors
    Type type = T_F32;
    std::array<DimExpr, 4> ne_expr;
    std::array<int64_t, 4> ne{1, 1, 1, 1};
    Json p;  // op parameters as written
    // parameters that are dims (a view's start, an arange's bounds) and their bound values
    std::vector<std::pair<std::string, DimExpr>> dim_params;
    std::vector<std::pair<std::string, int64_t>> p_bound;
    std::string loc;
    // Optional emitter fusion mark ("<kind>.<n>", kind qkv / glu / head / resid): every node of
    // one group the emitter expects to run as a fused kernel carries the same mark.
    std::string fuse;

    bool has(const char *key) const;
    double pnum(const char *key) const;  // bound value of a parameter; throws if missing
    int64_t pint(const char *key) const;
    float pfloat(const char *key) const { return (float)pnum(key); }
    std::string where() const { return id + " (" + op + ")" + (loc.empty() ? "" : " at " + loc); }

  private:
    double pint_or_num(const char *key, bool as_double) const;
};

struct StageSpec {
    std::string name;
    std::vector<TensorSpec> params;  // "a.0", "a.1", ...
    std::vector<std::string> outputs;
    std::vector<NodeSpec> nodes;
    uint64_t reads = 0;  // symbols any dim of the stage reads
    bool symbolic() const { return reads != 0; }
    bool reads_symbol(size_t k) const { return (reads >> k) & 1u; }
};

struct LoopSpec;

// One driver step: a call of a stage, or a loop.
struct DriverStep {
    bool is_loop = false;
    int stage = -1;  // call: index into ProgramSpec::stages
    std::vector<std::string> args, out;
    int call_site = -1;  // the executor's plan of this call
    std::shared_ptr<LoopSpec> loop;
};

// A loop (format 2+): per iteration i of `trips` (a constant, or a symbol's value at run time):
// counters[k].value := start_k + i (start_k read from counters[k].start once, before iteration 0),
// the re-bound symbols from expressions over the symbols and counters, mask rows for counter
// positions, per-iteration scalars, slice rows, the body, collected rows, then the stop test.
// Carries are copied once before iteration 0.
struct LoopSpec {
    struct Move {
        std::string dst, src;
    };
    struct Counter {
        std::string value, start;
    };
    struct Rebind {
        int symbol;
        DimExpr value;  // over the symbols, then the counters
    };
    struct MaskRow {
        std::string value;
        int counter;
    };
    struct StopIds {
        std::string value;
        std::vector<int32_t> ids;
    };
    struct Scalar {
        std::string value;
        std::vector<float> per_iteration;
    };
    int64_t trips = 0;      // a constant count, or the symbol's max
    int trip_symbol = -1;   // >= 0: the count is this symbol's value
    std::vector<Move> carry, collect, slices;  // collect: dst row i <- src; slices: dst <- src row i
    std::vector<Counter> counters;
    std::vector<Rebind> rebind;
    std::vector<MaskRow> masks;
    std::vector<StopIds> until;
    std::vector<Scalar> scalars;
    std::vector<DriverStep> body;
};

struct EntrySpec {
    std::string name;
    std::vector<std::string> inputs, outputs;
    std::vector<DriverStep> driver;
};

struct ProgramSpec {
    int format_version = 0;
    std::vector<Symbol> symbols;
    std::vector<TensorSpec> values;
    std::vector<StageSpec> stages;
    std::vector<EntrySpec> entries;
    std::vector<std::string> state;

    // Evaluates every dim and dim parameter for `binding` (one value per symbol, each in range).
    void bind(const std::vector<int64_t> &binding);
    int symbol_index(const std::string &name) const;
};

ProgramSpec parse_program(const std::string &json_text);  // throws std::runtime_error
Type parse_type(const std::string &name);

}  // namespace gcb
