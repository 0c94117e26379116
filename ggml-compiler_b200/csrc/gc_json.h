// A small JSON reader for the `ggml_compiler.program` document (the program JSON the reference's
// emitter writes, ggml_compiler/emit/gguf_runtime.py:117-202). Numbers keep their JSON kind:
// integers as int64, anything with a fraction or exponent as double (strtod, correctly rounded).
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace gcb {

class Json {
  public:
    enum Kind { Null, Bool, Int, Float, String, Array, Object };

    Kind kind() const { return kind_; }
    bool is_null() const { return kind_ == Null; }
    bool is_int() const { return kind_ == Int; }
    bool is_number() const { return kind_ == Int || kind_ == Float; }
    bool is_string() const { return kind_ == String; }
    bool is_array() const { return kind_ == Array; }
    bool is_object() const { return kind_ == Object; }

    int64_t as_int() const;          // Int, or a Float (truncated), else throws
    double as_double() const;        // any number
    float as_float() const { return (float)as_double(); }
    bool as_bool() const;
    const std::string &as_string() const;
    const std::vector<Json> &items() const;  // Array
    const std::vector<std::pair<std::string, Json>> &members() const;  // Object

    size_t size() const;
    const Json &operator[](size_t i) const;
    const Json *find(const std::string &key) const;  // nullptr if absent or not an object
    const Json &at(const std::string &key) const;    // throws if absent
    bool contains(const std::string &key) const { return find(key) != nullptr; }
    std::string dump() const;

    static Json parse(const std::string &text);
    static Json make_int(int64_t v) {
        Json j;
        j.kind_ = Int;
        j.i_ = v;
        return j;
    }

  private:
    Kind kind_ = Null;
    bool b_ = false;
    int64_t i_ = 0;
    double f_ = 0.0;
    std::string s_;
    std::vector<Json> a_;
    std::vector<std::pair<std::string, Json>> o_;
    friend class JsonParser;
};

}  // namespace gcb
