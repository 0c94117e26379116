#include "gc_json.h"

#include <cerrno>
#include <cstdlib>
#include <cstring>

namespace gcb {

class JsonParser {
  public:
    explicit JsonParser(const std::string &t) : s_(t.data()), n_(t.size()) {}

    Json parse_document() {
        Json v = value(0);
        ws();
        if (p_ != n_) fail("trailing characters");
        return v;
    }

  private:
    const char *s_;
    size_t n_, p_ = 0;

    [[noreturn]] void fail(const char *what) {
        throw std::runtime_error(std::string("JSON: ") + what + " at offset " + std::to_string(p_));
    }
    void ws() {
        while (p_ < n_ && (s_[p_] == ' ' || s_[p_] == '\n' || s_[p_] == '\t' || s_[p_] == '\r')) p_++;
    }
    bool lit(const char *w) {
        size_t k = std::strlen(w);
        if (p_ + k <= n_ && std::memcmp(s_ + p_, w, k) == 0) {
            p_ += k;
            return true;
        }
        return false;
    }
    Json value(int depth) {
        if (depth > 512) fail("nesting too deep");
        ws();
        if (p_ >= n_) fail("unexpected end");
        Json j;
        const char c = s_[p_];
        if (c == '{') {
            p_++;
            j.kind_ = Json::Object;
            ws();
            if (p_ < n_ && s_[p_] == '}') {
                p_++;
                return j;
            }
            for (;;) {
                ws();
                if (p_ >= n_ || s_[p_] != '"') fail("expected a key");
                std::string k = str();
                ws();
                if (p_ >= n_ || s_[p_] != ':') fail("expected ':'");
                p_++;
                j.o_.emplace_back(std::move(k), value(depth + 1));
                ws();
                if (p_ < n_ && s_[p_] == ',') {
                    p_++;
                    continue;
                }
                if (p_ < n_ && s_[p_] == '}') {
                    p_++;
                    return j;
                }
                fail("expected ',' or '}'");
            }
        }
        if (c == '[') {
            p_++;
            j.kind_ = Json::Array;
            ws();
            if (p_ < n_ && s_[p_] == ']') {
                p_++;
                return j;
            }
            for (;;) {
                j.a_.push_back(value(depth + 1));
                ws();
                if (p_ < n_ && s_[p_] == ',') {
                    p_++;
                    continue;
                }
                if (p_ < n_ && s_[p_] == ']') {
                    p_++;
                    return j;
                }
                fail("expected ',' or ']'");
            }
        }
        if (c == '"') {
            j.kind_ = Json::String;
            j.s_ = str();
            return j;
        }
        if (lit("true")) {
            j.kind_ = Json::Bool;
            j.b_ = true;
            return j;
        }
        if (lit("false")) {
            j.kind_ = Json::Bool;
            return j;
        }
        if (lit("null")) return j;
        if (lit("NaN")) {  // Python's json writes these for non-finite floats
            j.kind_ = Json::Float;
            j.f_ = __builtin_nan("");
            return j;
        }
        if (lit("Infinity")) {
            j.kind_ = Json::Float;
            j.f_ = __builtin_inf();
            return j;
        }
        if (lit("-Infinity")) {
            j.kind_ = Json::Float;
            j.f_ = -__builtin_inf();
            return j;
        }
        return number();
    }
    Json number() {
        const size_t start = p_;
        bool frac = false;
        if (p_ < n_ && (s_[p_] == '-' || s_[p_] == '+')) p_++;
        while (p_ < n_) {
            const char c = s_[p_];
            if (c >= '0' && c <= '9') {
                p_++;
            } else if (c == '.' || c == 'e' || c == 'E' || ((c == '-' || c == '+') && (s_[p_ - 1] == 'e' || s_[p_ - 1] == 'E'))) {
                frac = true;
                p_++;
            } else {
                break;
            }
        }
        if (p_ == start) fail("unexpected character");
        std::string tok(s_ + start, p_ - start);
        Json j;
        if (!frac) {
            errno = 0;
            char *end = nullptr;
            long long v = std::strtoll(tok.c_str(), &end, 10);
            if (errno == 0 && end && *end == 0) {
                j.kind_ = Json::Int;
                j.i_ = v;
                return j;
            }
        }
        char *end = nullptr;
        j.f_ = std::strtod(tok.c_str(), &end);
        if (!end || *end != 0) fail("malformed number");
        j.kind_ = Json::Float;
        return j;
    }
    static void put_utf8(std::string &o, uint32_t cp) {
        if (cp < 0x80) {
            o += (char)cp;
        } else if (cp < 0x800) {
            o += (char)(0xc0 | (cp >> 6));
            o += (char)(0x80 | (cp & 0x3f));
        } else if (cp < 0x10000) {
            o += (char)(0xe0 | (cp >> 12));
            o += (char)(0x80 | ((cp >> 6) & 0x3f));
            o += (char)(0x80 | (cp & 0x3f));
        } else {
            o += (char)(0xf0 | (cp >> 18));
            o += (char)(0x80 | ((cp >> 12) & 0x3f));
            o += (char)(0x80 | ((cp >> 6) & 0x3f));
            o += (char)(0x80 | (cp & 0x3f));
        }
    }
    uint32_t hex4() {
        if (p_ + 4 > n_) fail("short \\u escape");
        uint32_t v = 0;
        for (int i = 0; i < 4; i++) {
            const char c = s_[p_++];
            v <<= 4;
            if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
            else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
            else fail("bad \\u escape");
        }
        return v;
    }
    std::string str() {
        p_++;  // opening quote
        std::string o;
        while (p_ < n_) {
            const char c = s_[p_++];
            if (c == '"') return o;
            if (c != '\\') {
                o += c;
                continue;
            }
            if (p_ >= n_) break;
            const char e = s_[p_++];
            switch (e) {
                case '"': o += '"'; break;
                case '\\': o += '\\'; break;
                case '/': o += '/'; break;
                case 'b': o += '\b'; break;
                case 'f': o += '\f'; break;
                case 'n': o += '\n'; break;
                case 'r': o += '\r'; break;
                case 't': o += '\t'; break;
                case 'u': {
                    uint32_t cp = hex4();
                    if (cp >= 0xd800 && cp < 0xdc00 && p_ + 6 <= n_ && s_[p_] == '\\' && s_[p_ + 1] == 'u') {
                        p_ += 2;
                        const uint32_t lo = hex4();
                        cp = 0x10000 + ((cp - 0xd800) << 10) + (lo - 0xdc00);
                    }
                    put_utf8(o, cp);
                    break;
                }
                default: fail("bad escape");
            }
        }
        fail("unterminated string");
    }
};

Json Json::parse(const std::string &text) { return JsonParser(text).parse_document(); }

int64_t Json::as_int() const {
    if (kind_ == Int) return i_;
    if (kind_ == Float) return (int64_t)f_;
    if (kind_ == Bool) return b_ ? 1 : 0;
    throw std::runtime_error("JSON value is not a number: " + dump());
}

double Json::as_double() const {
    if (kind_ == Float) return f_;
    if (kind_ == Int) return (double)i_;
    if (kind_ == Bool) return b_ ? 1.0 : 0.0;
    throw std::runtime_error("JSON value is not a number: " + dump());
}

bool Json::as_bool() const {
    if (kind_ == Bool) return b_;
    if (kind_ == Int) return i_ != 0;
    throw std::runtime_error("JSON value is not a boolean: " + dump());
}

const std::string &Json::as_string() const {
    if (kind_ != String) throw std::runtime_error("JSON value is not a string: " + dump());
    return s_;
}

const std::vector<Json> &Json::items() const {
    if (kind_ != Array) throw std::runtime_error("JSON value is not an array: " + dump());
    return a_;
}

const std::vector<std::pair<std::string, Json>> &Json::members() const {
    if (kind_ != Object) throw std::runtime_error("JSON value is not an object: " + dump());
    return o_;
}

size_t Json::size() const {
    if (kind_ == Array) return a_.size();
    if (kind_ == Object) return o_.size();
    return 0;
}

const Json &Json::operator[](size_t i) const {
    if (kind_ != Array || i >= a_.size()) throw std::runtime_error("JSON index out of range in " + dump());
    return a_[i];
}

const Json *Json::find(const std::string &key) const {
    if (kind_ != Object) return nullptr;
    for (const auto &kv : o_)
        if (kv.first == key) return &kv.second;
    return nullptr;
}

const Json &Json::at(const std::string &key) const {
    const Json *j = find(key);
    if (!j) throw std::runtime_error("missing key '" + key + "'");
    return *j;
}

std::string Json::dump() const {
    switch (kind_) {
        case Null: return "null";
        case Bool: return b_ ? "true" : "false";
        case Int: return std::to_string(i_);
        case Float: {
            char buf[64];
            std::snprintf(buf, sizeof buf, "%.17g", f_);
            return buf;
        }
        case String: return "\"" + s_ + "\"";
        case Array: {
            std::string o = "[";
            for (size_t i = 0; i < a_.size(); i++) o += (i ? "," : "") + a_[i].dump();
            return o + "]";
        }
        case Object: {
            std::string o = "{";
            for (size_t i = 0; i < o_.size(); i++) o += (i ? ",\"" : "\"") + o_[i].first + "\":" + o_[i].second.dump();
            return o + "}";
        }
    }
    return "";
}

}  // namespace gcb
