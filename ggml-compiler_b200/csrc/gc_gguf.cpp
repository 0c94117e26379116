#include "gc_gguf.h"

#include <cstdio>
#include <cstring>
#include <memory>
#include <stdexcept>

namespace gcb {

namespace {

enum : uint32_t {
    G_U8 = 0, G_I8 = 1, G_U16 = 2, G_I16 = 3, G_U32 = 4, G_I32 = 5, G_F32 = 6, G_BOOL = 7,
    G_STRING = 8, G_ARRAY = 9, G_U64 = 10, G_I64 = 11, G_F64 = 12,
};

struct Closer {
    void operator()(FILE *f) const { std::fclose(f); }
};

class Reader {
  public:
    Reader(FILE *f, uint64_t size) : f_(f), size_(size) {}
    uint64_t pos() const { return pos_; }

    void read(void *dst, size_t n) {
        if (pos_ + n > size_ || std::fread(dst, 1, n, f_) != n) throw std::runtime_error("truncated GGUF header");
        pos_ += n;
    }
    void skip(uint64_t n) {
        if (pos_ + n > size_) throw std::runtime_error("truncated GGUF header");
        if (std::fseek(f_, (long)n, SEEK_CUR) != 0) throw std::runtime_error("seek failed in GGUF header");
        pos_ += n;
    }
    template <class T> T get() {
        T v;
        read(&v, sizeof v);
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (n > size_ - pos_) throw std::runtime_error("truncated GGUF header: a string runs past the end of the file");
        std::string s(n, '\0');
        if (n) read(&s[0], n);
        return s;
    }

  private:
    FILE *f_;
    uint64_t size_, pos_ = 0;
};

size_t scalar_size(uint32_t t) {
    switch (t) {
        case G_U8: case G_I8: case G_BOOL: return 1;
        case G_U16: case G_I16: return 2;
        case G_U32: case G_I32: case G_F32: return 4;
        case G_U64: case G_I64: case G_F64: return 8;
        default: return 0;
    }
}

}  // namespace

void GgufFile::open(const std::string &path) {
    path_ = path;
    std::unique_ptr<FILE, Closer> f(std::fopen(path.c_str(), "rb"));
    if (!f) throw std::runtime_error("cannot read GGUF '" + path + "'");
    if (std::fseek(f.get(), 0, SEEK_END) != 0) throw std::runtime_error("cannot seek in '" + path + "'");
    const long sz = std::ftell(f.get());
    if (sz < 0) throw std::runtime_error("cannot size '" + path + "'");
    file_size_ = (uint64_t)sz;
    std::fseek(f.get(), 0, SEEK_SET);
    Reader r(f.get(), file_size_);

    char magic[4];
    r.read(magic, 4);
    if (std::memcmp(magic, "GGUF", 4) != 0) throw std::runtime_error("'" + path + "' is not a GGUF file");
    version_ = r.get<uint32_t>();
    if (version_ < 2 || version_ > 3) throw std::runtime_error("GGUF version " + std::to_string(version_) + " is not supported");
    const uint64_t n_tensors = r.get<uint64_t>();
    const uint64_t n_kv = r.get<uint64_t>();
    if (n_tensors > (1u << 24) || n_kv > (1u << 24)) throw std::runtime_error("GGUF header counts are implausible");

    for (uint64_t i = 0; i < n_kv; i++) {
        const std::string key = r.str();
        const uint32_t t = r.get<uint32_t>();
        if (t == G_STRING) {
            strings_[key] = r.str();
        } else if (t == G_ARRAY) {
            const uint32_t et = r.get<uint32_t>();
            const uint64_t n = r.get<uint64_t>();
            if (et == G_STRING) {
                for (uint64_t k = 0; k < n; k++) (void)r.str();
            } else {
                const size_t es = scalar_size(et);
                if (!es) throw std::runtime_error("GGUF key '" + key + "' has an array of unknown type");
                if (n > file_size_ / es) throw std::runtime_error("truncated GGUF header");
                r.skip(n * es);
            }
        } else {
            const size_t es = scalar_size(t);
            if (!es) throw std::runtime_error("GGUF key '" + key + "' has unknown type " + std::to_string(t));
            uint64_t v = 0;
            r.read(&v, es);
            ints_[key] = v;
        }
    }

    for (uint64_t i = 0; i < n_tensors; i++) {
        GgufTensor t;
        t.name = r.str();
        const uint32_t nd = r.get<uint32_t>();
        if (nd > 4) throw std::runtime_error("GGUF tensor '" + t.name + "' has more than 4 dims");
        t.n_dims = (int)nd;
        for (uint32_t d = 0; d < nd; d++) {
            const uint64_t v = r.get<uint64_t>();
            if (v == 0 || v > (1ull << 40)) throw std::runtime_error("GGUF tensor '" + t.name + "' has a bad dim");
            t.ne[d] = (int64_t)v;
        }
        const uint32_t ty = r.get<uint32_t>();
        const TypeTraits *tr = type_traits((Type)ty);
        if (!tr) throw std::runtime_error("GGUF tensor '" + t.name + "' has unknown type " + std::to_string(ty));
        t.type = (Type)ty;
        t.offset = r.get<uint64_t>();
        if (t.ne[0] % tr->block) throw std::runtime_error("GGUF tensor '" + t.name + "' row is not whole blocks");
        t.nbytes = row_size(t.type, t.ne[0]) * (size_t)(t.ne[1] * t.ne[2] * t.ne[3]);
        if (by_name_.count(t.name)) throw std::runtime_error("GGUF has tensor '" + t.name + "' twice");
        by_name_[t.name] = tensors_.size();
        tensors_.push_back(std::move(t));
    }

    uint64_t align = 32;
    auto it = ints_.find("general.alignment");
    if (it != ints_.end() && it->second > 0) align = it->second;
    data_offset_ = (r.pos() + align - 1) / align * align;
    for (const auto &t : tensors_) {
        if (t.offset % align) throw std::runtime_error("GGUF tensor '" + t.name + "' is misaligned");
        if (data_offset_ + t.offset + t.nbytes > file_size_)
            throw std::runtime_error("GGUF tensor '" + t.name + "' runs past the end of the file (truncated GGUF)");
    }
}

const GgufTensor *GgufFile::tensor(const std::string &name) const {
    auto it = by_name_.find(name);
    return it == by_name_.end() ? nullptr : &tensors_[it->second];
}

const std::string *GgufFile::get_string(const std::string &key) const {
    auto it = strings_.find(key);
    return it == strings_.end() ? nullptr : &it->second;
}

bool GgufFile::get_u32(const std::string &key, uint32_t *out) const {
    auto it = ints_.find(key);
    if (it == ints_.end()) return false;
    *out = (uint32_t)it->second;
    return true;
}

}  // namespace gcb
