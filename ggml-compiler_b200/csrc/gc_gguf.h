// GGUF reader: header, key/value metadata, tensor infos and the aligned data section.
// Replaces the ggml C reader the reference runtime calls (gguf_init_from_file and friends,
// runtime/src/ggml_compiler_rt.cpp:255-267 and :445-479). Only GGUF versions 2 and 3 (64-bit
// counts) are read; every length and offset is checked against the file size.
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

#include "gc_types.h"

namespace gcb {

struct GgufTensor {
    std::string name;
    Type type = T_F32;
    int64_t ne[4] = {1, 1, 1, 1};  // innermost first
    int n_dims = 0;
    uint64_t offset = 0;  // from the start of the data section
    size_t nbytes = 0;
};

class GgufFile {
  public:
    void open(const std::string &path);  // throws std::runtime_error

    const std::string &path() const { return path_; }
    uint32_t version() const { return version_; }
    uint64_t data_offset() const { return data_offset_; }
    uint64_t file_size() const { return file_size_; }
    const std::vector<GgufTensor> &tensors() const { return tensors_; }
    const GgufTensor *tensor(const std::string &name) const;
    // String metadata value, or nullptr if the key is absent or not a string.
    const std::string *get_string(const std::string &key) const;
    bool get_u32(const std::string &key, uint32_t *out) const;

  private:
    std::string path_;
    uint32_t version_ = 0;
    uint64_t data_offset_ = 0, file_size_ = 0;
    std::vector<GgufTensor> tensors_;
    std::map<std::string, size_t> by_name_;
    std::map<std::string, std::string> strings_;
    std::map<std::string, uint64_t> ints_;
};

}  // namespace gcb
