// Minimal GGUF (v2/v3) reader: mmap + bounds-checked key/value and tensor-info
// parsing.  Stands in for GGML's gguf parser, which the reference reaches
// through src/gguf-model.cpp:164-245 (open, tensor_by_name) and
// src/native-model.cpp:157-279 (metadata keys).  Written from the public GGUF
// format description: header, KV section, tensor infos, aligned data section.
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace qkv {

enum GgmlType : uint32_t {
    kGgmlF32 = 0,
    kGgmlF16 = 1,
    kGgmlI8 = 24,      // one byte per element; e4m3 codes in the FP8 projection files
    kGgmlBF16 = 30,
};

struct GgufTensor {
    std::string name;
    uint32_t type = 0;
    std::vector<int64_t> ne;   // GGML order: ne[0] is the innermost (contiguous) dimension
    uint64_t offset = 0;       // relative to the data section
    size_t nbytes = 0;         // 0 when the type is not a plain float type
    const uint8_t *data = nullptr;
};

struct GgufValue {
    uint32_t type = 0;
    uint64_t u = 0;
    int64_t i = 0;
    double f = 0.0;
    std::string s;
    uint32_t arr_type = 0;
    uint64_t arr_n = 0;
    std::vector<std::string> strs;   // string arrays (tokenizer vocabulary and merges)
};

class GgufFile {
public:
    GgufFile() = default;
    ~GgufFile();
    GgufFile(const GgufFile &) = delete;
    GgufFile &operator=(const GgufFile &) = delete;

    // 0 on success, else a qkv_status code with *err set.
    int open(const char *path, std::string *err);
    void close();

    const GgufTensor *find(const std::string &name) const;
    const GgufValue *value(const std::string &key) const;
    bool get_u32(const std::string &key, uint32_t *out) const;
    bool get_f32(const std::string &key, float *out) const;
    bool get_str(const std::string &key, std::string *out) const;

    const std::vector<GgufTensor> &tensors() const { return tensors_; }
    uint32_t version() const { return version_; }
    size_t alignment() const { return alignment_; }
    size_t data_offset() const { return data_offset_; }
    size_t file_size() const { return size_; }
    const uint8_t *mapping() const { return map_; }

private:
    int parse(const char *path, std::string *err);

    int fd_ = -1;
    const uint8_t *map_ = nullptr;
    size_t size_ = 0;
    uint32_t version_ = 0;
    size_t alignment_ = 32;
    size_t data_offset_ = 0;
    std::vector<GgufTensor> tensors_;
    std::map<std::string, size_t> by_name_;
    std::map<std::string, GgufValue> kv_;
};

// Bytes per element of a plain float GGML type, 0 otherwise.
size_t ggml_type_size(uint32_t type);

}  // namespace qkv
