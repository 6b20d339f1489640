#include "gguf.h"

#include <cerrno>
#include <cstring>
#include <exception>
#include <fcntl.h>
#include <limits>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <utility>

#include "qkv.h"

namespace qkv {

size_t ggml_type_size(uint32_t type) {
    switch (type) {
        case kGgmlF32: return 4;
        case kGgmlF16: return 2;
        case kGgmlBF16: return 2;
        case kGgmlI8: return 1;
        default: return 0;
    }
}

namespace {

enum GgufValueType : uint32_t {
    kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32 = 6, kBool = 7,
    kString = 8, kArray = 9, kU64 = 10, kI64 = 11, kF64 = 12,
};

size_t scalar_size(uint32_t t) {
    switch (t) {
        case kU8: case kI8: case kBool: return 1;
        case kU16: case kI16: return 2;
        case kU32: case kI32: case kF32: return 4;
        case kU64: case kI64: case kF64: return 8;
        default: return 0;
    }
}

// Bounds-checked little-endian cursor over the mapping.
struct Cursor {
    const uint8_t *p;
    size_t size;
    size_t pos = 0;
    bool ok = true;

    bool take(void *dst, size_t n) {
        if (!ok || n > size - pos) {
            ok = false;
            return false;
        }
        std::memcpy(dst, p + pos, n);
        pos += n;
        return true;
    }
    bool skip(uint64_t n) {
        if (!ok || n > size - pos) {
            ok = false;
            return false;
        }
        pos += static_cast<size_t>(n);
        return true;
    }
    template <typename T> T get() {
        T v{};
        take(&v, sizeof(T));
        return v;
    }
    bool string(std::string *out) {
        const uint64_t n = get<uint64_t>();
        if (!ok || n > size - pos) {
            ok = false;
            return false;
        }
        if (out) out->assign(reinterpret_cast<const char *>(p + pos), static_cast<size_t>(n));
        pos += static_cast<size_t>(n);
        return true;
    }
};

bool read_value(Cursor &c, uint32_t type, GgufValue *v) {
    v->type = type;
    switch (type) {
        case kU8: v->u = c.get<uint8_t>(); v->i = static_cast<int64_t>(v->u); break;
        case kI8: v->i = c.get<int8_t>(); v->u = static_cast<uint64_t>(v->i); break;
        case kU16: v->u = c.get<uint16_t>(); v->i = static_cast<int64_t>(v->u); break;
        case kI16: v->i = c.get<int16_t>(); v->u = static_cast<uint64_t>(v->i); break;
        case kU32: v->u = c.get<uint32_t>(); v->i = static_cast<int64_t>(v->u); break;
        case kI32: v->i = c.get<int32_t>(); v->u = static_cast<uint64_t>(v->i); break;
        case kU64: v->u = c.get<uint64_t>(); v->i = static_cast<int64_t>(v->u); break;
        case kI64: v->i = c.get<int64_t>(); v->u = static_cast<uint64_t>(v->i); break;
        case kF32: v->f = c.get<float>(); break;
        case kF64: v->f = c.get<double>(); break;
        case kBool: v->u = c.get<uint8_t>() ? 1 : 0; break;
        case kString: c.string(&v->s); break;
        case kArray: {
            v->arr_type = c.get<uint32_t>();
            v->arr_n = c.get<uint64_t>();
            if (!c.ok) return false;
            if (v->arr_type == kString) {
                if (v->arr_n > (c.size - c.pos) / 8) return false;   // each string takes at least 8 bytes
                v->strs.resize(static_cast<size_t>(v->arr_n));
                for (uint64_t k = 0; k < v->arr_n && c.ok; ++k) c.string(&v->strs[static_cast<size_t>(k)]);
            } else {
                const size_t es = scalar_size(v->arr_type);
                if (es == 0) return false;  // nested arrays are not used by GGUF writers here
                if (v->arr_n > (std::numeric_limits<uint64_t>::max)() / es) return false;
                c.skip(v->arr_n * es);
            }
            break;
        }
        default: return false;
    }
    return c.ok;
}

}  // namespace

GgufFile::~GgufFile() { close(); }

void GgufFile::close() {
    if (map_) munmap(const_cast<uint8_t *>(map_), size_);
    if (fd_ >= 0) ::close(fd_);
    map_ = nullptr;
    fd_ = -1;
    size_ = 0;
    version_ = 0;
    alignment_ = 32;
    data_offset_ = 0;
    tensors_.clear();
    by_name_.clear();
    kv_.clear();
}

int GgufFile::open(const char *path, std::string *err) {
    // The metadata tables are sized by counts read from the file; a file whose
    // counts fit its size but not host memory fails here instead of throwing
    // through the C entry points that call this.
    try {
        return parse(path, err);
    } catch (const std::exception &ex) {
        close();
        if (err) *err = std::string("gguf: metadata does not fit in host memory (") + ex.what() + ")";
        return QKV_ERR_HOST_MEMORY;
    }
}

int GgufFile::parse(const char *path, std::string *err) {
    close();
    if (!path) {
        if (err) *err = "gguf: path is null";
        return QKV_ERR_INVALID_ARG;
    }
    fd_ = ::open(path, O_RDONLY);
    if (fd_ < 0) {
        if (err) *err = std::string("gguf: cannot open ") + path + ": " + std::strerror(errno);
        return QKV_ERR_IO;
    }
    struct stat st {};
    if (fstat(fd_, &st) != 0 || st.st_size <= 0) {
        if (err) *err = std::string("gguf: cannot stat or empty file: ") + path;
        close();
        return QKV_ERR_IO;
    }
    size_ = static_cast<size_t>(st.st_size);
    void *m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
    if (m == MAP_FAILED) {
        if (err) *err = std::string("gguf: mmap failed: ") + std::strerror(errno);
        size_ = 0;
        close();
        return QKV_ERR_IO;
    }
    map_ = static_cast<const uint8_t *>(m);

    Cursor c{map_, size_};
    char magic[4];
    c.take(magic, 4);
    if (!c.ok || std::memcmp(magic, "GGUF", 4) != 0) {
        if (err) *err = "gguf: bad magic";
        close();
        return QKV_ERR_FORMAT;
    }
    version_ = c.get<uint32_t>();
    if (version_ < 2 || version_ > 3) {
        if (err) *err = "gguf: unsupported version " + std::to_string(version_);
        close();
        return QKV_ERR_FORMAT;
    }
    const uint64_t n_tensors = c.get<uint64_t>();
    const uint64_t n_kv = c.get<uint64_t>();
    // Each KV needs >= 12 bytes and each tensor info >= 24; reject absurd counts early.
    if (!c.ok || n_kv > size_ / 12 || n_tensors > size_ / 24) {
        if (err) *err = "gguf: truncated header or absurd counts";
        close();
        return QKV_ERR_FORMAT;
    }
    for (uint64_t k = 0; k < n_kv; ++k) {
        std::string key;
        c.string(&key);
        const uint32_t type = c.get<uint32_t>();
        GgufValue v;
        if (!c.ok || !read_value(c, type, &v)) {
            if (err) *err = "gguf: bad key/value entry #" + std::to_string(k) + " (" + key + ")";
            close();
            return QKV_ERR_FORMAT;
        }
        kv_[key] = std::move(v);
    }
    auto al = kv_.find("general.alignment");
    if (al != kv_.end()) {
        alignment_ = static_cast<size_t>(al->second.u);
        if (alignment_ == 0 || (alignment_ & (alignment_ - 1)) != 0) {
            if (err) *err = "gguf: general.alignment is not a power of two";
            close();
            return QKV_ERR_FORMAT;
        }
    }
    tensors_.reserve(static_cast<size_t>(n_tensors));
    for (uint64_t t = 0; t < n_tensors; ++t) {
        GgufTensor ti;
        c.string(&ti.name);
        const uint32_t n_dims = c.get<uint32_t>();
        if (!c.ok || n_dims == 0 || n_dims > 4) {
            if (err) *err = "gguf: bad tensor info #" + std::to_string(t);
            close();
            return QKV_ERR_FORMAT;
        }
        uint64_t elems = 1;
        bool overflow = false;
        for (uint32_t d = 0; d < n_dims; ++d) {
            const int64_t ne = c.get<int64_t>();
            if (ne < 0) overflow = true;
            ti.ne.push_back(ne);
            if (ne > 0 && elems > (std::numeric_limits<uint64_t>::max)() / static_cast<uint64_t>(ne)) overflow = true;
            elems *= static_cast<uint64_t>(ne < 0 ? 0 : ne);
        }
        ti.type = c.get<uint32_t>();
        ti.offset = c.get<uint64_t>();
        const size_t es = ggml_type_size(ti.type);
        if (!c.ok || overflow || (es && elems > (std::numeric_limits<uint64_t>::max)() / es)) {
            if (err) *err = "gguf: bad tensor info for " + ti.name;
            close();
            return QKV_ERR_FORMAT;
        }
        ti.nbytes = static_cast<size_t>(elems * es);
        if (by_name_.count(ti.name)) {
            if (err) *err = "gguf: duplicate tensor name " + ti.name;
            close();
            return QKV_ERR_FORMAT;
        }
        by_name_[ti.name] = tensors_.size();
        tensors_.push_back(std::move(ti));
    }
    if (!c.ok) {
        if (err) *err = "gguf: truncated tensor infos";
        close();
        return QKV_ERR_FORMAT;
    }
    data_offset_ = (c.pos + alignment_ - 1) / alignment_ * alignment_;
    if (n_tensors > 0 && data_offset_ > size_) {
        if (err) *err = "gguf: data offset beyond end of file";
        close();
        return QKV_ERR_FORMAT;
    }
    // The same range check as gguf-model.cpp:138-149: offset + nbytes inside the file.
    for (GgufTensor &ti : tensors_) {
        if (ti.offset % alignment_ != 0) {
            if (err) *err = "gguf: misaligned tensor data: " + ti.name;
            close();
            return QKV_ERR_FORMAT;
        }
        if (ti.offset > size_ - data_offset_ || ti.nbytes > size_ - data_offset_ - ti.offset) {
            if (err) *err = "gguf: tensor data extends beyond file: " + ti.name;
            close();
            return QKV_ERR_FORMAT;
        }
        ti.data = map_ + data_offset_ + ti.offset;
    }
    return QKV_OK;
}

const GgufTensor *GgufFile::find(const std::string &name) const {
    auto it = by_name_.find(name);
    return it == by_name_.end() ? nullptr : &tensors_[it->second];
}

const GgufValue *GgufFile::value(const std::string &key) const {
    auto it = kv_.find(key);
    return it == kv_.end() ? nullptr : &it->second;
}

bool GgufFile::get_u32(const std::string &key, uint32_t *out) const {
    const GgufValue *v = value(key);
    if (!v || v->type != kU32) return false;
    *out = static_cast<uint32_t>(v->u);
    return true;
}

bool GgufFile::get_f32(const std::string &key, float *out) const {
    const GgufValue *v = value(key);
    if (!v || v->type != kF32) return false;
    *out = static_cast<float>(v->f);
    return true;
}

bool GgufFile::get_str(const std::string &key, std::string *out) const {
    const GgufValue *v = value(key);
    if (!v || v->type != kString) return false;
    *out = v->s;
    return true;
}

}  // namespace qkv
