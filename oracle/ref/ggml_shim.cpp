// Test infrastructure: definitions behind oracle/ref/include/*.h.
// - The GGUF reader is a small, independent parser of the public GGUF v2/v3
//   layout (header, key/values, tensor infos, aligned data); it fills a
//   metadata context with one ggml_tensor per GGUF tensor (type, ne, nb, name).
// - Graph and backend functions are stubs returning null / failure: the
//   reference's GGML paths report an error, its scalar CPU paths work.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "ggml-backend.h"
#include "ggml-cpu.h"
#include "ggml.h"
#include "gguf.h"

struct ggml_context {
    bool no_alloc = true;
    std::vector<ggml_tensor *> tensors;
};

struct gguf_context {
    std::vector<std::string> names;
    std::vector<size_t> offsets;
    size_t data_offset = 0;
    // metadata: every key, with its u32 value (scalar u32 keys) and its
    // strings (string arrays); other values are skipped
    std::vector<std::string> keys;
    std::vector<uint32_t> u32;
    std::vector<std::vector<std::string>> strs;
    std::vector<size_t> arr_n;
};

static size_t type_size(ggml_type t) {
    switch (t) {
        case GGML_TYPE_F32: case GGML_TYPE_I32: return 4;
        case GGML_TYPE_F16: case GGML_TYPE_BF16: return 2;
        default: return 0;
    }
}

namespace {
struct Rd {
    FILE *f;
    bool ok = true;
    template <typename T> T get() {
        T v{};
        if (ok && std::fread(&v, sizeof(T), 1, f) != 1) ok = false;
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || n > (1u << 30)) { ok = false; return {}; }
        std::string s(n, '\0');
        if (n && std::fread(&s[0], 1, n, f) != n) ok = false;
        return s;
    }
    void skip(uint64_t n) {
        if (ok && std::fseek(f, static_cast<long>(n), SEEK_CUR) != 0) ok = false;
    }
};
size_t scalar_bytes(uint32_t t) {
    static const size_t sz[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    return t < 13 ? sz[t] : 0;
}
}  // namespace

extern "C" {

ggml_context *ggml_init(ggml_init_params params) {
    ggml_context *c = new ggml_context();
    c->no_alloc = params.no_alloc;
    return c;
}

void ggml_free(ggml_context *ctx) {
    if (!ctx) return;
    for (ggml_tensor *t : ctx->tensors) {
        if (!ctx->no_alloc) std::free(t->data);
        delete t;
    }
    delete ctx;
}

size_t ggml_tensor_overhead(void) { return sizeof(ggml_tensor) + 64; }
size_t ggml_graph_overhead_custom(size_t size, bool) { return size * 16 + 256; }

size_t ggml_nbytes(const ggml_tensor *t) {
    size_t n = type_size(t->type);
    for (int i = 0; i < GGML_MAX_DIMS; ++i) n *= static_cast<size_t>(t->ne[i]);
    return n;
}

int ggml_n_dims(const ggml_tensor *t) {
    for (int i = GGML_MAX_DIMS - 1; i >= 1; --i) {
        if (t->ne[i] > 1) return i + 1;
    }
    return 1;
}

ggml_tensor *ggml_get_tensor(ggml_context *ctx, const char *name) {
    if (!ctx || !name) return nullptr;
    for (ggml_tensor *t : ctx->tensors) {
        if (std::strcmp(t->name, name) == 0) return t;
    }
    return nullptr;
}

float *ggml_get_data_f32(const ggml_tensor *t) { return t ? static_cast<float *>(t->data) : nullptr; }

ggml_tensor *ggml_new_tensor(ggml_context *ctx, ggml_type type, int n_dims, const int64_t *ne) {
    ggml_tensor *t = new ggml_tensor();
    t->type = type;
    for (int i = 0; i < GGML_MAX_DIMS; ++i) t->ne[i] = i < n_dims ? ne[i] : 1;
    t->nb[0] = type_size(type);
    for (int i = 1; i < GGML_MAX_DIMS; ++i) t->nb[i] = t->nb[i - 1] * static_cast<size_t>(t->ne[i - 1]);
    t->data = (ctx && !ctx->no_alloc) ? std::calloc(1, ggml_nbytes(t) + 1) : nullptr;
    t->name[0] = '\0';
    if (ctx) ctx->tensors.push_back(t);
    return t;
}
ggml_tensor *ggml_new_tensor_1d(ggml_context *ctx, ggml_type type, int64_t ne0) {
    const int64_t ne[1] = {ne0};
    return ggml_new_tensor(ctx, type, 1, ne);
}
ggml_tensor *ggml_new_tensor_2d(ggml_context *ctx, ggml_type type, int64_t ne0, int64_t ne1) {
    const int64_t ne[2] = {ne0, ne1};
    return ggml_new_tensor(ctx, type, 2, ne);
}
ggml_tensor *ggml_new_tensor_3d(ggml_context *ctx, ggml_type type, int64_t ne0, int64_t ne1, int64_t ne2) {
    const int64_t ne[3] = {ne0, ne1, ne2};
    return ggml_new_tensor(ctx, type, 3, ne);
}
ggml_tensor *ggml_set_name(ggml_tensor *t, const char *name) {
    if (t && name) {
        std::strncpy(t->name, name, sizeof(t->name) - 1);
        t->name[sizeof(t->name) - 1] = '\0';
    }
    return t;
}
void ggml_set_input(ggml_tensor *) {}
void ggml_set_output(ggml_tensor *) {}

// ---- graph ops: not available in this shim ----
ggml_tensor *ggml_mul_mat(ggml_context *, ggml_tensor *, ggml_tensor *) { return nullptr; }
void ggml_mul_mat_set_prec(ggml_tensor *, ggml_prec) {}
ggml_tensor *ggml_mul(ggml_context *, ggml_tensor *, ggml_tensor *) { return nullptr; }
ggml_tensor *ggml_add(ggml_context *, ggml_tensor *, ggml_tensor *) { return nullptr; }
ggml_tensor *ggml_rms_norm(ggml_context *, ggml_tensor *, float) { return nullptr; }
ggml_tensor *ggml_silu(ggml_context *, ggml_tensor *) { return nullptr; }
ggml_tensor *ggml_cont(ggml_context *, ggml_tensor *) { return nullptr; }
ggml_tensor *ggml_cpy(ggml_context *, ggml_tensor *, ggml_tensor *) { return nullptr; }
ggml_tensor *ggml_transpose(ggml_context *, ggml_tensor *) { return nullptr; }
ggml_tensor *ggml_permute(ggml_context *, ggml_tensor *, int, int, int, int) { return nullptr; }
ggml_tensor *ggml_reshape_2d(ggml_context *, ggml_tensor *, int64_t, int64_t) { return nullptr; }
ggml_tensor *ggml_reshape_3d(ggml_context *, ggml_tensor *, int64_t, int64_t, int64_t) { return nullptr; }
ggml_tensor *ggml_view_2d(ggml_context *, ggml_tensor *, int64_t, int64_t, size_t, size_t) { return nullptr; }
ggml_tensor *ggml_view_3d(ggml_context *, ggml_tensor *, int64_t, int64_t, int64_t, size_t, size_t, size_t) { return nullptr; }
ggml_tensor *ggml_diag_mask_inf(ggml_context *, ggml_tensor *, int) { return nullptr; }
ggml_tensor *ggml_soft_max_ext(ggml_context *, ggml_tensor *, ggml_tensor *, float, float) { return nullptr; }
ggml_tensor *ggml_rope_ext(ggml_context *, ggml_tensor *, ggml_tensor *, ggml_tensor *, int, int, int, float, float, float,
                           float, float, float) {
    return nullptr;
}
ggml_cgraph *ggml_new_graph(ggml_context *) { return nullptr; }
ggml_cgraph *ggml_new_graph_custom(ggml_context *, size_t, bool) { return nullptr; }
void ggml_build_forward_expand(ggml_cgraph *, ggml_tensor *) {}
ggml_status ggml_graph_compute_with_ctx(ggml_context *, ggml_cgraph *, int) { return GGML_STATUS_FAILED; }

// ---- backends: none ----
void ggml_backend_tensor_set(ggml_tensor *, const void *, size_t, size_t) {}
void ggml_backend_tensor_get(const ggml_tensor *, void *, size_t, size_t) {}
ggml_backend_sched_t ggml_backend_sched_new(ggml_backend_t *, ggml_backend_buffer_type_t *, int, size_t, bool, bool) {
    return nullptr;
}
void ggml_backend_sched_free(ggml_backend_sched_t) {}
void ggml_backend_sched_reset(ggml_backend_sched_t) {}
bool ggml_backend_sched_alloc_graph(ggml_backend_sched_t, ggml_cgraph *) { return false; }
ggml_status ggml_backend_sched_graph_compute(ggml_backend_sched_t, ggml_cgraph *) { return GGML_STATUS_FAILED; }
ggml_backend_buffer_t ggml_backend_alloc_ctx_tensors(ggml_context *, ggml_backend_t) { return nullptr; }
void ggml_backend_buffer_free(ggml_backend_buffer_t) {}
void ggml_backend_buffer_set_usage(ggml_backend_buffer_t, ggml_backend_buffer_usage) {}
void ggml_backend_buffer_clear(ggml_backend_buffer_t, uint8_t) {}
void ggml_backend_free(ggml_backend_t) {}
ggml_backend_t ggml_backend_init_by_type(enum ggml_backend_dev_type, const char *) { return nullptr; }
const char *ggml_backend_name(ggml_backend_t) { return "none"; }
ggml_backend_dev_t ggml_backend_get_device(ggml_backend_t) { return nullptr; }
enum ggml_backend_dev_type ggml_backend_dev_type(ggml_backend_dev_t) { return GGML_BACKEND_DEVICE_TYPE_CPU; }
ggml_backend_t ggml_backend_cpu_init(void) { return nullptr; }
void ggml_backend_cpu_set_n_threads(ggml_backend_t, int) {}

// ---- GGUF ----

gguf_context *gguf_init_from_file(const char *fname, gguf_init_params params) {
    FILE *f = std::fopen(fname, "rb");
    if (!f) return nullptr;
    Rd r{f};
    char magic[4];
    if (std::fread(magic, 1, 4, f) != 4 || std::memcmp(magic, "GGUF", 4) != 0) { std::fclose(f); return nullptr; }
    const uint32_t version = r.get<uint32_t>();
    const uint64_t n_tensors = r.get<uint64_t>();
    const uint64_t n_kv = r.get<uint64_t>();
    if (!r.ok || version < 2 || version > 3) { std::fclose(f); return nullptr; }
    size_t alignment = 32;
    gguf_context *g = new gguf_context();
    for (uint64_t i = 0; i < n_kv && r.ok; ++i) {
        const std::string key = r.str();
        const uint32_t t = r.get<uint32_t>();
        uint32_t u = 0;
        size_t an = 0;
        std::vector<std::string> strs;
        if (t == 8) {
            r.str();
        } else if (t == 9) {
            const uint32_t at = r.get<uint32_t>();
            const uint64_t n = r.get<uint64_t>();
            an = static_cast<size_t>(n);
            if (at == 8) { for (uint64_t k = 0; k < n && r.ok; ++k) strs.push_back(r.str()); }
            else if (scalar_bytes(at)) r.skip(n * scalar_bytes(at));
            else r.ok = false;
        } else if (t == 4) {
            u = r.get<uint32_t>();
            if (key == "general.alignment") alignment = u;
        } else if (scalar_bytes(t)) {
            r.skip(scalar_bytes(t));
        } else {
            r.ok = false;
        }
        g->keys.push_back(key);
        g->u32.push_back(u);
        g->strs.push_back(std::move(strs));
        g->arr_n.push_back(an);
    }
    ggml_context *meta = ggml_init({0, nullptr, true});
    for (uint64_t i = 0; i < n_tensors && r.ok; ++i) {
        const std::string name = r.str();
        const uint32_t nd = r.get<uint32_t>();
        if (nd == 0 || nd > 4) { r.ok = false; break; }
        int64_t ne[4] = {1, 1, 1, 1};
        for (uint32_t d = 0; d < nd; ++d) ne[d] = static_cast<int64_t>(r.get<uint64_t>());
        const uint32_t type = r.get<uint32_t>();
        const uint64_t off = r.get<uint64_t>();
        ggml_tensor *t = ggml_new_tensor(meta, static_cast<ggml_type>(type), static_cast<int>(nd), ne);
        ggml_set_name(t, name.c_str());
        g->names.push_back(name);
        g->offsets.push_back(static_cast<size_t>(off));
    }
    const long pos = std::ftell(f);
    std::fclose(f);
    if (!r.ok || pos < 0) {
        ggml_free(meta);
        delete g;
        return nullptr;
    }
    g->data_offset = (static_cast<size_t>(pos) + alignment - 1) / alignment * alignment;
    if (params.ctx) *params.ctx = meta;
    else ggml_free(meta);
    return g;
}

void gguf_free(gguf_context *ctx) { delete ctx; }
int64_t gguf_get_n_tensors(const gguf_context *ctx) { return ctx ? static_cast<int64_t>(ctx->names.size()) : 0; }
const char *gguf_get_tensor_name(const gguf_context *ctx, int64_t id) {
    return (ctx && id >= 0 && id < static_cast<int64_t>(ctx->names.size())) ? ctx->names[static_cast<size_t>(id)].c_str() : nullptr;
}
size_t gguf_get_tensor_offset(const gguf_context *ctx, int64_t id) {
    return (ctx && id >= 0 && id < static_cast<int64_t>(ctx->offsets.size())) ? ctx->offsets[static_cast<size_t>(id)] : 0;
}
size_t gguf_get_data_offset(const gguf_context *ctx) { return ctx ? ctx->data_offset : 0; }
int64_t gguf_find_key(const gguf_context *ctx, const char *key) {
    if (!ctx || !key) return -1;
    for (size_t i = 0; i < ctx->keys.size(); ++i) {
        if (ctx->keys[i] == key) return static_cast<int64_t>(i);
    }
    return -1;
}
uint32_t gguf_get_val_u32(const gguf_context *ctx, int64_t id) {
    return (ctx && id >= 0 && id < static_cast<int64_t>(ctx->u32.size())) ? ctx->u32[static_cast<size_t>(id)] : 0;
}
size_t gguf_get_arr_n(const gguf_context *ctx, int64_t id) {
    return (ctx && id >= 0 && id < static_cast<int64_t>(ctx->arr_n.size())) ? ctx->arr_n[static_cast<size_t>(id)] : 0;
}
const char *gguf_get_arr_str(const gguf_context *ctx, int64_t id, size_t i) {
    if (!ctx || id < 0 || id >= static_cast<int64_t>(ctx->strs.size())) return nullptr;
    const auto &v = ctx->strs[static_cast<size_t>(id)];
    return i < v.size() ? v[i].c_str() : nullptr;
}
int64_t gguf_find_tensor(const gguf_context *ctx, const char *name) {
    if (!ctx || !name) return -1;
    for (size_t i = 0; i < ctx->names.size(); ++i) {
        if (ctx->names[i] == name) return static_cast<int64_t>(i);
    }
    return -1;
}

}  // extern "C"
