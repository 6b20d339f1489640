// The reference's decoder operator surface (src/text-decoder.h) on the B200
// C ABI.  Each function keeps the reference's argument checks and error
// messages where they describe the same condition (text-decoder.cpp:1476-1525,
// 1641-1655, 2209-2240).
#include "text-decoder.h"

#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "gguf.h"
#include "qkv.h"

namespace {

void set_error(std::string *error, const std::string &message) {
    if (error) *error = message;
}

int env_dtype(const char *name, int dflt) {
    const char *v = std::getenv(name);
    if (!v || !*v) return dflt;
    const std::string s(v);
    if (s == "f32") return QKV_F32;
    if (s == "bf16") return QKV_BF16;
    if (s == "fp8") return QKV_FP8_E4M3;
    if (s == "e4i8") return QKV_E4M3K_I8V;
    return dflt;
}

bool device_ordinal(QwenAsrGgmlDevice device, int *ordinal, std::string *error) {
    if (device == QwenAsrGgmlDevice::Cpu) {
        set_error(error, "this text-decoder backend runs on a B200 GPU only (no CPU fallback); use --device gpu");
        return false;
    }
    const char *v = std::getenv("QWENASR_B200_DEVICE");
    *ordinal = v && *v ? std::atoi(v) : 0;
    return true;
}

bool create(const QwenAsrGgufModel &model, const qkv_model_config &cfg, int max_seq_len, int max_streams,
            QwenAsrGgmlDevice device, qkv_handle **out, std::string *error) {
    int ordinal = 0;
    if (!device_ordinal(device, &ordinal, error)) return false;
    if (model.path.empty()) {
        set_error(error, "GGUF model is not open");
        return false;
    }
    qkv_runtime_config rt{};
    rt.device = ordinal;
    {
        const int wd = env_dtype("QWENASR_B200_WEIGHTS", QKV_F32);
        rt.weight_dtype = (wd == QKV_BF16 || wd == QKV_FP8_E4M3) ? wd : QKV_F32;
    }
    rt.kv_dtype = env_dtype("QWENASR_B200_KV", QKV_F32);
    rt.page_tokens = 16;
    rt.max_streams = max_streams;
    rt.max_context = max_seq_len;
    rt.max_pages = 0;
    rt.max_batch_tokens = max_seq_len;
    rt.page_order_seed = 0;
    char err[1024] = {0};
    const int rc = qkv_create(model.path.c_str(), &cfg, &rt, out, err, sizeof err);
    if (rc != QKV_OK) {
        set_error(error, err);
        return false;
    }
    return true;
}

}  // namespace

// ---- gguf-model.h ----

bool qwenasr_gguf_model_open(const char *path, QwenAsrGgufModel *model, std::string *error) {
    if (!path || !model) {
        set_error(error, "qwenasr_gguf_model_open: path or model is null");
        return false;
    }
    qwenasr_gguf_model_close(model);
    auto *f = new qkv::GgufFile();
    std::string e;
    if (f->open(path, &e) != QKV_OK) {
        delete f;
        set_error(error, e);
        return false;
    }
    model->file = f;
    model->path = path;
    model->file_size = f->file_size();
    model->data_offset = f->data_offset();
    model->mapping = f->mapping();
    return true;
}

void qwenasr_gguf_model_close(QwenAsrGgufModel *model) {
    if (!model) return;
    delete model->file;
    model->file = nullptr;
    model->path.clear();
    model->mapping = nullptr;
    model->file_size = 0;
    model->data_offset = 0;
}

int64_t qwenasr_gguf_model_tensor_count(const QwenAsrGgufModel &model) {
    return model.file ? static_cast<int64_t>(model.file->tensors().size()) : 0;
}

static void fill_view(const qkv::GgufTensor &t, QwenAsrGgufTensorView *out) {
    out->name = t.name;
    out->type = static_cast<ggml_type>(t.type);
    // GGML's view drops trailing unit dimensions (ggml_n_dims), gguf-model.cpp:150-154.
    size_t nd = t.ne.size();
    while (nd > 1 && t.ne[nd - 1] == 1) --nd;
    out->ne.assign(t.ne.begin(), t.ne.begin() + static_cast<long>(nd));
    out->nbytes = t.nbytes;
    out->offset = t.offset;
    out->data = t.data;
}

bool qwenasr_gguf_model_tensor_by_index(const QwenAsrGgufModel &model, int64_t index, QwenAsrGgufTensorView *out,
                                        std::string *error) {
    if (!model.file) {
        set_error(error, "GGUF model is not open");
        return false;
    }
    if (index < 0 || index >= qwenasr_gguf_model_tensor_count(model)) {
        set_error(error, "GGUF tensor index is out of range");
        return false;
    }
    if (out) fill_view(model.file->tensors()[static_cast<size_t>(index)], out);
    return true;
}

bool qwenasr_gguf_model_tensor_by_name(const QwenAsrGgufModel &model, const char *name, QwenAsrGgufTensorView *out,
                                       std::string *error) {
    if (!model.file || !name) {
        set_error(error, "GGUF model is not open or tensor name is null");
        return false;
    }
    const qkv::GgufTensor *t = model.file->find(name);
    if (!t) {
        set_error(error, std::string("missing GGUF tensor: ") + name);
        return false;
    }
    if (out) fill_view(*t, out);
    return true;
}

// ---- ggml-backends.h (device selector only) ----

QwenAsrGgmlDevice qwenasr_ggml_device_auto() { return QwenAsrGgmlDevice::Auto; }
QwenAsrGgmlDevice qwenasr_ggml_device_cpu() { return QwenAsrGgmlDevice::Cpu; }
QwenAsrGgmlDevice qwenasr_ggml_device_gpu() { return QwenAsrGgmlDevice::Gpu; }

bool qwenasr_ggml_device_from_string(const std::string &value, QwenAsrGgmlDevice *out, std::string *error) {
    if (!out) {
        set_error(error, "qwenasr_ggml_device_from_string: out is null");
        return false;
    }
    std::string v(value);
    std::transform(v.begin(), v.end(), v.begin(), [](unsigned char c) { return static_cast<char>(std::tolower(c)); });
    if (v == "auto") *out = QwenAsrGgmlDevice::Auto;
    else if (v == "cpu") *out = QwenAsrGgmlDevice::Cpu;
    else if (v == "gpu" || v == "cuda") *out = QwenAsrGgmlDevice::Gpu;
    else {
        set_error(error, "device must be auto, cpu, gpu, or cuda");
        return false;
    }
    return true;
}

const char *qwenasr_ggml_device_name(QwenAsrGgmlDevice device) {
    switch (device) {
        case QwenAsrGgmlDevice::Auto: return "auto";
        case QwenAsrGgmlDevice::Cpu: return "cpu";
        case QwenAsrGgmlDevice::Gpu: return "gpu";
    }
    return "unknown";
}

// ---- text-decoder.h ----

struct QwenAsrTextLayerBackend {
    qkv_handle *h = nullptr;
    int layer = 0;
    int hidden = 0;
};

struct QwenAsrTextDecoderBackend {
    qkv_handle *h = nullptr;
    int hidden = 0;
    int vocab = 0;
    int max_seq_len = 0;
};

bool qwenasr_text_layer_backend_init(const QwenAsrGgufModel &model, int layer, int, int hidden, int n_heads,
                                     int n_kv_heads, int head_dim, int intermediate, float rope_theta,
                                     float rms_norm_eps, QwenAsrTextLayerBackend **out, std::string *error,
                                     QwenAsrGgmlDevice device) {
    if (!out) {
        set_error(error, "qwenasr_text_layer_backend_init: out is null");
        return false;
    }
    *out = nullptr;
    qkv_model_config cfg{};
    char err[512] = {0};
    if (qkv_read_gguf_config(model.path.c_str(), &cfg, err, sizeof err) != QKV_OK) {
        set_error(error, err);
        return false;
    }
    if (layer < 0 || layer >= cfg.n_layers || hidden != cfg.hidden || n_heads <= 0 || n_kv_heads <= 0 ||
        n_heads % n_kv_heads != 0) {
        set_error(error, "invalid text layer backend configuration");
        return false;
    }
    cfg.hidden = hidden;
    cfg.n_heads = n_heads;
    cfg.n_kv_heads = n_kv_heads;
    cfg.head_dim = head_dim;
    cfg.intermediate = intermediate;
    cfg.rope_theta = rope_theta;
    cfg.rms_norm_eps = rms_norm_eps;
    auto *b = new QwenAsrTextLayerBackend();
    if (!create(model, cfg, 4096, 1, device, &b->h, error)) {
        delete b;
        return false;
    }
    b->layer = layer;
    b->hidden = hidden;
    *out = b;
    return true;
}

void qwenasr_text_layer_backend_free(QwenAsrTextLayerBackend *backend) {
    if (!backend) return;
    qkv_destroy(backend->h);
    delete backend;
}

bool qwenasr_text_layer_backend_forward(QwenAsrTextLayerBackend *backend, const QwenAsrDecoderInputOutput &input,
                                        QwenAsrTextLayerOutput *out, std::string *error) {
    if (!backend || !out) {
        set_error(error, "qwenasr_text_layer_backend_forward: backend or out is null");
        return false;
    }
    if (input.tokens <= 0 || input.hidden != backend->hidden ||
        input.values.size() != static_cast<size_t>(input.tokens) * input.hidden) {
        set_error(error, "invalid decoder input for text layer backend");
        return false;
    }
    QwenAsrTextLayerOutput result;
    result.tokens = input.tokens;
    result.hidden = input.hidden;
    result.values.assign(input.values.size(), 0.0f);
    if (qkv_layer_forward(backend->h, backend->layer, input.tokens, input.values.data(), result.values.data()) !=
        QKV_OK) {
        set_error(error, qkv_last_error(backend->h));
        return false;
    }
    *out = std::move(result);
    return true;
}

bool qwenasr_text_decoder_backend_init_cached(const QwenAsrGgufModel &model, int, int n_layers, int hidden,
                                              int n_heads, int n_kv_heads, int head_dim, int intermediate, int vocab,
                                              int max_seq_len, float rope_theta, float rms_norm_eps,
                                              QwenAsrTextDecoderBackend **out, std::string *error,
                                              QwenAsrGgmlDevice device) {
    if (!out) {
        set_error(error, "qwenasr_text_decoder_backend_init_cached: out is null");
        return false;
    }
    *out = nullptr;
    if (n_layers <= 0 || hidden <= 0 || n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || intermediate <= 0 ||
        vocab <= 0 || n_heads % n_kv_heads != 0) {
        set_error(error, "invalid text decoder backend configuration");
        return false;
    }
    if (max_seq_len <= 0) {
        set_error(error, "invalid text decoder KV-cache configuration");
        return false;
    }
    const qkv_model_config cfg{n_layers, hidden, n_heads, n_kv_heads, head_dim, intermediate, vocab, rope_theta,
                               rms_norm_eps};
    auto *b = new QwenAsrTextDecoderBackend();
    if (!create(model, cfg, max_seq_len, 2, device, &b->h, error)) {
        delete b;
        return false;
    }
    b->hidden = hidden;
    b->vocab = vocab;
    b->max_seq_len = max_seq_len;
    *out = b;
    return true;
}

bool qwenasr_text_decoder_backend_init(const QwenAsrGgufModel &model, int n_threads, int n_layers, int hidden,
                                       int n_heads, int n_kv_heads, int head_dim, int intermediate, int vocab,
                                       float rope_theta, float rms_norm_eps, QwenAsrTextDecoderBackend **out,
                                       std::string *error, QwenAsrGgmlDevice device) {
    // The uncached backend serves prefill-only calls; a 4096-token context covers them.
    return qwenasr_text_decoder_backend_init_cached(model, n_threads, n_layers, hidden, n_heads, n_kv_heads, head_dim,
                                                    intermediate, vocab, 4096, rope_theta, rms_norm_eps, out, error,
                                                    device);
}

void qwenasr_text_decoder_backend_free(QwenAsrTextDecoderBackend *backend) {
    if (!backend) return;
    qkv_destroy(backend->h);
    delete backend;
}

bool qwenasr_text_prefill_backend_forward(QwenAsrTextDecoderBackend *backend, const QwenAsrDecoderInputOutput &input,
                                          QwenAsrTextPrefillOutput *out, std::string *error) {
    if (!backend || !out) {
        set_error(error, "qwenasr_text_prefill_backend_forward: backend or out is null");
        return false;
    }
    if (input.tokens <= 0 || input.hidden != backend->hidden ||
        input.values.size() != static_cast<size_t>(input.tokens) * input.hidden) {
        set_error(error, "invalid decoder input for text prefill backend");
        return false;
    }
    int32_t s = -1;
    if (qkv_stream_open(backend->h, &s) != QKV_OK) {
        set_error(error, qkv_last_error(backend->h));
        return false;
    }
    QwenAsrTextPrefillOutput result;
    result.tokens = input.tokens;
    result.hidden = input.hidden;
    result.vocab = backend->vocab;
    result.logits.assign(static_cast<size_t>(backend->vocab), 0.0f);
    int32_t id = -1;
    const int32_t len = input.tokens;
    const int rc = qkv_prefill(backend->h, 1, &s, &len, input.values.data(), &id, result.logits.data());
    const std::string msg = rc == QKV_OK ? std::string() : std::string(qkv_last_error(backend->h));
    qkv_stream_close(backend->h, s);
    if (rc != QKV_OK) {
        set_error(error, msg);
        return false;
    }
    *out = std::move(result);
    return true;
}

bool qwenasr_text_generate_cached_backend(QwenAsrTextDecoderBackend *backend, const QwenAsrGgufModel &,
                                          const QwenAsrDecoderInputOutput &input, int max_new_tokens,
                                          const std::vector<int32_t> &stop_ids, QwenAsrTextGenerateOutput *out,
                                          std::string *error) {
    if (!backend || !out) {
        set_error(error, "qwenasr_text_generate_cached_backend: backend or out is null");
        return false;
    }
    if (max_new_tokens < 0) {
        set_error(error, "max_new_tokens must be non-negative");
        return false;
    }
    if (input.tokens <= 0 || input.hidden != backend->hidden ||
        input.values.size() != static_cast<size_t>(input.tokens) * input.hidden) {
        set_error(error, "invalid backend cached text generation input");
        return false;
    }
    if (input.tokens + max_new_tokens > backend->max_seq_len) {
        set_error(error, "backend text generation exceeds KV-cache capacity");
        return false;
    }
    QwenAsrTextGenerateOutput result;
    result.prompt_tokens = input.tokens;
    result.total_tokens = input.tokens;
    result.hidden = input.hidden;
    result.vocab = backend->vocab;
    std::vector<int32_t> ids(static_cast<size_t>(std::max(max_new_tokens, 1)));
    int32_t n = 0, stopped = 0;
    if (qkv_generate(backend->h, input.values.data(), input.tokens, max_new_tokens, stop_ids.data(),
                     static_cast<int32_t>(stop_ids.size()), ids.data(), &n, &stopped) != QKV_OK) {
        set_error(error, qkv_last_error(backend->h));
        return false;
    }
    result.generated_ids.assign(ids.begin(), ids.begin() + n);
    result.total_tokens = input.tokens + n;
    result.stopped = stopped != 0;
    *out = std::move(result);
    return true;
}
