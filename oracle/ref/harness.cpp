// Test infrastructure: extern "C" entry points into the reference's own
// scalar text-decoder functions (src/text-decoder.h), for ctypes.  Each call
// opens the GGUF with the reference's loader (src/gguf-model.cpp) and runs
// the reference function unchanged.
#include <cstring>
#include <string>
#include <vector>

#include "gguf-model.h"
#include "text-decoder.h"

namespace {
std::string g_error;

struct Cfg {
    int n_layers, hidden, n_heads, n_kv_heads, head_dim, intermediate, vocab;
    float rope_theta, rms_norm_eps;
};

QwenAsrDecoderInputOutput make_input(const float *x, int tokens, int hidden) {
    QwenAsrDecoderInputOutput in;
    in.tokens = tokens;
    in.hidden = hidden;
    in.values.assign(x, x + static_cast<size_t>(tokens) * hidden);
    return in;
}
}  // namespace

extern "C" {

const char *ref_last_error() { return g_error.c_str(); }

// qwenasr_text_prefill_forward_cpu (text-decoder.cpp:1856): logits of the last row.
int ref_prefill_logits(const char *gguf, const Cfg *c, const float *x, int tokens, float *logits) {
    QwenAsrGgufModel model;
    if (!qwenasr_gguf_model_open(gguf, &model, &g_error)) return 1;
    QwenAsrTextPrefillOutput out;
    const bool ok = qwenasr_text_prefill_forward_cpu(model, make_input(x, tokens, c->hidden), c->n_layers, c->n_heads,
                                                     c->n_kv_heads, c->head_dim, c->intermediate, c->vocab,
                                                     c->rope_theta, c->rms_norm_eps, &out, &g_error);
    if (ok) std::memcpy(logits, out.logits.data(), out.logits.size() * sizeof(float));
    qwenasr_gguf_model_close(&model);
    return ok ? 0 : 2;
}

// qwenasr_text_generate_cached_cpu (text-decoder.cpp:2033).
int ref_generate_cached(const char *gguf, const Cfg *c, const float *x, int tokens, int max_new, const int *stop,
                        int n_stop, int *ids, int *n_out, int *stopped) {
    QwenAsrGgufModel model;
    if (!qwenasr_gguf_model_open(gguf, &model, &g_error)) return 1;
    std::vector<int32_t> stop_ids(stop, stop + n_stop);
    QwenAsrTextGenerateOutput out;
    const bool ok = qwenasr_text_generate_cached_cpu(model, make_input(x, tokens, c->hidden), max_new, c->n_layers,
                                                     c->n_heads, c->n_kv_heads, c->head_dim, c->intermediate,
                                                     c->vocab, c->rope_theta, c->rms_norm_eps, stop_ids, &out, &g_error);
    if (ok) {
        *n_out = static_cast<int>(out.generated_ids.size());
        *stopped = out.stopped ? 1 : 0;
        for (size_t i = 0; i < out.generated_ids.size(); ++i) ids[i] = out.generated_ids[i];
    }
    qwenasr_gguf_model_close(&model);
    return ok ? 0 : 2;
}

// qwenasr_text_generate_greedy_cpu (text-decoder.cpp:1927): recompute, no cache.
int ref_generate_greedy(const char *gguf, const Cfg *c, const float *x, int tokens, int max_new, int *ids, int *n_out) {
    QwenAsrGgufModel model;
    if (!qwenasr_gguf_model_open(gguf, &model, &g_error)) return 1;
    QwenAsrTextGenerateOutput out;
    const bool ok = qwenasr_text_generate_greedy_cpu(model, make_input(x, tokens, c->hidden), max_new, c->n_layers,
                                                     c->n_heads, c->n_kv_heads, c->head_dim, c->intermediate,
                                                     c->vocab, c->rope_theta, c->rms_norm_eps, {}, &out, &g_error);
    if (ok) {
        *n_out = static_cast<int>(out.generated_ids.size());
        for (size_t i = 0; i < out.generated_ids.size(); ++i) ids[i] = out.generated_ids[i];
    }
    qwenasr_gguf_model_close(&model);
    return ok ? 0 : 2;
}

// qwenasr_text_layer_forward_cpu (text-decoder.cpp:1100): one block, positions 0..T-1.
int ref_layer_forward(const char *gguf, const Cfg *c, int layer, const float *x, int tokens, float *out_values) {
    QwenAsrGgufModel model;
    if (!qwenasr_gguf_model_open(gguf, &model, &g_error)) return 1;
    QwenAsrTextLayerOutput out;
    const bool ok = qwenasr_text_layer_forward_cpu(model, make_input(x, tokens, c->hidden), layer, c->n_heads,
                                                   c->n_kv_heads, c->head_dim, c->intermediate, c->rope_theta,
                                                   c->rms_norm_eps, &out, &g_error);
    if (ok) std::memcpy(out_values, out.values.data(), out.values.size() * sizeof(float));
    qwenasr_gguf_model_close(&model);
    return ok ? 0 : 2;
}

}  // extern "C"
