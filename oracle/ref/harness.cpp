// Test infrastructure: extern "C" entry points into the reference's own
// scalar text-decoder functions (src/text-decoder.h) and its decoder-input
// assembly (src/decoder-input.h, with src/tokenizer.cpp), for ctypes.  Each call
// opens the GGUF with the reference's loader (src/gguf-model.cpp) and runs
// the reference function unchanged.
#include <cstring>
#include <string>
#include <vector>

#include "decoder-input.h"
#include "gguf-model.h"
#include "text-decoder.h"
#include "tokenizer.h"

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

// qwenasr_decoder_input_from_audio (decoder-input.cpp:26-101): prompt template
// + tokenizer (from the same GGUF) + embedding rows with the audio rows
// spliced in.  out_ids / out_values must hold max_tokens rows; *tokens gets
// the prompt length (also when it exceeds max_tokens, with return 3).
int ref_decoder_input(const char *gguf, int audio_tokens, int hidden, const float *audio_values, int audio_token_id,
                      const char *system_text, const char *language, int max_tokens, int32_t *out_ids,
                      float *out_values, int *tokens) {
    QwenAsrGgufModel model;
    if (!qwenasr_gguf_model_open(gguf, &model, &g_error)) return 1;
    QwenAsrTokenizer tok;
    if (!qwenasr_tokenizer_load_gguf(gguf, &tok, &g_error)) {
        qwenasr_gguf_model_close(&model);
        return 1;
    }
    QwenAsrAudioEncoderOutput audio;
    audio.tokens = audio_tokens;
    audio.hidden = hidden;
    audio.values.assign(audio_values, audio_values + static_cast<size_t>(audio_tokens) * hidden);
    QwenAsrDecoderInputOutput out;
    const bool ok = qwenasr_decoder_input_from_audio(model, tok, audio, audio_token_id, system_text, language, &out,
                                                     &g_error);
    qwenasr_gguf_model_close(&model);
    if (!ok) return 2;
    *tokens = out.tokens;
    if (out.tokens > max_tokens) return 3;
    for (int i = 0; i < out.tokens; ++i) out_ids[i] = out.input_ids[static_cast<size_t>(i)];
    std::memcpy(out_values, out.values.data(), out.values.size() * sizeof(float));
    return 0;
}

// qwenasr_tokenizer_decode (tokenizer.cpp:482-527) with the tokenizer of `gguf`:
// bytes into out (cap), *len = their count (return 3 when they do not fit).
int ref_tokenizer_decode(const char *gguf, const int32_t *ids, int n, int skip_special, char *out, int cap, int *len) {
    QwenAsrTokenizer tok;
    if (!qwenasr_tokenizer_load_gguf(gguf, &tok, &g_error)) return 1;
    const std::string s = qwenasr_tokenizer_decode(tok, std::vector<int32_t>(ids, ids + n), skip_special != 0);
    *len = static_cast<int>(s.size());
    if (static_cast<int>(s.size()) > cap) return 3;
    std::memcpy(out, s.data(), s.size());
    return 0;
}

// qwenasr_tokenizer_encode (tokenizer.cpp:438-480) with the tokenizer of `gguf`.
int ref_tokenizer_encode(const char *gguf, const char *text, int text_len, int add_eos, int32_t *ids, int cap,
                         int *n) {
    QwenAsrTokenizer tok;
    if (!qwenasr_tokenizer_load_gguf(gguf, &tok, &g_error)) return 1;
    const std::vector<int32_t> v = qwenasr_tokenizer_encode(tok, std::string(text, static_cast<size_t>(text_len)),
                                                            add_eos != 0);
    *n = static_cast<int>(v.size());
    if (*n > cap) return 3;
    for (int i = 0; i < *n; ++i) ids[i] = v[static_cast<size_t>(i)];
    return 0;
}

}  // extern "C"

// The reference's GGML audio encoder is not built here (GGML is an empty
// submodule in its tree); decoder-input.cpp names it, so this stub fails.
bool qwenasr_audio_encoder_forward_ggml(const QwenAsrGgufModel &, const QwenAsrFeatures &, int, int, int, int,
                                        QwenAsrAudioEncoderOutput *, std::string *error) {
    if (error) *error = "GGML audio encoder unavailable in the test harness";
    return false;
}
