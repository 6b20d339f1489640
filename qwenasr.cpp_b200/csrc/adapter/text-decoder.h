// Drop-in mirror of the GPU-backend half of the reference's operator surface
// (src/text-decoder.h:10-33 result types, :35-83 layer backend, :85-124 decoder
// backend, :156-163 cached generation), implemented on the B200 C ABI
// (include/qkv.h).  Same names, argument meaning and bool + std::string*
// error convention.  The reference's *_cpu and *_ggml functions are not
// provided: this path has no CPU fallback.
//
// Precision: weights and KV cache default to f32 (the reference's f32 path);
// QWENASR_B200_WEIGHTS=bf16 and QWENASR_B200_KV=bf16|fp8 select the fast modes.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "decoder-input.h"
#include "ggml-backends.h"
#include "gguf-model.h"

struct QwenAsrTextLayerOutput {
    int tokens = 0;
    int hidden = 0;
    std::vector<float> values;   // [token, hidden]
};

struct QwenAsrTextPrefillOutput {
    int tokens = 0;
    int hidden = 0;
    int vocab = 0;
    std::vector<float> logits;   // [vocab], next-token logits of the last prompt position
};

struct QwenAsrTextGenerateOutput {
    int prompt_tokens = 0;
    int total_tokens = 0;
    int hidden = 0;
    int vocab = 0;
    bool stopped = false;
    std::vector<int32_t> generated_ids;
};

struct QwenAsrTextLayerBackend;
struct QwenAsrTextDecoderBackend;

bool qwenasr_text_layer_backend_init(const QwenAsrGgufModel &model, int layer, int n_threads, int hidden, int n_heads,
                                     int n_kv_heads, int head_dim, int intermediate, float rope_theta,
                                     float rms_norm_eps, QwenAsrTextLayerBackend **out, std::string *error,
                                     QwenAsrGgmlDevice device = qwenasr_ggml_device_auto());
void qwenasr_text_layer_backend_free(QwenAsrTextLayerBackend *backend);
bool qwenasr_text_layer_backend_forward(QwenAsrTextLayerBackend *backend, const QwenAsrDecoderInputOutput &input,
                                        QwenAsrTextLayerOutput *out, std::string *error);

bool qwenasr_text_decoder_backend_init(const QwenAsrGgufModel &model, int n_threads, int n_layers, int hidden,
                                       int n_heads, int n_kv_heads, int head_dim, int intermediate, int vocab,
                                       float rope_theta, float rms_norm_eps, QwenAsrTextDecoderBackend **out,
                                       std::string *error, QwenAsrGgmlDevice device = qwenasr_ggml_device_auto());
bool qwenasr_text_decoder_backend_init_cached(const QwenAsrGgufModel &model, int n_threads, int n_layers, int hidden,
                                              int n_heads, int n_kv_heads, int head_dim, int intermediate, int vocab,
                                              int max_seq_len, float rope_theta, float rms_norm_eps,
                                              QwenAsrTextDecoderBackend **out, std::string *error,
                                              QwenAsrGgmlDevice device = qwenasr_ggml_device_auto());
void qwenasr_text_decoder_backend_free(QwenAsrTextDecoderBackend *backend);
bool qwenasr_text_prefill_backend_forward(QwenAsrTextDecoderBackend *backend, const QwenAsrDecoderInputOutput &input,
                                          QwenAsrTextPrefillOutput *out, std::string *error);
bool qwenasr_text_generate_cached_backend(QwenAsrTextDecoderBackend *backend, const QwenAsrGgufModel &model,
                                          const QwenAsrDecoderInputOutput &input, int max_new_tokens,
                                          const std::vector<int32_t> &stop_ids, QwenAsrTextGenerateOutput *out,
                                          std::string *error);
