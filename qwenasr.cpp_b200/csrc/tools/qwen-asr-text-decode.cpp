// qwen-asr-text-decode: the decoder harness of the reference's
// tools/qwen-asr-text-layer.cpp (:93-627), driven by a ready-made decoder input
// instead of a WAV (the audio tower is upstream of this path).  Same modes
// (--layer N, --prefill, --generate N), same `key=value` stdout protocol and
// raw f32 --out files, same text-decoder.h calls.
//
//   qwen-asr-text-decode MODEL.gguf INPUT.f32 [--generate N | --prefill | --layer L]
//                        [--out PATH] [--device auto|gpu|cpu] [--stop-ids a,b,..] [--no-stop]
//                        [--kv-dtype f32|bf16|fp8|e4i8] [--weights f32|bf16|fp8] [--page-size 16] [--gpu N]
//                        (the reference tool's --threads, --backend, --audio-backend, --kv-cache,
//                         --language and --system are accepted; see main)
// INPUT.f32 = raw float32 [tokens][hidden] (audio rows already spliced in).
// The B200 options pick the cache element type (f32 keeps the reference's
// numerics), the device weight type, and the GPU; the paged cache has
// 16-token pages only.  They set the backend's QWENASR_B200_KV /
// QWENASR_B200_WEIGHTS / QWENASR_B200_DEVICE switches for this process.
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <initializer_list>
#include <iostream>
#include <sstream>
#include <string>
#include <vector>

#include "gguf.h"
#include "qkv.h"
#include "text-decoder.h"

namespace {

int usage(const char *argv0) {
    std::cerr << "usage: " << argv0
              << " MODEL.gguf INPUT.f32 [--generate N | --prefill | --layer L] [--out PATH]"
                 " [--device auto|gpu|cpu] [--stop-ids a,b] [--no-stop]"
                 " [--kv-dtype f32|bf16|fp8|e4i8] [--weights f32|bf16|fp8] [--page-size 16] [--gpu N]\n";
    return 2;
}

bool read_f32(const std::string &path, std::vector<float> *out, std::string *err) {
    std::ifstream in(path, std::ios::binary | std::ios::ate);
    if (!in) {
        *err = "cannot open input: " + path;
        return false;
    }
    const std::streamoff n = in.tellg();
    if (n <= 0 || n % 4 != 0) {
        *err = "input is empty or not float32: " + path;
        return false;
    }
    out->resize(static_cast<size_t>(n / 4));
    in.seekg(0);
    in.read(reinterpret_cast<char *>(out->data()), n);
    return static_cast<bool>(in);
}

// The reference tool's text_json value: the text in double quotes with
// backslash, quote, \n, \r, \t escaped and other bytes below 0x20 as \u00xx.
std::string json_escape(const std::string &text) {
    static const char hex[] = "0123456789abcdef";
    std::string out = "\"";
    for (const unsigned char c : text) {
        if (c == '\\') out += "\\\\";
        else if (c == '"') out += "\\\"";
        else if (c == '\n') out += "\\n";
        else if (c == '\r') out += "\\r";
        else if (c == '\t') out += "\\t";
        else if (c < 0x20) {
            out += "\\u00";
            out.push_back(hex[c >> 4]);
            out.push_back(hex[c & 0x0F]);
        } else {
            out.push_back(static_cast<char>(c));
        }
    }
    return out + "\"";
}

// Generated ids -> text with the model file's tokenizer (special tokens
// skipped, as the reference tool decodes); false when the file has none.
bool detokenize(const std::string &model_path, const std::vector<int32_t> &ids, std::string *text) {
    qkv_tokenizer *tok = nullptr;
    char err[256];
    if (qkv_tokenizer_open(model_path.c_str(), &tok, err, sizeof err) != QKV_OK) return false;
    size_t n = 0;
    std::string buf(ids.size() * 16 + 64, '\0');
    int rc = qkv_tokenizer_decode(tok, ids.data(), static_cast<int32_t>(ids.size()), 1, &buf[0], buf.size(), &n);
    if (rc == QKV_ERR_CAPACITY) {
        buf.assign(n, '\0');
        rc = qkv_tokenizer_decode(tok, ids.data(), static_cast<int32_t>(ids.size()), 1, &buf[0], buf.size(), &n);
    }
    qkv_tokenizer_close(tok);
    if (rc != QKV_OK) return false;
    text->assign(buf.data(), n);
    return true;
}

bool write_f32(const std::string &path, const std::vector<float> &v, std::string *err) {
    std::ofstream out(path, std::ios::binary);
    out.write(reinterpret_cast<const char *>(v.data()), static_cast<std::streamsize>(v.size() * sizeof(float)));
    if (!out) {
        *err = "cannot write " + path;
        return false;
    }
    return true;
}

// The element type a backend switch selects, as the backend reads it: one of
// `other`, else f32 (unset, empty or unrecognised values keep f32).
std::string switch_value(const char *name, std::initializer_list<const char *> other) {
    const char *v = std::getenv(name);
    if (v) {
        for (const char *o : other) {
            if (std::string(v) == o) return o;
        }
    }
    return "f32";
}

// min / max / mean of an output, as the reference tool prints them for its
// prefill logits and layer rows (the mean summed in double).
struct Summary {
    float min = 0.f, max = 0.f;
    double mean = 0.0;
};
Summary summarize(const std::vector<float> &v) {
    Summary s;
    if (v.empty()) return s;
    s.min = s.max = v[0];
    double sum = 0.0;
    for (const float x : v) {
        s.min = x < s.min ? x : s.min;
        s.max = x > s.max ? x : s.max;
        sum += x;
    }
    s.mean = sum / static_cast<double>(v.size());
    return s;
}

double ms_since(std::chrono::steady_clock::time_point t0) {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
}

}  // namespace

int main(int argc, char **argv) {
    if (argc < 3) return usage(argv[0]);
    std::string model_path, input_path, out_path, error;
    int generate = -1, layer = 0;
    bool prefill = false, no_stop = false, have_stop = false;
    std::vector<int32_t> stop_ids;
    QwenAsrGgmlDevice device = qwenasr_ggml_device_auto();
    std::string kv_dtype, weights, gpu, threads = "1";
    for (int i = 1; i < argc; ++i) {
        const std::string a = argv[i];
        auto need = [&](const char *what) -> const char * {
            if (++i >= argc) {
                std::cerr << a << " requires " << what << "\n";
                std::exit(2);
            }
            return argv[i];
        };
        if (a == "-h" || a == "--help") { usage(argv[0]); return 0; }
        else if (a == "--prefill") prefill = true;
        else if (a == "--no-stop") no_stop = true;
        else if (a == "--generate") {
            char *end = nullptr;
            const long v = std::strtol(need("a non-negative integer"), &end, 10);
            if (!end || *end || v < 0 || v > 1024) { std::cerr << "--generate requires 0..1024\n"; return 2; }
            generate = static_cast<int>(v);
        } else if (a == "--layer") {
            char *end = nullptr;
            const long v = std::strtol(need("a non-negative integer"), &end, 10);
            if (!end || *end || v < 0) { std::cerr << "--layer requires a non-negative integer\n"; return 2; }
            layer = static_cast<int>(v);
        } else if (a == "--out") out_path = need("a path");
        else if (a == "--device") {
            if (!qwenasr_ggml_device_from_string(need("auto, cpu or gpu"), &device, &error)) {
                std::cerr << error << "\n";
                return 2;
            }
        } else if (a == "--stop-ids") {
            std::stringstream ss(need("a comma-separated list"));
            std::string tok;
            while (std::getline(ss, tok, ',')) if (!tok.empty()) stop_ids.push_back(static_cast<int32_t>(std::atoi(tok.c_str())));
            have_stop = true;
        } else if (a == "--kv-dtype") {
            kv_dtype = need("f32, bf16, fp8 or e4i8");
            if (kv_dtype != "f32" && kv_dtype != "bf16" && kv_dtype != "fp8" && kv_dtype != "e4i8") {
                std::cerr << "--kv-dtype must be f32, bf16, fp8 (e4m3 K and V) or e4i8 (e4m3 K, int8 V)\n";
                return 2;
            }
        } else if (a == "--weights") {
            weights = need("f32, bf16 or fp8");
            if (weights != "f32" && weights != "bf16" && weights != "fp8") {
                std::cerr << "--weights must be f32, bf16 or fp8\n";
                return 2;
            }
        } else if (a == "--page-size") {
            if (std::string(need("16")) != "16") { std::cerr << "--page-size: the paged cache has 16-token pages only\n"; return 2; }
        } else if (a == "--gpu") {
            char *end = nullptr;
            const long v = std::strtol(need("a device ordinal"), &end, 10);
            if (!end || *end || v < 0 || v > 255) { std::cerr << "--gpu requires a device ordinal 0..255\n"; return 2; }
            gpu = std::to_string(v);
        } else if (a == "--threads") threads = need("a positive integer");   // accepted and echoed; the GPU path has no host threads to size
        // The reference tool's other flags, accepted so its scripts run unchanged:
        // the text backend is always this library's, generation always uses the
        // KV cache, and the prompt options shape a decoder input that arrives
        // ready-made in INPUT.f32.
        else if (a == "--backend") {
            const std::string v = need("scalar, ggml, or sched");
            if (v != "scalar" && v != "ggml" && v != "sched") { std::cerr << "--backend requires scalar, ggml, or sched\n"; return 2; }
        } else if (a == "--audio-backend") {
            const std::string v = need("ggml or sched");
            if (v != "ggml" && v != "sched") { std::cerr << "--audio-backend requires ggml or sched\n"; return 2; }
        } else if (a == "--kv-cache") {
        } else if (a == "--language" || a == "--system") {
            need("a value");
            std::cerr << "note: " << a << " is ignored: INPUT.f32 already holds the assembled prompt rows\n";
        }
        else if (model_path.empty()) model_path = a;
        else if (input_path.empty()) input_path = a;
        else { std::cerr << "too many positional arguments\n"; return 2; }
    }
    if (prefill && generate >= 0) { std::cerr << "--prefill and --generate are mutually exclusive\n"; return 2; }
    // A flag overrides the switch; without one the switch (or its f32 default) stands.
    if (!kv_dtype.empty()) setenv("QWENASR_B200_KV", kv_dtype.c_str(), 1);
    if (!weights.empty()) setenv("QWENASR_B200_WEIGHTS", weights.c_str(), 1);
    if (!gpu.empty()) setenv("QWENASR_B200_DEVICE", gpu.c_str(), 1);
    const std::string kv_shown = switch_value("QWENASR_B200_KV", {"bf16", "fp8", "e4i8"});
    const std::string weights_shown = switch_value("QWENASR_B200_WEIGHTS", {"bf16", "fp8"});

    const auto t_init = std::chrono::steady_clock::now();
    QwenAsrGgufModel model;
    if (!qwenasr_gguf_model_open(model_path.c_str(), &model, &error)) { std::cerr << error << "\n"; return 1; }
    uint32_t L = 0, H = 0, Hq = 0, Hkv = 0, D = 0, F = 0, V = 0;
    float theta = 0.f, eps = 0.f;
    const qkv::GgufFile &f = *model.file;
    if (!f.get_u32("qwen3-asr.text.num_hidden_layers", &L) || !f.get_u32("qwen3-asr.text.hidden_size", &H) ||
        !f.get_u32("qwen3-asr.text.num_attention_heads", &Hq) || !f.get_u32("qwen3-asr.text.num_key_value_heads", &Hkv) ||
        !f.get_u32("qwen3-asr.text.head_dim", &D) || !f.get_u32("qwen3-asr.text.intermediate_size", &F) ||
        !f.get_u32("qwen3-asr.text.vocab_size", &V) || !f.get_f32("qwen3-asr.text.rope_theta", &theta) ||
        !f.get_f32("qwen3-asr.text.rms_norm_eps", &eps)) {
        std::cerr << "GGUF lacks qwen3-asr.text.* metadata\n";
        return 1;
    }
    if (!have_stop && !no_stop) {   // the reference CLI's stop set (tools/qwen-asr-text-layer.cpp:395-399)
        uint32_t id = 0;
        if (f.get_u32("qwen3-asr.token.im_end_token_id", &id)) stop_ids.push_back(static_cast<int32_t>(id));
        if (f.get_u32("qwen3-asr.token.endoftext_token_id", &id)) stop_ids.push_back(static_cast<int32_t>(id));
        if (f.get_u32("tokenizer.ggml.eos_token_id", &id)) stop_ids.push_back(static_cast<int32_t>(id));
    }
    if (no_stop) stop_ids.clear();

    const double init_ms = ms_since(t_init);
    // decoder_input_ms: the reference tool assembles the decoder input from
    // audio here; this harness reads the assembled rows from INPUT.f32.
    const auto t_input = std::chrono::steady_clock::now();
    QwenAsrDecoderInputOutput input;
    if (!read_f32(input_path, &input.values, &error)) { std::cerr << error << "\n"; return 1; }
    if (input.values.size() % H != 0) { std::cerr << "input size is not a multiple of hidden\n"; return 1; }
    input.hidden = static_cast<int>(H);
    input.tokens = static_cast<int>(input.values.size() / H);
    const double decoder_input_ms = ms_since(t_input);

    std::cout << "backend=b200\n";
    std::cout << "device=" << qwenasr_ggml_device_name(device) << "\n";
    std::cout << "threads=" << threads << "\n";
    std::cout << "init_ms=" << init_ms << "\n";
    std::cout << "decoder_input_ms=" << decoder_input_ms << "\n";
    std::cout << "layers=" << L << "\n";
    std::cout << "prompt_tokens=" << input.tokens << "\n";
    std::cout << "hidden=" << H << "\n";
    std::cout << "kv_dtype=" << kv_shown << "\n";
    std::cout << "weights=" << weights_shown << "\n";
    std::cout << "page_tokens=16\n";

    if (generate >= 0) {
        const auto t0 = std::chrono::steady_clock::now();
        QwenAsrTextDecoderBackend *b = nullptr;
        if (!qwenasr_text_decoder_backend_init_cached(model, 1, static_cast<int>(L), static_cast<int>(H), static_cast<int>(Hq),
                                                      static_cast<int>(Hkv), static_cast<int>(D), static_cast<int>(F),
                                                      static_cast<int>(V), input.tokens + generate, theta, eps, &b,
                                                      &error, device)) {
            std::cerr << error << "\n";
            return 1;
        }
        const double text_init_ms = ms_since(t0);
        QwenAsrTextGenerateOutput out;
        const auto t1 = std::chrono::steady_clock::now();
        const bool ok = qwenasr_text_generate_cached_backend(b, model, input, generate, stop_ids, &out, &error);
        const double generate_ms = ms_since(t1);
        qwenasr_text_decoder_backend_free(b);
        if (!ok) { std::cerr << error << "\n"; return 1; }
        std::cout << "mode=generate\n";
        std::cout << "decode_backend=kv-cache\n";
        std::cout << "text_init_ms=" << text_init_ms << "\n";
        std::cout << "generate_ms=" << generate_ms << "\n";
        std::cout << "total_tokens=" << out.total_tokens << "\n";
        std::cout << "vocab=" << out.vocab << "\n";
        std::cout << "requested_tokens=" << generate << "\n";
        std::cout << "generated_tokens=" << out.generated_ids.size() << "\n";
        std::cout << "tokens_per_s=" << (generate_ms > 0 ? 1e3 * static_cast<double>(out.generated_ids.size()) / generate_ms : 0.0)
                  << "\n";
        std::cout << "stopped=" << (out.stopped ? "true" : "false") << "\n";
        std::cout << "generated_ids=";
        for (size_t i = 0; i < out.generated_ids.size(); ++i) std::cout << (i ? "," : "") << out.generated_ids[i];
        std::cout << "\n";
        std::string text;
        if (detokenize(model_path, out.generated_ids, &text)) {   // the model file has a tokenizer
            if (!out_path.empty()) {
                std::ofstream o(out_path, std::ios::binary);
                o.write(text.data(), static_cast<std::streamsize>(text.size()));
                if (!o) { std::cerr << "cannot write " << out_path << "\n"; return 1; }
            }
            std::cout << "text_json=" << json_escape(text) << "\n";
        }
        return 0;
    }
    if (prefill) {
        const auto t0 = std::chrono::steady_clock::now();
        QwenAsrTextDecoderBackend *b = nullptr;
        if (!qwenasr_text_decoder_backend_init(model, 1, static_cast<int>(L), static_cast<int>(H), static_cast<int>(Hq),
                                               static_cast<int>(Hkv), static_cast<int>(D), static_cast<int>(F),
                                               static_cast<int>(V), theta, eps, &b, &error, device)) {
            std::cerr << error << "\n";
            return 1;
        }
        const double text_init_ms = ms_since(t0);
        QwenAsrTextPrefillOutput out;
        const auto t1 = std::chrono::steady_clock::now();
        const bool ok = qwenasr_text_prefill_backend_forward(b, input, &out, &error);
        const double prefill_ms = ms_since(t1);
        qwenasr_text_decoder_backend_free(b);
        if (!ok) { std::cerr << error << "\n"; return 1; }
        int top = 0;
        for (int i = 1; i < out.vocab; ++i) if (out.logits[static_cast<size_t>(i)] > out.logits[static_cast<size_t>(top)]) top = i;
        if (!out_path.empty() && !write_f32(out_path, out.logits, &error)) { std::cerr << error << "\n"; return 1; }
        const Summary sm = summarize(out.logits);
        std::cout << "mode=prefill\n";
        std::cout << "text_init_ms=" << text_init_ms << "\n";
        std::cout << "prefill_ms=" << prefill_ms << "\n";
        std::cout << "tokens=" << out.tokens << "\n";
        std::cout << "vocab=" << out.vocab << "\n";
        std::cout << "values=" << out.logits.size() << "\n";
        std::cout << "top_id=" << top << "\n";
        std::cout << "top_logit=" << out.logits[static_cast<size_t>(top)] << "\n";
        std::cout << "min=" << sm.min << "\n";
        std::cout << "max=" << sm.max << "\n";
        std::cout << "mean=" << sm.mean << "\n";
        return 0;
    }
    QwenAsrTextLayerBackend *b = nullptr;
    if (!qwenasr_text_layer_backend_init(model, layer, 1, static_cast<int>(H), static_cast<int>(Hq), static_cast<int>(Hkv),
                                         static_cast<int>(D), static_cast<int>(F), theta, eps, &b, &error, device)) {
        std::cerr << error << "\n";
        return 1;
    }
    QwenAsrTextLayerOutput out;
    const auto t1 = std::chrono::steady_clock::now();
    const bool ok = qwenasr_text_layer_backend_forward(b, input, &out, &error);
    const double layer_ms = ms_since(t1);
    qwenasr_text_layer_backend_free(b);
    if (!ok) { std::cerr << error << "\n"; return 1; }
    if (!out_path.empty() && !write_f32(out_path, out.values, &error)) { std::cerr << error << "\n"; return 1; }
    const Summary sm = summarize(out.values);
    std::cout << "mode=layer\n";
    std::cout << "text_layer_ms=" << layer_ms << "\n";
    std::cout << "layer=" << layer << "\n";
    std::cout << "tokens=" << out.tokens << "\n";
    std::cout << "values=" << out.values.size() << "\n";
    std::cout << "min=" << sm.min << "\n";
    std::cout << "max=" << sm.max << "\n";
    std::cout << "mean=" << sm.mean << "\n";
    return 0;
}
