// Detokenisation of generated ids: the step after the decoder's greedy loop
// (the reference decodes with qwenasr_tokenizer_decode, src/tokenizer.cpp:
// 482-527, at tools/qwen-asr-text-layer.cpp:478).  Host only.
//
// Byte-level BPE vocabulary from the model file's metadata: each token is a
// string of "byte symbols" (the published GPT-2 mapping of the 256 byte values
// to printable code points: printable Latin-1 bytes map to themselves, the
// other 68 to U+0100.. in byte order).  Decoding concatenates the tokens of
// the ids and turns every byte symbol back into its byte; other characters
// are copied as they are.  Ids outside the vocabulary are skipped, and so are
// the seven special tokens when asked (the same keys and checks as the
// reference's loader, tokenizer.cpp:306-372).
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "gguf.h"
#include "qkv.h"

struct qkv_tokenizer {
    std::vector<std::string> id_to_token;
    std::vector<unsigned char> special;              // 1: one of the special tokens
    std::unordered_map<std::string, unsigned char> byte_of;   // byte symbol (UTF-8) -> byte
};

namespace {

void set_err(char *err, size_t len, const std::string &msg) {
    if (err && len) {
        std::strncpy(err, msg.c_str(), len - 1);
        err[len - 1] = '\0';
    }
}

std::string utf8(int cp) {
    std::string s;
    if (cp < 0x80) {
        s.push_back(static_cast<char>(cp));
    } else if (cp < 0x800) {
        s.push_back(static_cast<char>(0xC0 | (cp >> 6)));
        s.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    } else {
        s.push_back(static_cast<char>(0xE0 | (cp >> 12)));
        s.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
        s.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    }
    return s;
}

// Length of the UTF-8 sequence a lead byte announces (1 for anything else),
// clamped to the bytes left in the token.
int piece_len(unsigned char c, int left) {
    int n = 1;
    if ((c & 0xE0) == 0xC0) n = 2;
    else if ((c & 0xF0) == 0xE0) n = 3;
    else if ((c & 0xF8) == 0xF0) n = 4;
    return n < left ? n : left;
}

}  // namespace

extern "C" {

int qkv_tokenizer_open(const char *gguf_path, qkv_tokenizer **out, char *err, size_t err_len) {
    if (!gguf_path || !out) {
        set_err(err, err_len, "qkv_tokenizer_open: null path or out");
        return QKV_ERR_INVALID_ARG;
    }
    qkv::GgufFile f;
    std::string e;
    int rc = f.open(gguf_path, &e);
    if (rc != QKV_OK) {
        set_err(err, err_len, e);
        return rc;
    }
    const qkv::GgufValue *tokens = f.value("tokenizer.ggml.tokens");
    if (!tokens || !f.value("tokenizer.ggml.merges") || !f.value("tokenizer.ggml.eos_token_id") ||
        tokens->strs.size() != tokens->arr_n) {
        set_err(err, err_len, "GGUF tokenizer metadata is incomplete");
        return QKV_ERR_FORMAT;
    }
    auto *t = new qkv_tokenizer();
    t->id_to_token = tokens->strs;
    t->special.assign(t->id_to_token.size(), 0);
    static const char *keys[] = {
        "qwen3-asr.token.endoftext_token_id", "qwen3-asr.token.im_start_token_id",
        "qwen3-asr.token.im_end_token_id",    "qwen3-asr.token.audio_start_token_id",
        "qwen3-asr.token.audio_end_token_id", "qwen3-asr.token.audio_token_id",
        "qwen3-asr.token.asr_text_token_id",
    };
    for (const char *k : keys) {
        uint32_t id = 0;
        if (!f.get_u32(k, &id)) {
            set_err(err, err_len, std::string("missing tokenizer special key: ") + k);
            delete t;
            return QKV_ERR_FORMAT;
        }
        if (id >= t->special.size()) {
            set_err(err, err_len, std::string("tokenizer special id out of range for key: ") + k);
            delete t;
            return QKV_ERR_FORMAT;
        }
        t->special[id] = 1;
    }
    // byte symbols: printable bytes keep their code point, the rest get 256, 257, ...
    int extra = 0;
    for (int b = 0; b < 256; ++b) {
        const bool printable = (b >= 0x21 && b <= 0x7E) || (b >= 0xA1 && b <= 0xAC) || (b >= 0xAE && b <= 0xFF);
        t->byte_of[utf8(printable ? b : 256 + extra++)] = static_cast<unsigned char>(b);
    }
    *out = t;
    return QKV_OK;
}

int qkv_tokenizer_decode(const qkv_tokenizer *t, const int32_t *ids, int32_t n, int32_t skip_special, char *out,
                         size_t cap, size_t *len) {
    if (!t || (n > 0 && !ids) || !len) return QKV_ERR_INVALID_ARG;
    std::string s;
    for (int32_t k = 0; k < n; ++k) {
        const int32_t id = ids[k];
        if (id < 0 || static_cast<size_t>(id) >= t->id_to_token.size()) continue;
        if (skip_special && t->special[static_cast<size_t>(id)]) continue;
        const std::string &tok = t->id_to_token[static_cast<size_t>(id)];
        const int L = static_cast<int>(tok.size());
        for (int pos = 0; pos < L;) {
            const int adv = piece_len(static_cast<unsigned char>(tok[static_cast<size_t>(pos)]), L - pos);
            const std::string piece = tok.substr(static_cast<size_t>(pos), static_cast<size_t>(adv));
            const auto it = t->byte_of.find(piece);
            if (it != t->byte_of.end()) s.push_back(static_cast<char>(it->second));
            else s += piece;
            pos += adv;
        }
    }
    *len = s.size();
    if (s.size() > cap || (s.size() > 0 && !out)) return QKV_ERR_CAPACITY;
    if (!s.empty()) std::memcpy(out, s.data(), s.size());
    return QKV_OK;
}

void qkv_tokenizer_close(qkv_tokenizer *t) { delete t; }

}  // extern "C"
