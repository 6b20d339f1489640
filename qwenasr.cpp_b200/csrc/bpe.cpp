// Byte-level BPE tokenizer of the model file, host only: the ASR prompt
// template (src/tokenizer.cpp:529-549) and its encoding (:438-480), which
// produce the ids the device decoder input takes, and the detokenisation of
// generated ids (:482-527, used at tools/qwen-asr-text-layer.cpp:478).
//
// The vocabulary, merges and the seven special-token ids come from the file's
// metadata (the keys and checks of the reference's loader, :306-372).  Tokens
// are strings of "byte symbols": the published GPT-2 mapping of the 256 byte
// values to printable code points (printable Latin-1 bytes map to
// themselves, the other 68 to U+0100.. in byte order).
//
// Encoding must reproduce the reference's ids, so its steps are kept alike:
// split at special tokens (the earliest occurrence, the longest on a tie);
// pre-tokenise each piece (a contraction 's 't 're 've 'm 'll 'd; a
// space-or-tab run of one followed by letters; a letter run; one digit; a
// newline run; a space run; a run of anything else); byte-map each chunk and
// merge the adjacent pair of lowest rank until none is in the table; look the
// pieces up (pieces not in the vocabulary are dropped).  A UTF-8 sequence cut
// off at a segment's end is read to its announced length, into zero bytes,
// as the reference reads it (code_point_padded).
#include <algorithm>
#include <cctype>
#include <climits>
#include <cstring>
#include <exception>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "gguf.h"
#include "qkv.h"

struct qkv_tokenizer {
    std::vector<std::string> id_to_token;
    std::unordered_map<std::string, int32_t> vocab;          // token -> id (the last id of a repeated token)
    std::unordered_map<std::string, int32_t> merge_rank;     // "a b" -> rank
    std::vector<std::pair<std::string, int32_t>> specials;   // longest first, then by text
    std::vector<unsigned char> special;                      // 1: one of the special tokens
    std::unordered_map<std::string, unsigned char> byte_of;  // byte symbol (UTF-8) -> byte
    std::string symbol[256];                                 // byte -> byte symbol (UTF-8)
    int32_t eos = -1;
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

// Code point of the UTF-8 sequence at s (its length in *adv, 1 for a byte
// that starts none), reading no further than `left` bytes.
int code_point(const char *s, int left, int *adv) {
    const unsigned char c = static_cast<unsigned char>(s[0]);
    const int n = piece_len(c, left);
    *adv = n;
    if (n == 1) return c;
    int cp = n == 2 ? (c & 0x1F) : n == 3 ? (c & 0x0F) : (c & 0x07);
    for (int k = 1; k < n; ++k) cp = (cp << 6) | (static_cast<unsigned char>(s[k]) & 0x3F);
    return cp;
}

// The reference's reading of a segment (src/tokenizer.cpp:71-96 inside the
// loops of :140-262): the code point at s takes the whole length its lead
// byte announces, even where the segment ends sooner, and a chunk is cut with
// that length.  Past the end the reference reads the segment's string
// terminator (zero) and, for a sequence short by two or three bytes, the
// bytes after it, which were zero in its runs here.  pre_tokenize therefore
// reads a copy of the segment followed by three zero bytes: a sequence cut
// off at a segment's end gives a chunk ending in zero bytes, byte-level
// encoded like any other byte, as the reference does.
int code_point_padded(const char *s, int *adv) {
    const unsigned char c = static_cast<unsigned char>(s[0]);
    const int n = piece_len(c, 4);
    *adv = n;
    if (n == 1) return c;
    int cp = n == 2 ? (c & 0x1F) : n == 3 ? (c & 0x0F) : (c & 0x07);
    for (int k = 1; k < n; ++k) cp = (cp << 6) | (static_cast<unsigned char>(s[k]) & 0x3F);
    return cp;
}

bool is_letter(int cp) {
    if ((cp >= 'A' && cp <= 'Z') || (cp >= 'a' && cp <= 'z')) return true;
    if (cp < 0x80) return false;
    return (cp >= 0xC0 && cp <= 0x024F && cp != 0xD7 && cp != 0xF7) || (cp >= 0x0370 && cp <= 0x1FFF) ||
           (cp >= 0x2C00 && cp <= 0x2DFF) || (cp >= 0x3040 && cp <= 0x9FFF) || (cp >= 0xAC00 && cp <= 0xD7AF) ||
           (cp >= 0xF900 && cp <= 0xFAFF) || cp >= 0x10000;
}
bool is_digit(int cp) { return cp >= '0' && cp <= '9'; }
bool is_newline(int cp) { return cp == '\n' || cp == '\r'; }
bool is_space(int cp) { return cp == ' ' || cp == '\t' || cp == 0x0B || cp == 0x0C || cp == 0xA0; }

std::vector<std::string> pre_tokenize(const std::string &text) {
    std::vector<std::string> chunks;
    const std::string padded = text + std::string(3, '\0');   // reads and chunks may run 3 bytes past the end
    const char *s = padded.data();
    const int len = static_cast<int>(text.size());
    auto run = [&](int i, bool (*keep)(int)) {   // end of the run of `keep` code points from i
        while (i < len) {
            int a = 0;
            if (!keep(code_point_padded(s + i, &a))) break;
            i += a;
        }
        return i;
    };
    int i = 0;
    while (i < len) {
        int adv = 0;
        const int cp = code_point_padded(s + i, &adv);
        if (cp == '\'' && i + adv < len) {
            static const char *suffixes[] = {"ll", "re", "ve", "s", "t", "m", "d"};
            const char *rest = s + i + adv;
            const int rlen = len - i - adv;
            bool matched = false;
            for (const char *suf : suffixes) {
                const int sl = static_cast<int>(std::strlen(suf));
                if (rlen < sl) continue;
                bool ok = true;
                for (int k = 0; k < sl && ok; ++k) ok = std::tolower(static_cast<unsigned char>(rest[k])) == suf[k];
                if (ok) {
                    chunks.emplace_back(s + i, static_cast<size_t>(adv + sl));
                    i += adv + sl;
                    matched = true;
                    break;
                }
            }
            if (matched) continue;
        }
        if (is_space(cp) && i + adv < len) {
            int a2 = 0;
            if (is_letter(code_point_padded(s + i + adv, &a2))) {
                const int end = run(i + adv + a2, is_letter);
                chunks.emplace_back(s + i, static_cast<size_t>(end - i));
                i = end;
                continue;
            }
        }
        int end;
        if (is_letter(cp)) end = run(i + adv, is_letter);
        else if (is_digit(cp)) end = i + adv;
        else if (is_newline(cp)) end = run(i + adv, is_newline);
        else if (is_space(cp)) end = run(i + adv, is_space);
        else end = run(i + adv, [](int c) { return !(is_letter(c) || is_digit(c) || is_newline(c) || is_space(c)); });
        chunks.emplace_back(s + i, static_cast<size_t>(end - i));
        i = end;
    }
    return chunks;
}

void encode_chunk(const qkv_tokenizer *t, const std::string &chunk, std::vector<int32_t> *ids) {
    std::string mapped;
    for (unsigned char c : chunk) mapped += t->symbol[c];
    std::vector<std::string> work;
    for (int i = 0, L = static_cast<int>(mapped.size()); i < L;) {
        int adv = 0;
        code_point(mapped.data() + i, L - i, &adv);
        work.emplace_back(mapped, static_cast<size_t>(i), static_cast<size_t>(adv));
        i += adv;
    }
    while (work.size() > 1) {
        int best = -1;
        int32_t best_rank = INT32_MAX;
        for (size_t i = 0; i + 1 < work.size(); ++i) {
            const auto it = t->merge_rank.find(work[i] + " " + work[i + 1]);
            if (it != t->merge_rank.end() && it->second < best_rank) {
                best_rank = it->second;
                best = static_cast<int>(i);
            }
        }
        if (best < 0) break;
        work[static_cast<size_t>(best)] += work[static_cast<size_t>(best) + 1];
        work.erase(work.begin() + best + 1);
    }
    for (const std::string &piece : work) {
        const auto it = t->vocab.find(piece);
        if (it != t->vocab.end()) ids->push_back(it->second);
    }
}

std::vector<int32_t> encode(const qkv_tokenizer *t, const std::string &text, bool add_eos) {
    std::vector<int32_t> ids;
    auto segment = [&](const std::string &seg) {
        for (const std::string &c : pre_tokenize(seg)) encode_chunk(t, c, &ids);
    };
    size_t pos = 0;
    while (pos < text.size()) {
        size_t best_pos = std::string::npos;
        int best = -1;
        for (size_t i = 0; i < t->specials.size(); ++i) {
            const size_t p = text.find(t->specials[i].first, pos);
            if (p != std::string::npos &&
                (p < best_pos || (p == best_pos && best >= 0 &&
                                  t->specials[i].first.size() > t->specials[static_cast<size_t>(best)].first.size()))) {
                best_pos = p;
                best = static_cast<int>(i);
            }
        }
        if (best < 0) {
            segment(text.substr(pos));
            break;
        }
        if (best_pos > pos) segment(text.substr(pos, best_pos - pos));
        ids.push_back(t->specials[static_cast<size_t>(best)].second);
        pos = best_pos + t->specials[static_cast<size_t>(best)].first.size();
    }
    if (add_eos && t->eos >= 0) ids.push_back(t->eos);
    return ids;
}

int emit_ids(const std::vector<int32_t> &v, int32_t *out, size_t cap, size_t *n) {
    *n = v.size();
    if (v.size() > cap || (!v.empty() && !out)) return QKV_ERR_CAPACITY;
    if (!v.empty()) std::memcpy(out, v.data(), v.size() * sizeof(int32_t));
    return QKV_OK;
}

// The C entry points return a status.  Their tables and strings are sized by
// the caller's input (a long text, a prompt with many audio placeholders) or
// the file's vocabulary; an allocation failure there becomes a status instead
// of an exception crossing the C ABI.  A distinct status, so that it is not
// mistaken for the capacity protocol's "give me a larger buffer".
template <typename F> int no_throw(F &&body) {
    try {
        return body();
    } catch (const std::exception &) {
        return QKV_ERR_HOST_MEMORY;
    }
}

int open_tokenizer(const char *gguf_path, qkv_tokenizer **out, char *err, size_t err_len) {
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
    auto t = std::make_unique<qkv_tokenizer>();
    t->id_to_token = tokens->strs;
    t->special.assign(t->id_to_token.size(), 0);
    for (size_t i = 0; i < t->id_to_token.size(); ++i) t->vocab[t->id_to_token[i]] = static_cast<int32_t>(i);
    const qkv::GgufValue *merges = f.value("tokenizer.ggml.merges");
    for (size_t i = 0; i < merges->strs.size(); ++i) t->merge_rank[merges->strs[i]] = static_cast<int32_t>(i);
    uint32_t eos = 0;
    if (f.get_u32("tokenizer.ggml.eos_token_id", &eos)) t->eos = static_cast<int32_t>(eos);
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
            return QKV_ERR_FORMAT;
        }
        if (id >= t->special.size()) {
            set_err(err, err_len, std::string("tokenizer special id out of range for key: ") + k);
            return QKV_ERR_FORMAT;
        }
        // A special joins the list (and is skipped by decode) unless its token
        // is empty or already listed under an earlier key, as :265-281 keep it.
        const std::string &tok = t->id_to_token[id];
        bool seen = tok.empty();
        for (const auto &sp : t->specials) seen = seen || sp.first == tok;
        if (!seen) {
            t->specials.emplace_back(tok, static_cast<int32_t>(id));
            t->special[id] = 1;
        }
    }
    std::sort(t->specials.begin(), t->specials.end(), [](const auto &a, const auto &b) {
        return a.first.size() != b.first.size() ? a.first.size() > b.first.size() : a.first < b.first;
    });
    // byte symbols: printable bytes keep their code point, the rest get 256, 257, ...
    int extra = 0;
    for (int b = 0; b < 256; ++b) {
        const bool printable = (b >= 0x21 && b <= 0x7E) || (b >= 0xA1 && b <= 0xAC) || (b >= 0xAE && b <= 0xFF);
        t->symbol[b] = utf8(printable ? b : 256 + extra++);
        t->byte_of[t->symbol[b]] = static_cast<unsigned char>(b);
    }
    *out = t.release();
    return QKV_OK;
}

}  // namespace

extern "C" {

int qkv_tokenizer_open(const char *gguf_path, qkv_tokenizer **out, char *err, size_t err_len) {
    if (!gguf_path || !out) {
        set_err(err, err_len, "qkv_tokenizer_open: null path or out");
        return QKV_ERR_INVALID_ARG;
    }
    try {
        return open_tokenizer(gguf_path, out, err, err_len);
    } catch (const std::exception &) {
        set_err(err, err_len, "tokenizer tables do not fit in host memory");
        return QKV_ERR_HOST_MEMORY;
    }
}

int qkv_tokenizer_decode(const qkv_tokenizer *t, const int32_t *ids, int32_t n, int32_t skip_special, char *out,
                         size_t cap, size_t *len) {
    if (!t || (n > 0 && !ids) || !len) return QKV_ERR_INVALID_ARG;
    return no_throw([&] {
        std::string s;
        for (int32_t k = 0; k < n; ++k) {
            const int32_t id = ids[k];
            if (id < 0 || static_cast<size_t>(id) >= t->id_to_token.size()) continue;
            if (skip_special && t->special[static_cast<size_t>(id)]) continue;
            const std::string &tok = t->id_to_token[static_cast<size_t>(id)];
            const int L = static_cast<int>(tok.size());
            for (int pos = 0; pos < L;) {
                // A piece is the sequence the lead byte announces; one cut off at
                // the token's end runs on into zero bytes, as the reference's
                // piece does (it reads the token's terminator: :513-516).
                const int adv = piece_len(static_cast<unsigned char>(tok[static_cast<size_t>(pos)]), 4);
                std::string piece = tok.substr(static_cast<size_t>(pos), static_cast<size_t>(adv));
                piece.resize(static_cast<size_t>(adv), '\0');
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
    });
}

int qkv_tokenizer_encode(const qkv_tokenizer *t, const char *text, size_t text_len, int32_t add_eos, int32_t *ids,
                         size_t cap, size_t *n) {
    if (!t || (text_len > 0 && !text) || !n) return QKV_ERR_INVALID_ARG;
    return no_throw([&] { return emit_ids(encode(t, std::string(text ? text : "", text_len), add_eos != 0), ids, cap, n); });
}

int qkv_asr_prompt_ids(const qkv_tokenizer *t, int32_t audio_tokens, const char *system_text, const char *language,
                       int32_t *ids, size_t cap, size_t *n) {
    if (!t || !n) return QKV_ERR_INVALID_ARG;
    return no_throw([&] {
        // the template of src/tokenizer.cpp:529-549
        std::string p = "<|im_start|>system\n";
        p += system_text ? system_text : "";
        p += "<|im_end|>\n<|im_start|>user\n<|audio_start|>";
        for (int32_t i = 0; i < audio_tokens; ++i) p += "<|audio_pad|>";
        p += "<|audio_end|><|im_end|>\n<|im_start|>assistant\n";
        if (language && language[0]) {
            p += "language ";
            p += language;
            p += "<asr_text>";
        }
        return emit_ids(encode(t, p, false), ids, cap, n);
    });
}

void qkv_tokenizer_close(qkv_tokenizer *t) { delete t; }

}  // extern "C"
