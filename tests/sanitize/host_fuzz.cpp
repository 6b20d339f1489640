// Host-side fuzz driver, built with -fsanitize=address,undefined by
// tests/test_host_sanitize.py: the page allocator, the GGUF parser and the
// byte-level BPE tokenizer run on seeded random operations and inputs, each
// checked against a property that needs no reference:
//
//   pager SEED ITERS            open / append / close / compact against a shadow
//                               model (lengths, page counts, free pages, the
//                               out-of-pages and per-stream limits, check() == 0)
//   gguf FILE SCRATCH SEED ITERS   byte flips, extreme u64 fields and truncations of
//                               a valid file's metadata: every open returns a status,
//                               and every tensor of a file that opens lies inside it
//   tokenizer FILE SEED ITERS   (a file whose vocabulary holds all 256 byte
//                               symbols) decode(encode(text)) == text up to zero
//                               bytes for random byte strings, decode of arbitrary
//                               ids, and the ASR prompt template's ids decode back
//                               to its text (the encoder adds a zero byte for each
//                               byte missing from a UTF-8 sequence cut off at the
//                               end of a segment, as the reference does, and
//                               nothing else)
//
// Exit status 0 when every property held; a sanitizer report aborts the run.
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <random>
#include <string>
#include <vector>

#include "gguf.h"
#include "pager.h"
#include "qkv.h"

namespace {

int failures = 0;

void expect(bool ok, const std::string &what) {
    if (!ok) {
        if (failures < 20) std::fprintf(stderr, "FAIL: %s\n", what.c_str());
        ++failures;
    }
}

// ---- pager ----

int fuzz_pager(uint32_t seed, int iters) {
    std::mt19937_64 rng(seed);
    const int64_t n_pages = 64 + static_cast<int64_t>(rng() % 192);
    const int32_t max_streams = 2 + static_cast<int32_t>(rng() % 7);
    const int32_t max_per_stream = 4 + static_cast<int32_t>(rng() % 40);
    const int32_t page = 16;
    qkv::Pager p(n_pages, page, max_streams, max_per_stream, seed);
    std::vector<int32_t> len(static_cast<size_t>(max_streams), -1);   // -1: closed
    auto pages_of = [&](int32_t tokens) { return (static_cast<int64_t>(tokens) + page - 1) / page; };
    auto used = [&]() {
        int64_t u = 0;
        for (int32_t l : len) u += l >= 0 ? pages_of(l) : 0;
        return u;
    };
    for (int it = 0; it < iters; ++it) {
        const int op = static_cast<int>(rng() % 10);
        const std::string at = " (op " + std::to_string(op) + ", iteration " + std::to_string(it) + ")";
        if (op < 2) {
            int32_t s = -1;
            const int rc = p.open(&s, nullptr);
            const bool room = std::count(len.begin(), len.end(), -1) > 0;
            expect((rc == QKV_OK) == room, "open succeeds iff a slot is free" + at);
            if (rc == QKV_OK) {
                expect(s >= 0 && s < max_streams && len[static_cast<size_t>(s)] == -1, "open returns a free slot" + at);
                if (s >= 0 && s < max_streams) len[static_cast<size_t>(s)] = 0;
            }
        } else if (op < 7) {
            const int32_t s = static_cast<int32_t>(rng() % static_cast<uint64_t>(max_streams + 1)) - (rng() % 8 == 0 ? 1 : 0);
            const int32_t tokens = static_cast<int32_t>(rng() % 70) - (rng() % 16 == 0 ? 5 : 0);
            std::vector<int32_t> added;
            const int rc = p.append(s, tokens, &added, nullptr);
            const bool open = s >= 0 && s < max_streams && len[static_cast<size_t>(s)] >= 0;
            if (!open || tokens < 0) {
                expect(rc == QKV_ERR_INVALID_ARG, "append on a closed stream or negative count is rejected" + at);
                continue;
            }
            const int32_t old = len[static_cast<size_t>(s)];
            const int64_t need = pages_of(old + tokens);
            const int64_t extra = need - pages_of(old);
            const int64_t free_pages = n_pages - used();
            if (need > max_per_stream) {
                expect(rc == QKV_ERR_CAPACITY, "per-stream page limit" + at);
            } else if (extra > free_pages) {
                expect(rc == QKV_ERR_OUT_OF_PAGES, "out of pages" + at);
            } else {
                expect(rc == QKV_OK, "append within limits succeeds" + at);
                expect(static_cast<int64_t>(added.size()) == extra, "append adds exactly the pages it needs" + at);
                len[static_cast<size_t>(s)] = old + tokens;
            }
            if (rc != QKV_OK) expect(added.empty(), "a failed append adds nothing" + at);
        } else if (op < 9) {
            const int32_t s = static_cast<int32_t>(rng() % static_cast<uint64_t>(max_streams));
            const int rc = p.close(s, nullptr);
            expect((rc == QKV_OK) == (len[static_cast<size_t>(s)] >= 0), "close succeeds iff the stream is open" + at);
            len[static_cast<size_t>(s)] = -1;
        } else {
            std::vector<int32_t> src, dst;
            p.compact(&src, &dst);
            const int64_t live = used();
            expect(src.size() == dst.size(), "compaction moves are pairs" + at);
            for (size_t k = 0; k < src.size(); ++k) {
                expect(src[k] >= live && dst[k] < live, "compaction moves live pages down" + at);
            }
            for (int32_t s = 0; s < max_streams; ++s) {
                const std::vector<int32_t> *pg = p.pages(s);
                if (!pg) continue;
                for (int32_t q : *pg) expect(q >= 0 && q < live, "after compaction every page is below the live count" + at);
            }
        }
        expect(p.check(nullptr) == 0, "pager consistency" + at);
        expect(p.free_pages() == n_pages - used(), "free pages match the shadow model" + at);
        for (int32_t s = 0; s < max_streams; ++s) {
            int32_t t = -1;
            const int rc = p.length(s, &t, nullptr);
            if (len[static_cast<size_t>(s)] >= 0) expect(rc == QKV_OK && t == len[static_cast<size_t>(s)], "length matches" + at);
            const std::vector<int32_t> *pg = p.pages(s);
            if (len[static_cast<size_t>(s)] >= 0 && pg) {
                expect(static_cast<int64_t>(pg->size()) == pages_of(len[static_cast<size_t>(s)]), "page count matches" + at);
            }
        }
    }
    return failures;
}

// ---- gguf ----

bool read_file(const char *path, std::vector<uint8_t> *out) {
    std::ifstream in(path, std::ios::binary);
    if (!in) return false;
    out->assign(std::istreambuf_iterator<char>(in), std::istreambuf_iterator<char>());
    return true;
}

bool write_file(const char *path, const uint8_t *data, size_t n) {
    std::ofstream out(path, std::ios::binary | std::ios::trunc);
    out.write(reinterpret_cast<const char *>(data), static_cast<std::streamsize>(n));
    return static_cast<bool>(out);
}

void check_opened(const qkv::GgufFile &f, const std::string &at) {
    const uint8_t *lo = f.mapping(), *hi = f.mapping() + f.file_size();
    for (const qkv::GgufTensor &t : f.tensors()) {
        expect(t.data >= lo && t.data <= hi && t.nbytes <= static_cast<size_t>(hi - t.data),
               "tensor " + t.name + " lies inside the file" + at);
        if (t.nbytes) {
            volatile uint8_t first = t.data[0], last = t.data[t.nbytes - 1];   // touch both ends
            (void)first;
            (void)last;
        }
    }
}

int fuzz_gguf(const char *path, const char *scratch, uint32_t seed, int iters) {
    std::vector<uint8_t> orig;
    if (!read_file(path, &orig)) {
        std::fprintf(stderr, "cannot read %s\n", path);
        return 1;
    }
    qkv::GgufFile base;
    std::string err;
    if (base.open(path, &err) != QKV_OK) {
        std::fprintf(stderr, "the unmodified file does not open: %s\n", err.c_str());
        return 1;
    }
    const size_t meta = base.data_offset();   // mutate the header, key/values and tensor infos
    base.close();
    std::mt19937_64 rng(seed);
    static const uint64_t extremes[] = {0, 1, 7, 8, 0xFFFFFFFFull, 0x7FFFFFFFFFFFFFFFull, 0xFFFFFFFFFFFFFFFFull,
                                        1ull << 40, 1ull << 32};
    int opened = 0;
    for (int it = 0; it < iters; ++it) {
        std::vector<uint8_t> d = orig;
        size_t n = d.size();
        const int kind = static_cast<int>(rng() % 4);
        if (kind == 0) {   // a few byte flips
            const int flips = 1 + static_cast<int>(rng() % 4);
            for (int k = 0; k < flips; ++k) d[rng() % meta] ^= static_cast<uint8_t>(1u << (rng() % 8));
        } else if (kind == 1) {   // an extreme 64-bit field (lengths, counts, dims, offsets are u64)
            const size_t pos = rng() % (meta - 8);
            uint64_t v = extremes[rng() % (sizeof extremes / sizeof extremes[0])];
            if (rng() % 2) v = orig.size() + (rng() % 64) - 32;
            std::memcpy(&d[pos], &v, 8);
        } else if (kind == 2) {   // a 32-bit field (types, dimension counts)
            const size_t pos = rng() % (meta - 4);
            const uint32_t v = static_cast<uint32_t>(rng() % 3 ? rng() % 40 : rng());
            std::memcpy(&d[pos], &v, 4);
        } else {   // truncation
            n = rng() % (orig.size() + 1);
        }
        if (!write_file(scratch, d.data(), n)) {
            std::fprintf(stderr, "cannot write %s\n", scratch);
            return 1;
        }
        const std::string at = " (kind " + std::to_string(kind) + ", iteration " + std::to_string(it) + ")";
        qkv::GgufFile f;
        const int rc = f.open(scratch, &err);
        expect(rc == QKV_OK || rc == QKV_ERR_FORMAT || rc == QKV_ERR_IO || rc == QKV_ERR_HOST_MEMORY,
               "open returns a parse status, got " + std::to_string(rc) + at);
        if (rc == QKV_OK) {
            ++opened;
            check_opened(f, at);
        }
        f.close();
        qkv_tokenizer *tok = nullptr;
        char msg[256];
        if (qkv_tokenizer_open(scratch, &tok, msg, sizeof msg) == QKV_OK) {   // whatever the tables hold
            std::vector<int32_t> ids(64);
            size_t m = 0;
            qkv_tokenizer_encode(tok, "hello 123 <|im_end|> x", 22, 1, ids.data(), ids.size(), &m);
            std::string out(256, '\0');
            size_t len = 0;
            qkv_tokenizer_decode(tok, ids.data(), static_cast<int32_t>(std::min(m, ids.size())), 0, &out[0], out.size(), &len);
            qkv_tokenizer_close(tok);
        }
    }
    std::printf("gguf: %d of %d mutated files opened\n", opened, iters);
    return failures;
}

// ---- tokenizer ----

std::string random_text(std::mt19937_64 &rng) {
    static const char *pieces[] = {"a", "Z", "q", " ", "  ", "\t", "\n", "\r\n", "0", "7", "'s", "'t", "'re", "'ll",
                                   "'d", "'x", "!", "?", ".", ",", "\xc3\xa9", "\xe4\xb8\xad", "\xf0\x9f\x98\x80",
                                   "\xff", "\xc3", "\x80", "<|im_start|>", "<|im_end|>", "<|audio_pad|>", "<asr_text>",
                                   "<|im_", "|>", "<", "language", " the", "hello"};
    std::string s;
    const int n = static_cast<int>(rng() % 24);
    for (int k = 0; k < n; ++k) {
        if (rng() % 6 == 0) s.push_back(static_cast<char>(rng() % 256));
        else s += pieces[rng() % (sizeof pieces / sizeof pieces[0])];
    }
    return s;
}

std::string without_zeros(std::string s) {
    s.erase(std::remove(s.begin(), s.end(), '\0'), s.end());
    return s;
}

std::vector<int32_t> encode(const qkv_tokenizer *t, const std::string &text) {
    size_t n = 0;
    std::vector<int32_t> ids(text.size() + 4);
    int rc = qkv_tokenizer_encode(t, text.data(), text.size(), 0, ids.data(), ids.size(), &n);
    if (rc == QKV_ERR_CAPACITY) {
        ids.resize(n);
        rc = qkv_tokenizer_encode(t, text.data(), text.size(), 0, ids.data(), ids.size(), &n);
    }
    expect(rc == QKV_OK, "encode succeeds");
    ids.resize(rc == QKV_OK ? n : 0);
    return ids;
}

std::string decode(const qkv_tokenizer *t, const std::vector<int32_t> &ids, int skip_special) {
    size_t n = 0;
    std::string out(8, '\0');
    int rc = qkv_tokenizer_decode(t, ids.data(), static_cast<int32_t>(ids.size()), skip_special, &out[0], out.size(), &n);
    if (rc == QKV_ERR_CAPACITY) {
        out.assign(n, '\0');
        rc = qkv_tokenizer_decode(t, ids.data(), static_cast<int32_t>(ids.size()), skip_special,
                                  out.empty() ? nullptr : &out[0], out.size(), &n);
    }
    expect(rc == QKV_OK, "decode succeeds");
    out.resize(rc == QKV_OK ? n : 0);
    return out;
}

int fuzz_tokenizer(const char *path, uint32_t seed, int iters) {
    qkv_tokenizer *t = nullptr;
    char msg[256];
    if (qkv_tokenizer_open(path, &t, msg, sizeof msg) != QKV_OK) {
        std::fprintf(stderr, "tokenizer open failed: %s\n", msg);
        return 1;
    }
    std::mt19937_64 rng(seed);
    for (int it = 0; it < iters; ++it) {
        const std::string text = random_text(rng);
        const std::vector<int32_t> ids = encode(t, text);
        const std::string back = decode(t, ids, 0);
        expect(without_zeros(back) == without_zeros(text) && back.size() >= text.size() && back.size() <= text.size() + 3 * (ids.size() + 1),
               "decode(encode(text)) == text up to zero bytes at iteration " + std::to_string(it));
        std::vector<int32_t> junk(rng() % 16);
        for (int32_t &v : junk) v = static_cast<int32_t>(rng() % 1400) - 100;   // includes negatives and ids past the vocabulary
        (void)decode(t, junk, static_cast<int>(rng() % 2));
        // The ASR prompt template (audio placeholders, optional language line).
        const int32_t audio = static_cast<int32_t>(rng() % 40);
        const std::string system = rng() % 2 ? random_text(rng) : std::string();
        const bool lang = rng() % 2;
        const std::string language = lang ? std::string("English") : std::string();
        std::string want = "<|im_start|>system\n" + system + "<|im_end|>\n<|im_start|>user\n<|audio_start|>";
        for (int32_t k = 0; k < audio; ++k) want += "<|audio_pad|>";
        want += "<|audio_end|><|im_end|>\n<|im_start|>assistant\n";
        if (lang) want += "language English<asr_text>";
        std::vector<int32_t> pids(want.size() + 4);
        size_t n = 0;
        const int rc = qkv_asr_prompt_ids(t, audio, system.c_str(), lang ? language.c_str() : nullptr, pids.data(),
                                          pids.size(), &n);
        expect(rc == QKV_OK, "prompt ids succeed");
        pids.resize(rc == QKV_OK ? n : 0);
        if (system.find('\0') == std::string::npos) {   // a C string stops at the first NUL
            expect(without_zeros(decode(t, pids, 0)) == without_zeros(want),
                   "prompt ids decode to the template at iteration " + std::to_string(it));
        }
    }
    qkv_tokenizer_close(t);
    return failures;
}

}  // namespace

int main(int argc, char **argv) {
    const std::string mode = argc > 1 ? argv[1] : "";
    if (mode == "pager" && argc == 4) return fuzz_pager(static_cast<uint32_t>(std::atoi(argv[2])), std::atoi(argv[3])) ? 1 : 0;
    if (mode == "gguf" && argc == 6)
        return fuzz_gguf(argv[2], argv[3], static_cast<uint32_t>(std::atoi(argv[4])), std::atoi(argv[5])) ? 1 : 0;
    if (mode == "tokenizer" && argc == 5)
        return fuzz_tokenizer(argv[2], static_cast<uint32_t>(std::atoi(argv[3])), std::atoi(argv[4])) ? 1 : 0;
    std::fprintf(stderr, "usage: host_fuzz pager SEED ITERS | gguf FILE SCRATCH SEED ITERS | tokenizer FILE SEED ITERS\n");
    return 2;
}
