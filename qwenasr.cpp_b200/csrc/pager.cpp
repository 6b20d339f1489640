#include "pager.h"

#include <algorithm>

#include "qkv.h"

namespace qkv {

namespace {
uint64_t splitmix64(uint64_t *state) {
    uint64_t z = (*state += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
}  // namespace

Pager::Pager(int64_t n_pages, int32_t page_tokens, int32_t max_streams, int32_t max_pages_per_stream,
             uint32_t seed)
    : n_pages_(n_pages),
      page_tokens_(page_tokens),
      max_streams_(max_streams),
      max_pages_per_stream_(max_pages_per_stream) {
    // Hand-out order: page 0 first (stack filled in reverse), or a seeded
    // Fisher-Yates permutation of the pool so that consecutive pages of a
    // stream are scattered, as in the microbench's permuted page table.
    std::vector<int32_t> order(static_cast<size_t>(n_pages));
    for (int64_t i = 0; i < n_pages; ++i) order[static_cast<size_t>(i)] = static_cast<int32_t>(i);
    if (seed != 0) {
        uint64_t st = seed;
        for (int64_t i = n_pages - 1; i > 0; --i) {
            const int64_t j = static_cast<int64_t>(splitmix64(&st) % static_cast<uint64_t>(i + 1));
            std::swap(order[static_cast<size_t>(i)], order[static_cast<size_t>(j)]);
        }
    }
    free_.assign(order.rbegin(), order.rend());
    streams_.resize(static_cast<size_t>(max_streams));
    free_slots_.reserve(static_cast<size_t>(max_streams));
    for (int32_t s = max_streams - 1; s >= 0; --s) free_slots_.push_back(s);
}

int Pager::open(int32_t *stream_id, std::string *err) {
    if (!stream_id) {
        if (err) *err = "pager open: stream_id is null";
        return QKV_ERR_INVALID_ARG;
    }
    if (free_slots_.empty()) {
        if (err) *err = "pager open: all " + std::to_string(max_streams_) + " stream slots in use";
        return QKV_ERR_CAPACITY;
    }
    const int32_t s = free_slots_.back();
    free_slots_.pop_back();
    Stream &st = streams_[static_cast<size_t>(s)];
    st.open = true;
    st.tokens = 0;
    st.pages.clear();
    *stream_id = s;
    return QKV_OK;
}

bool Pager::is_open(int32_t s) const {
    return s >= 0 && s < max_streams_ && streams_[static_cast<size_t>(s)].open;
}

int Pager::close(int32_t s, std::string *err) {
    if (!is_open(s)) {
        if (err) *err = "pager close: stream " + std::to_string(s) + " is not open";
        return QKV_ERR_INVALID_ARG;
    }
    Stream &st = streams_[static_cast<size_t>(s)];
    // Returned pages go on top of the stack in reverse so the stream's first
    // page is reused first.
    for (auto it = st.pages.rbegin(); it != st.pages.rend(); ++it) free_.push_back(*it);
    st.pages.clear();
    st.tokens = 0;
    st.open = false;
    free_slots_.push_back(s);
    return QKV_OK;
}

int Pager::append(int32_t s, int32_t tokens, std::vector<int32_t> *added, std::string *err) {
    if (!is_open(s) || tokens < 0) {
        if (err) *err = "pager append: stream " + std::to_string(s) + " is not open or tokens < 0";
        return QKV_ERR_INVALID_ARG;
    }
    Stream &st = streams_[static_cast<size_t>(s)];
    const int64_t new_tokens = static_cast<int64_t>(st.tokens) + tokens;
    const int64_t need = (new_tokens + page_tokens_ - 1) / page_tokens_;
    if (need > max_pages_per_stream_) {
        if (err) {
            *err = "pager append: stream " + std::to_string(s) + " would need " + std::to_string(need) +
                   " pages, limit " + std::to_string(max_pages_per_stream_);
        }
        return QKV_ERR_CAPACITY;
    }
    const int64_t extra = need - static_cast<int64_t>(st.pages.size());
    if (extra > static_cast<int64_t>(free_.size())) {
        if (err) {
            *err = "pager append: out of pages (need " + std::to_string(extra) + ", free " +
                   std::to_string(free_.size()) + ")";
        }
        return QKV_ERR_OUT_OF_PAGES;
    }
    if (extra > 0) {   // reserve first: a page never leaves the free list without landing in the stream
        st.pages.reserve(static_cast<size_t>(need));
        if (added) added->reserve(added->size() + static_cast<size_t>(extra));
    }
    for (int64_t i = 0; i < extra; ++i) {
        const int32_t p = free_.back();
        free_.pop_back();
        st.pages.push_back(p);
        if (added) added->push_back(p);
    }
    st.tokens = static_cast<int32_t>(new_tokens);
    return QKV_OK;
}

int Pager::length(int32_t s, int32_t *tokens, std::string *err) const {
    if (!is_open(s) || !tokens) {
        if (err) *err = "pager length: stream " + std::to_string(s) + " is not open";
        return QKV_ERR_INVALID_ARG;
    }
    *tokens = streams_[static_cast<size_t>(s)].tokens;
    return QKV_OK;
}

const std::vector<int32_t> *Pager::pages(int32_t s) const {
    return is_open(s) ? &streams_[static_cast<size_t>(s)].pages : nullptr;
}

void Pager::compact(std::vector<int32_t> *src, std::vector<int32_t> *dst) {
    const int64_t live = n_pages_ - static_cast<int64_t>(free_.size());
    std::vector<int32_t> low_free;
    for (int32_t p : free_) {
        if (p < live) low_free.push_back(p);
    }
    std::sort(low_free.begin(), low_free.end());
    // Every move fills one low free page, so the lists never outgrow
    // low_free: reserving them here means nothing below allocates, and an
    // allocation failure leaves the pager as it was.
    if (src) src->reserve(src->size() + low_free.size());
    if (dst) dst->reserve(dst->size() + low_free.size());
    size_t next = 0;
    for (Stream &st : streams_) {
        if (!st.open) continue;
        for (int32_t &p : st.pages) {
            if (p >= live) {
                const int32_t to = low_free[next++];
                if (src) src->push_back(p);
                if (dst) dst->push_back(to);
                p = to;
            }
        }
    }
    free_.clear();
    for (int64_t p = n_pages_ - 1; p >= live; --p) free_.push_back(static_cast<int32_t>(p));
}

int Pager::check(std::string *err) const {
    std::vector<uint8_t> seen(static_cast<size_t>(n_pages_), 0);
    auto mark = [&](int32_t p, const char *what) -> bool {
        if (p < 0 || p >= n_pages_) {
            if (err) *err = std::string(what) + ": page id out of range: " + std::to_string(p);
            return false;
        }
        if (seen[static_cast<size_t>(p)]) {
            if (err) *err = std::string(what) + ": page " + std::to_string(p) + " owned twice";
            return false;
        }
        seen[static_cast<size_t>(p)] = 1;
        return true;
    };
    for (int32_t p : free_) {
        if (!mark(p, "free list")) return QKV_ERR_STATE;
    }
    for (const Stream &st : streams_) {
        if (!st.open) continue;
        const int64_t need = (static_cast<int64_t>(st.tokens) + page_tokens_ - 1) / page_tokens_;
        if (static_cast<int64_t>(st.pages.size()) != need) {
            if (err) *err = "stream page count does not match its length";
            return QKV_ERR_STATE;
        }
        for (int32_t p : st.pages) {
            if (!mark(p, "stream")) return QKV_ERR_STATE;
        }
    }
    for (int64_t p = 0; p < n_pages_; ++p) {
        if (!seen[static_cast<size_t>(p)]) {
            if (err) *err = "page " + std::to_string(p) + " leaked";
            return QKV_ERR_STATE;
        }
    }
    return QKV_OK;
}

}  // namespace qkv
