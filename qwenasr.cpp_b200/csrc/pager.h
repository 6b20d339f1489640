// Host-side paged KV-cache allocator.
//
// The reference keeps one contiguous f32 cache per layer sized max_seq_len for
// a single stream (text-decoder.cpp:1420-1474, cur_len at :186).  Here a pool
// of fixed-size pages is shared by many streams: a page holds page_tokens
// tokens of K and V for every layer and kv head of one stream, and each stream
// owns an ordered page list (its page table row on the device).
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace qkv {

class Pager {
public:
    Pager(int64_t n_pages, int32_t page_tokens, int32_t max_streams, int32_t max_pages_per_stream,
          uint32_t seed);

    int64_t n_pages() const { return n_pages_; }
    int32_t page_tokens() const { return page_tokens_; }
    int32_t max_streams() const { return max_streams_; }
    int32_t max_pages_per_stream() const { return max_pages_per_stream_; }
    int64_t free_pages() const { return static_cast<int64_t>(free_.size()); }

    // All return 0 on success or a qkv_status code; `err` gets a message.
    int open(int32_t *stream_id, std::string *err);
    int close(int32_t stream_id, std::string *err);
    // Make room for `tokens` more tokens; the new pages (in table order) are
    // appended to *added when it is non-null.  All-or-nothing.
    int append(int32_t stream_id, int32_t tokens, std::vector<int32_t> *added, std::string *err);
    int length(int32_t stream_id, int32_t *tokens, std::string *err) const;
    const std::vector<int32_t> *pages(int32_t stream_id) const;
    bool is_open(int32_t stream_id) const;
    // Compaction plan: every live page with id >= live count moves to the
    // lowest free id; page lists are rewritten and the free list becomes
    // [live, n_pages) in ascending order.
    void compact(std::vector<int32_t> *src, std::vector<int32_t> *dst);
    // 0 when every page is owned by exactly one stream or is free.
    int check(std::string *err) const;

private:
    struct Stream {
        bool open = false;
        int32_t tokens = 0;
        std::vector<int32_t> pages;
    };
    int64_t n_pages_;
    int32_t page_tokens_;
    int32_t max_streams_;
    int32_t max_pages_per_stream_;
    std::vector<int32_t> free_;          // stack: back() is handed out next
    std::vector<Stream> streams_;
    std::vector<int32_t> free_slots_;    // stack of closed stream ids
};

}  // namespace qkv
