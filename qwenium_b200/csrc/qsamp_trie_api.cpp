// qsamp_trie_api.cpp -- the C ABI of the compact token trie (include/qsamp.h,
// qsamp_trie_*), over qwenium_b200::CompactTokenTrie (trie/compact_trie.h).
#include <new>
#include <set>
#include <string>
#include <vector>

#include "../../include/qsamp.h"
#include "../trie/compact_trie.h"

struct qsamp_trie {
    qwenium_b200::CompactTokenTrie t;
};

namespace {

std::set<char> char_set(const uint8_t* chars, int32_t n) {
    std::set<char> s;
    for (int32_t i = 0; i < n; ++i) s.insert((char)chars[i]);
    return s;
}

int64_t emit(const std::vector<int32_t>& v, int32_t* out, int64_t cap) {
    const int64_t n = (int64_t)v.size();
    for (int64_t i = 0; i < n && i < cap; ++i) out[i] = v[(size_t)i];
    return n;
}

}  // namespace

extern "C" {

qsamp_status qsamp_trie_build(const char* const* strs, const int32_t* lens, int32_t V, qsamp_trie** out) {
    if (!out) return QSAMP_ERR_INVALID_ARG;
    *out = nullptr;
    if (V < 0 || (V > 0 && (!strs || !lens))) return QSAMP_ERR_INVALID_ARG;
    qsamp_trie* t = new (std::nothrow) qsamp_trie();
    if (!t) return QSAMP_ERR_NO_MEMORY;
    try {
        std::vector<std::string> vocab((size_t)V);
        for (int32_t i = 0; i < V; ++i) {
            if (lens[i] < 0 || (lens[i] > 0 && !strs[i])) {
                delete t;
                return QSAMP_ERR_INVALID_ARG;
            }
            if (lens[i] > 0) vocab[(size_t)i].assign(strs[i], (size_t)lens[i]);
        }
        t->t.build(vocab);
    } catch (const std::bad_alloc&) {
        delete t;
        return QSAMP_ERR_NO_MEMORY;
    }
    *out = t;
    return QSAMP_OK;
}

void qsamp_trie_free(qsamp_trie* t) { delete t; }

int64_t qsamp_trie_token_count(const qsamp_trie* t) { return t ? (int64_t)t->t.token_count() : -1; }

int64_t qsamp_trie_memory_bytes(const qsamp_trie* t) { return t ? (int64_t)t->t.memory_bytes() : -1; }

int64_t qsamp_trie_collect_by_prefix(const qsamp_trie* t, const char* prefix, int32_t len, int32_t offset,
                                     int32_t* out, int64_t cap) {
    if (!t || len < 0 || offset < 0 || (len > 0 && !prefix) || (cap > 0 && !out)) return -1;
    std::vector<int32_t> v;
    t->t.collect_by_prefix(prefix ? prefix : "", (size_t)len, (size_t)offset, v);
    return emit(v, out, cap);
}

int64_t qsamp_trie_collect_by_char_class(const qsamp_trie* t, const uint8_t* chars, int32_t n, int32_t negated,
                                         int32_t* out, int64_t cap) {
    if (!t || n < 0 || (n > 0 && !chars) || (cap > 0 && !out)) return -1;
    std::vector<int32_t> v;
    t->t.collect_by_char_class(char_set(chars, n), negated != 0, v);
    return emit(v, out, cap);
}

int64_t qsamp_trie_collect_by_first_char(const qsamp_trie* t, uint8_t c, int32_t* out, int64_t cap) {
    if (!t || (cap > 0 && !out)) return -1;
    std::vector<int32_t> v;
    t->t.collect_by_first_char((char)c, v);
    return emit(v, out, cap);
}

qsamp_status qsamp_trie_mark_char_class(const qsamp_trie* t, const uint8_t* chars, int32_t n, int32_t negated,
                                        int32_t V, uint8_t* mask_out) {
    if (!t || n < 0 || (n > 0 && !chars) || V < 0 || (V > 0 && !mask_out)) return QSAMP_ERR_INVALID_ARG;
    std::vector<bool> m((size_t)V, false);
    const std::set<char> cs = char_set(chars, n);
    // (ids beyond V would not fit the caller's mask: refuse rather than write past it)
    bool allowed[256];
    t->t.allowed_first_bytes(cs, negated != 0, allowed);
    for (int c = 0; c < 256; ++c) {
        if (!allowed[c]) continue;
        uint32_t lo, hi;
        t->t.first_byte_range((unsigned char)c, lo, hi);
        for (uint32_t j = lo; j < hi; ++j)
            if (t->t.sorted_ids()[j] >= V) return QSAMP_ERR_INVALID_ARG;
    }
    t->t.mark_char_class(cs, negated != 0, m);
    for (int32_t i = 0; i < V; ++i) mask_out[i] = m[(size_t)i] ? 1 : 0;
    return QSAMP_OK;
}

}  // extern "C"
