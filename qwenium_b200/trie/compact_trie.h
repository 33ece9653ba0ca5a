// compact_trie.h -- a flat token trie for grammar-constrained decoding.
//
// Same queries, with the same results in the same order, as the reference's
// qwenium::TokenTrie (src/sampling/token-trie.h:20-64, token-trie.cpp:8-126),
// without its 256-pointer nodes (token-trie.h:11-16): the reference spends
// 2 KB of child pointers per node, about 2.1 GB and 29 s of build time on a
// 151,936-token byte vocabulary; this one stores the non-empty token strings
// once, sorted.
//
// Representation. The reference's depth-first collection order (a node's own
// tokens by ascending id, then its children by ascending byte) is the
// lexicographic order of the token strings over unsigned bytes, a string
// before its extensions, equal strings by ascending id. The tokens are kept
// in exactly that order (ids_, with their bytes concatenated in bytes_ and
// delimited by off_), so every trie node is a contiguous range of that
// array: the node of a prefix P holds the tokens whose string starts with P,
// the tokens equal to P first. A walk narrows the range one byte at a time by
// binary search; a subtree collection copies the range.
//
// Build: O(n log n) string compares; memory: the token bytes plus 8 bytes per
// token plus a 257-entry first-byte index. Immutable after build(), so
// concurrent queries are safe.
#pragma once

#include <cstddef>
#include <cstdint>
#include <set>
#include <string>
#include <vector>

namespace qwenium_b200 {

class CompactTokenTrie {
public:
    // vocab[i] is the decoded string of token i; empty strings are skipped
    // (token-trie.cpp:18).
    void build(const std::vector<std::string>& vocab);

    // Tokens whose string is a prefix of prefix[offset:] (shortest first),
    // then the tokens that extend prefix[offset:] (token-trie.cpp:39-70).
    void collect_by_prefix(const std::string& prefix, size_t offset, std::vector<int32_t>& out) const;
    // Tokens whose first byte is (negated: is not) in chars, by first byte.
    void collect_by_char_class(const std::set<char>& chars, bool negated, std::vector<int32_t>& out) const;
    // Tokens whose first byte is c.
    void collect_by_first_char(char c, std::vector<int32_t>& out) const;
    // valid_mask[id] = true for the tokens collect_by_char_class returns
    // (valid_mask holds at least as many entries as the vocabulary).
    void mark_char_class(const std::set<char>& chars, bool negated, std::vector<bool>& valid_mask) const;

    size_t token_count() const { return ids_.size(); }
    // Bytes held by the trie (its arrays' capacities).
    size_t memory_bytes() const;

    // The same queries with plain outputs (the C ABI uses them).
    void collect_by_prefix(const char* prefix, size_t len, size_t offset, std::vector<int32_t>& out) const;
    void allowed_first_bytes(const std::set<char>& chars, bool negated, bool allowed[256]) const;
    void first_byte_range(unsigned char c, uint32_t& lo, uint32_t& hi) const {
        lo = first_[c];
        hi = first_[c + 1];
    }
    const int32_t* sorted_ids() const { return ids_.data(); }

private:
    std::vector<char> bytes_;     // token strings in sorted order, concatenated
    std::vector<uint32_t> off_;   // string j is bytes_[off_[j], off_[j + 1])
    std::vector<int32_t> ids_;    // token id of sorted string j
    uint32_t first_[257] = {};    // sorted range of the strings starting with byte c

    // Byte d of sorted string j, or -1 when the string has only d bytes.
    int byte_at(uint32_t j, size_t d) const {
        return off_[j] + d < off_[j + 1] ? (int)(unsigned char)bytes_[off_[j] + d] : -1;
    }
    // Within [lo, hi), whose strings share their first d bytes, the range of
    // strings whose byte d is c.
    void narrow(uint32_t& lo, uint32_t& hi, size_t d, unsigned char c) const;
};

}  // namespace qwenium_b200
