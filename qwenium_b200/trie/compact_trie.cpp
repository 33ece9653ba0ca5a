// compact_trie.cpp -- see compact_trie.h.
#include "compact_trie.h"

#include <algorithm>
#include <cstring>
#include <numeric>

namespace qwenium_b200 {

void CompactTokenTrie::build(const std::vector<std::string>& vocab) {
    std::vector<int32_t> order;
    order.reserve(vocab.size());
    size_t total = 0;
    for (size_t i = 0; i < vocab.size(); ++i)
        if (!vocab[i].empty()) {
            order.push_back((int32_t)i);
            total += vocab[i].size();
        }
    // lexicographic over unsigned bytes (memcmp), a prefix first, equal
    // strings by ascending id: the reference trie's depth-first order
    std::sort(order.begin(), order.end(), [&](int32_t a, int32_t b) {
        const std::string& x = vocab[(size_t)a];
        const std::string& y = vocab[(size_t)b];
        const size_t n = std::min(x.size(), y.size());
        const int c = std::memcmp(x.data(), y.data(), n);
        if (c != 0) return c < 0;
        if (x.size() != y.size()) return x.size() < y.size();
        return a < b;
    });
    ids_.assign(order.begin(), order.end());
    bytes_.clear();
    bytes_.reserve(total);
    off_.assign(ids_.size() + 1, 0u);
    for (size_t j = 0; j < ids_.size(); ++j) {
        const std::string& s = vocab[(size_t)ids_[j]];
        off_[j] = (uint32_t)bytes_.size();
        bytes_.insert(bytes_.end(), s.begin(), s.end());
    }
    off_[ids_.size()] = (uint32_t)bytes_.size();
    // first-byte index (every string has at least one byte)
    uint32_t j = 0;
    for (int c = 0; c < 256; ++c) {
        first_[c] = j;
        while (j < ids_.size() && (unsigned char)bytes_[off_[j]] == c) ++j;
    }
    first_[256] = j;
    bytes_.shrink_to_fit();
}

size_t CompactTokenTrie::memory_bytes() const {
    return bytes_.capacity() + off_.capacity() * sizeof(uint32_t) + ids_.capacity() * sizeof(int32_t) +
           sizeof(first_);
}

void CompactTokenTrie::narrow(uint32_t& lo, uint32_t& hi, size_t d, unsigned char c) const {
    // byte_at(j, d) is non-decreasing over [lo, hi) (-1 for strings that
    // end at depth d, which sort first)
    uint32_t a = lo, b = hi;
    while (a < b) {  // first j with byte_at(j, d) >= c
        const uint32_t mid = a + (b - a) / 2;
        if (byte_at(mid, d) < (int)c) a = mid + 1;
        else b = mid;
    }
    uint32_t e = a, f = hi;
    while (e < f) {  // first j with byte_at(j, d) > c
        const uint32_t mid = e + (f - e) / 2;
        if (byte_at(mid, d) <= (int)c) e = mid + 1;
        else f = mid;
    }
    lo = a;
    hi = e;
}

void CompactTokenTrie::collect_by_prefix(const char* prefix, size_t len, size_t offset,
                                         std::vector<int32_t>& out) const {
    if (offset >= len) {  // the root: every token, in depth-first order
        out.insert(out.end(), ids_.begin(), ids_.end());
        return;
    }
    uint32_t lo = 0, hi = (uint32_t)ids_.size(), own_end = 0;
    for (size_t i = offset; i < len; ++i) {
        const size_t d = i - offset;
        narrow(lo, hi, d, (unsigned char)prefix[i]);
        if (lo == hi) return;  // no token continues this path
        // the tokens ending here are prefixes of prefix[offset:]
        own_end = lo;
        while (own_end < hi && off_[own_end + 1] - off_[own_end] == d + 1) out.push_back(ids_[own_end++]);
    }
    // the node's subtree without its own tokens (already collected)
    out.insert(out.end(), ids_.begin() + own_end, ids_.begin() + hi);
}

void CompactTokenTrie::collect_by_prefix(const std::string& prefix, size_t offset, std::vector<int32_t>& out) const {
    collect_by_prefix(prefix.data(), prefix.size(), offset, out);
}

void CompactTokenTrie::allowed_first_bytes(const std::set<char>& chars, bool negated, bool allowed[256]) const {
    for (int c = 0; c < 256; ++c) allowed[c] = negated;
    for (char c : chars) allowed[(unsigned char)c] = !negated;
}

void CompactTokenTrie::collect_by_char_class(const std::set<char>& chars, bool negated,
                                             std::vector<int32_t>& out) const {
    bool allowed[256];
    allowed_first_bytes(chars, negated, allowed);
    for (int c = 0; c < 256; ++c)
        if (allowed[c]) out.insert(out.end(), ids_.begin() + first_[c], ids_.begin() + first_[c + 1]);
}

void CompactTokenTrie::collect_by_first_char(char c, std::vector<int32_t>& out) const {
    const unsigned char u = (unsigned char)c;
    out.insert(out.end(), ids_.begin() + first_[u], ids_.begin() + first_[u + 1]);
}

void CompactTokenTrie::mark_char_class(const std::set<char>& chars, bool negated,
                                       std::vector<bool>& valid_mask) const {
    bool allowed[256];
    allowed_first_bytes(chars, negated, allowed);
    for (int c = 0; c < 256; ++c)
        if (allowed[c])
            for (uint32_t j = first_[c]; j < first_[c + 1]; ++j) valid_mask[(size_t)ids_[j]] = true;
}

}  // namespace qwenium_b200
