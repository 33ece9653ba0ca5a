// token-trie.h -- drop-in replacement of the reference's token trie header
// (src/sampling/token-trie.h of rye-001/Qwenium): the same qwenium::TokenTrie
// class and public interface (build, collect_by_prefix,
// collect_by_char_class, collect_by_first_char, mark_char_class,
// token_count; non-copyable, movable), backed by the flat sorted-string trie
// of compact_trie.h instead of 256-pointer nodes. Results are identical,
// element for element, so GrammarVocab::get_valid_tokens
// (grammar_vocab.cpp:571-755) is unchanged. To use it, build the reference's
// src/sampling with this header in place of its token-trie.h and
// compact_trie.cpp in place of its token-trie.cpp.
#pragma once

#include <cstdint>
#include <set>
#include <string>
#include <vector>

#include "compact_trie.h"

namespace qwenium {

class TokenTrie {
public:
    TokenTrie() = default;
    ~TokenTrie() = default;
    TokenTrie(const TokenTrie&) = delete;
    TokenTrie& operator=(const TokenTrie&) = delete;
    TokenTrie(TokenTrie&&) = default;
    TokenTrie& operator=(TokenTrie&&) = default;

    void build(const std::vector<std::string>& vocab) { impl_.build(vocab); }
    void collect_by_prefix(const std::string& prefix, size_t offset, std::vector<int32_t>& out) const {
        impl_.collect_by_prefix(prefix, offset, out);
    }
    void collect_by_char_class(const std::set<char>& chars, bool negated, std::vector<int32_t>& out) const {
        impl_.collect_by_char_class(chars, negated, out);
    }
    void collect_by_first_char(char c, std::vector<int32_t>& out) const { impl_.collect_by_first_char(c, out); }
    void mark_char_class(const std::set<char>& chars, bool negated, std::vector<bool>& valid_mask) const {
        impl_.mark_char_class(chars, negated, valid_mask);
    }
    size_t token_count() const { return impl_.token_count(); }

private:
    qwenium_b200::CompactTokenTrie impl_;
};

}  // namespace qwenium
