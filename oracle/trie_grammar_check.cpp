// trie_grammar_check.cpp -- TEST INFRASTRUCTURE ONLY (the checker, never the product).
//
// The reference's GrammarVocab (src/sampling/grammar_vocab.cpp, compiled
// unmodified) with the compact trie attached in place of the reference's
// TokenTrie: oracle/Makefile compiles grammar_vocab.cpp through a directory
// of symbolic links in which "token-trie.h" is qwenium_b200/trie/token-trie.h
// (the drop-in header), so the grammar code calls the compact trie. As in the
// reference's own equivalence test (tests/unit/test_token_trie.cpp:443-464),
// every grammar state of a random walk must give the same valid set with the
// trie attached as without any trie (the brute-force scan,
// grammar_vocab.cpp:713-747).
//
// usage: trie_grammar_check GBNF_FILE VOCAB_FILE STEPS SEED
//   VOCAB_FILE: u32 count, then per token u32 length and its bytes.
// Prints one line; exit 0 iff every state agrees.
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <fstream>
#include <random>
#include <sstream>
#include <string>
#include <vector>

#include "grammar_vocab.h"
#include "token-trie.h"

static std::vector<std::string> read_vocab(const char* path) {
    std::ifstream f(path, std::ios::binary);
    uint32_t n = 0;
    f.read((char*)&n, 4);
    std::vector<std::string> v(n);
    for (uint32_t i = 0; i < n; ++i) {
        uint32_t len = 0;
        f.read((char*)&len, 4);
        v[i].resize(len);
        if (len) f.read(&v[i][0], len);
    }
    return v;
}

int main(int argc, char** argv) {
    if (argc < 5) {
        std::fprintf(stderr, "usage: %s GBNF_FILE VOCAB_FILE STEPS SEED\n", argv[0]);
        return 2;
    }
    std::ifstream g(argv[1]);
    std::stringstream ss;
    ss << g.rdbuf();
    const std::string gbnf = ss.str();
    const std::vector<std::string> vocab = read_vocab(argv[2]);
    const int steps = std::atoi(argv[3]);
    std::mt19937 rng((uint32_t)std::atoi(argv[4]));
    qwenium::TokenTrie trie;
    trie.build(vocab);
    auto with = qwenium::GrammarVocab::parse_impl(gbnf);
    auto without = qwenium::GrammarVocab::parse_impl(gbnf);
    if (!with || !without) {
        std::printf("GBNF parse failed\n");
        return 2;
    }
    with->set_token_trie(&trie);
    int bad = 0, states = 0;
    size_t largest = 0;
    for (int t = 0; t < steps; ++t) {
        std::vector<int32_t> a = with->get_valid_tokens(vocab);
        std::vector<int32_t> b = without->get_valid_tokens(vocab);
        std::sort(a.begin(), a.end());
        std::sort(b.begin(), b.end());
        ++states;
        largest = std::max(largest, b.size());
        if (a != b) {
            if (bad < 3) std::printf("  state %d: %zu ids with the trie, %zu without\n", t, a.size(), b.size());
            ++bad;
        }
        if (b.empty()) break;
        // advance both grammars by one valid token (a short one half the time,
        // so walks reach nested values)
        int32_t pick = b[std::uniform_int_distribution<size_t>(0, b.size() - 1)(rng)];
        if (rng() & 1)
            for (int32_t id : b)
                if (vocab[(size_t)id].size() == 1) {
                    if (std::uniform_int_distribution<int>(0, 3)(rng) == 0) {
                        pick = id;
                        break;
                    }
                }
        with->accept_token(pick, vocab);
        without->accept_token(pick, vocab);
    }
    std::printf("%d grammar states, %d differ (largest valid set %zu)\n", states, bad, largest);
    return bad ? 1 : 0;
}
