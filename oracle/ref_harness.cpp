// ref_harness.cpp -- TEST INFRASTRUCTURE ONLY (the checker, never the product).
//
// extern "C" shims over the reference's UNMODIFIED token-selection sources
// (src/sampling/{sampling,grammar_vocab,token-trie}.cpp of rye-001/Qwenium),
// compiled from where they lie by oracle/Makefile into oracle/_ref/*.so.
// Tests, __graft_entry__.smoke() and bench.py's cpu_baseline / reference leg
// load these libraries through ctypes (oracle/oracle.py); nothing in the
// product links or calls them.
//
// What the shims add on top of the reference API:
//   * seeding of TemperatureSampler::gen_ (private; src/sampling/sampling.h:92,
//     seeded from std::random_device in sampling.cpp:114-122). Access uses the
//     explicit-instantiation access rule, which is standard C++ and leaves the
//     class layout untouched;
//   * the per-row uniform draw u the reference's own engine will consume:
//     std::generate_canonical<double,53> on a COPY of the engine, taken right
//     before sample(), so the GPU path can be fed the identical u;
//   * a copy of the logits after sample(): the reference mutates them in place
//     (pruning, grammar mask, repetition penalty, temperature), which pins the
//     transform stage separately from the selection stage.
#include "sampling.h"
#include "grammar_vocab.h"
#include "token-trie.h"
#include "speculative.h"
#include "ref_access.h"

#include <atomic>
#include <set>
#include <cstdint>
#include <cstring>
#include <random>
#include <thread>
#include <string>
#include <unordered_set>
#include <vector>

namespace {

using qwref_access::engine_of;

struct Vocab {
    std::vector<std::string> strs;
};

}  // namespace

extern "C" {

// TemperatureSampler::sample (sampling.cpp:137-194) on one row.
//   seed      : the engine is std::mt19937(seed) before the call.
//   u_out     : generate_canonical<double,53> of a copy of that engine, i.e.
//               the uniform discrete_distribution consumes if it draws.
//   drew_out  : 1 if the engine advanced (discrete_distribution drew), else 0
//               (it does not draw for a single survivor, or for T<=0).
//   logits_out: optional [V] copy of the logits after sample() returned.
int qwref_temperature_sample(const float* logits, int V, const int32_t* hist, int H,
                             float temperature, float rep_penalty, int rep_lookback,
                             int top_k, float top_p, uint32_t seed, double* u_out,
                             int* drew_out, float* logits_out) {
    qwenium::TemperatureSampler s(temperature, rep_penalty, rep_lookback, top_k, top_p);
    std::mt19937& gen = engine_of(s);
    gen = std::mt19937(seed);
    std::mt19937 probe = gen;
    const double u = std::generate_canonical<double, 53>(probe);
    if (u_out) *u_out = u;
    std::vector<float> lv(logits, logits + V);
    std::vector<int32_t> hv(hist, hist + (H > 0 ? H : 0));
    const int id = s.sample(lv, hv, {});
    if (drew_out) *drew_out = (gen == std::mt19937(seed)) ? 0 : 1;
    if (logits_out) std::memcpy(logits_out, lv.data(), sizeof(float) * (size_t)V);
    return id;
}

// GreedySampler::sample (sampling.cpp:98-108) on one row.
int qwref_greedy_sample(const float* logits, int V, const int32_t* hist, int H,
                        float rep_penalty, int rep_lookback, float* logits_out) {
    qwenium::GreedySampler s(rep_penalty, rep_lookback);
    std::vector<float> lv(logits, logits + V);
    std::vector<int32_t> hv(hist, hist + (H > 0 ? H : 0));
    const int id = s.sample(lv, hv, {});
    if (logits_out) std::memcpy(logits_out, lv.data(), sizeof(float) * (size_t)V);
    return id;
}

// ---- vocabulary / trie / grammar handles -----------------------------------
void* qwref_vocab_new(const char* const* strs, const int32_t* lens, int V) {
    Vocab* v = new Vocab();
    v->strs.reserve((size_t)V);
    for (int i = 0; i < V; ++i) v->strs.emplace_back(strs[i], (size_t)lens[i]);
    return v;
}
void qwref_vocab_free(void* v) { delete static_cast<Vocab*>(v); }

void* qwref_trie_new(void* vocab) {
    qwenium::TokenTrie* t = new qwenium::TokenTrie();
    t->build(static_cast<Vocab*>(vocab)->strs);
    return t;
}
void qwref_trie_free(void* t) { delete static_cast<qwenium::TokenTrie*>(t); }

void* qwref_grammar_parse(const char* gbnf) {
    auto g = qwenium::GrammarVocab::parse_impl(std::string(gbnf));
    return g.release();
}
void qwref_grammar_free(void* g) { delete static_cast<qwenium::GrammarVocab*>(g); }
void qwref_grammar_set_trie(void* g, void* trie) {
    static_cast<qwenium::GrammarVocab*>(g)->set_token_trie(static_cast<qwenium::TokenTrie*>(trie));
}
// get_valid_tokens (grammar_vocab.cpp:571-755): ascending ids; returns the
// full count even when it exceeds cap (only the first cap are written).
int qwref_grammar_valid(void* g, void* vocab, int32_t* out, int cap) {
    std::vector<int32_t> ids =
        static_cast<qwenium::GrammarVocab*>(g)->get_valid_tokens(static_cast<Vocab*>(vocab)->strs);
    const int n = (int)ids.size();
    for (int i = 0; i < n && i < cap; ++i) out[i] = ids[i];
    return n;
}
void qwref_grammar_accept(void* g, int32_t id, void* vocab) {
    static_cast<qwenium::GrammarVocab*>(g)->accept_token(id, static_cast<Vocab*>(vocab)->strs);
}
int qwref_grammar_accepting(void* g) {
    return static_cast<qwenium::GrammarVocab*>(g)->is_accepting_state() ? 1 : 0;
}
void qwref_grammar_reset(void* g) { static_cast<qwenium::GrammarVocab*>(g)->reset(); }

// SpeculativeDecoder::try_speculative_step (speculative.h:150-239) with a
// given draft: the prompt ends with three sentinel ids followed by the draft
// and the generated tokens end with the same three ids, so the n-gram lookup
// (prompt_lookup.h:33-80, n = 3, max_draft = K) proposes exactly the draft;
// the verify callback returns the K given logits rows.
void qwref_spec_verify(const float* logits, int K, int V, const int32_t* draft, int eos, int32_t* accepted,
                       int32_t* bonus, int32_t* has_bonus) {
    const int32_t s0 = -1000001, s1 = -1000002, s2 = -1000003;
    std::vector<int32_t> prompt = {s0, s1, s2};
    prompt.insert(prompt.end(), draft, draft + K);
    const std::vector<int32_t> generated = {s0, s1, s2};
    qwenium::PromptLookupConfig cfg;
    cfg.ngram_size = 3;
    cfg.max_draft = K;
    cfg.min_draft = 1;
    qwenium::SpeculativeDecoder dec(cfg, V);
    auto verify = [&](int, const std::vector<int32_t>&, int) {
        return std::vector<float>(logits, logits + (size_t)K * (size_t)V);
    };
    auto rewind = [](int, int) {};
    const qwenium::SpeculativeResult r = dec.try_speculative_step(prompt, generated, 0, 0, verify, rewind, eos);
    *accepted = (int32_t)r.accepted_tokens.size();
    *bonus = r.bonus_token;
    *has_bonus = r.has_bonus ? 1 : 0;
}

// TokenTrie::mark_char_class (token-trie.cpp:93-116) into a fresh mask:
// out[i] = 1 when the reference marks token i.
void qwref_trie_mark_char_class(void* trie, const unsigned char* chars, int n, int negated, int V,
                                unsigned char* out) {
    std::set<char> cs;
    for (int i = 0; i < n; ++i) cs.insert(static_cast<char>(chars[i]));
    std::vector<bool> mask(static_cast<size_t>(V), false);
    static_cast<qwenium::TokenTrie*>(trie)->mark_char_class(cs, negated != 0, mask);
    for (int i = 0; i < V; ++i) out[i] = mask[static_cast<size_t>(i)] ? 1 : 0;
}

// TokenTrie::collect_by_prefix / collect_by_char_class / collect_by_first_char
// (token-trie.cpp:39-91): the ids in the reference's order; at most cap are
// written, the full count is returned.
static int emit_ids(const std::vector<int32_t>& v, int32_t* out, int cap) {
    for (size_t i = 0; i < v.size() && (int)i < cap; ++i) out[i] = v[i];
    return (int)v.size();
}
int qwref_trie_collect_by_prefix(void* trie, const char* prefix, int len, int offset, int32_t* out, int cap) {
    std::vector<int32_t> v;
    static_cast<qwenium::TokenTrie*>(trie)->collect_by_prefix(std::string(prefix, (size_t)len), (size_t)offset, v);
    return emit_ids(v, out, cap);
}
int qwref_trie_collect_by_char_class(void* trie, const unsigned char* chars, int n, int negated, int32_t* out,
                                     int cap) {
    std::set<char> cs;
    for (int i = 0; i < n; ++i) cs.insert(static_cast<char>(chars[i]));
    std::vector<int32_t> v;
    static_cast<qwenium::TokenTrie*>(trie)->collect_by_char_class(cs, negated != 0, v);
    return emit_ids(v, out, cap);
}
int qwref_trie_collect_by_first_char(void* trie, unsigned char c, int32_t* out, int cap) {
    std::vector<int32_t> v;
    static_cast<qwenium::TokenTrie*>(trie)->collect_by_first_char(static_cast<char>(c), v);
    return emit_ids(v, out, cap);
}
long long qwref_trie_token_count(void* trie) {
    return (long long)static_cast<qwenium::TokenTrie*>(trie)->token_count();
}

// The full Sampler::sample path with a grammar, an EOS id and/or a pruning
// keep-set attached (sampling.cpp:12-81): exercises apply_vocab_pruning,
// apply_grammar_constraints (EOS allowance, stuck-grammar EOS forcing) and
// the lazily built trie. kind 0 = GreedySampler, 1 = TemperatureSampler.
// grammar may be NULL; keep_ids with n_keep < 0 means "no pruning".
int qwref_sampler_sample_full(int kind, float temperature, float rep_penalty, int rep_lookback,
                              int top_k, float top_p, void* grammar, void* vocab, int32_t eos_id,
                              const int32_t* keep_ids, int n_keep, const float* logits, int V,
                              const int32_t* hist, int H, uint32_t seed, double* u_out,
                              float* logits_out) {
    std::unordered_set<int32_t> keep;
    if (n_keep >= 0) keep.insert(keep_ids, keep_ids + n_keep);
    std::vector<float> lv(logits, logits + V);
    std::vector<int32_t> hv(hist, hist + (H > 0 ? H : 0));
    const std::vector<std::string> empty;
    const std::vector<std::string>& strs = vocab ? static_cast<Vocab*>(vocab)->strs : empty;
    int id;
    if (kind == 0) {
        qwenium::GreedySampler s(rep_penalty, rep_lookback);
        if (grammar) s.set_grammar(static_cast<qwenium::GrammarVocab*>(grammar));
        if (n_keep >= 0) s.set_pruned_vocab(&keep);
        if (eos_id >= 0) s.set_eos_token_id(eos_id);
        id = s.sample(lv, hv, strs);
        if (u_out) *u_out = 0.0;
    } else {
        qwenium::TemperatureSampler s(temperature, rep_penalty, rep_lookback, top_k, top_p);
        if (grammar) s.set_grammar(static_cast<qwenium::GrammarVocab*>(grammar));
        if (n_keep >= 0) s.set_pruned_vocab(&keep);
        if (eos_id >= 0) s.set_eos_token_id(eos_id);
        std::mt19937& gen = engine_of(s);
        gen = std::mt19937(seed);
        std::mt19937 probe = gen;
        if (u_out) *u_out = std::generate_canonical<double, 53>(probe);
        id = s.sample(lv, hv, strs);
    }
    if (logits_out) std::memcpy(logits_out, lv.data(), sizeof(float) * (size_t)V);
    return id;
}

// Many rows through TemperatureSampler::sample, split over n_threads
// std::threads with one sampler per row (rows spread over all host cores).
// Used to time the reference on the host cores.
int qwref_temperature_sample_batch(const float* logits, int B, int V, int64_t row_stride,
                                   const float* temperature, const int32_t* top_k,
                                   const float* top_p, const float* rep_penalty,
                                   const int32_t* rep_lookback, const int32_t* hist,
                                   int hist_stride, const int32_t* hist_len,
                                   const uint32_t* seeds, int32_t* out, int n_threads) {
    if (n_threads < 1) n_threads = 1;
    std::vector<std::thread> pool;
    std::atomic<int> next{0};
    for (int t = 0; t < n_threads; ++t) {
        pool.emplace_back([&]() {
            for (int b = next.fetch_add(1); b < B; b = next.fetch_add(1)) {
                out[b] = qwref_temperature_sample(
                    logits + (size_t)b * (size_t)row_stride, V, hist + (size_t)b * (size_t)hist_stride,
                    hist_len[b], temperature[b], rep_penalty[b], rep_lookback[b], top_k[b], top_p[b],
                    seeds[b], nullptr, nullptr, nullptr);
            }
        });
    }
    for (auto& th : pool) th.join();
    return 0;
}

// std::generate_canonical<double,53>(std::mt19937(seed)) -- the u the
// reference's engine yields first for a given seed.
double qwref_first_uniform(uint32_t seed) {
    std::mt19937 g(seed);
    return std::generate_canonical<double, 53>(g);
}

}  // extern "C"
