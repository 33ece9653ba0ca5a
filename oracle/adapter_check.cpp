// adapter_check.cpp -- TEST INFRASTRUCTURE ONLY (the checker, never the product).
//
// Drives the reference's own samplers (src/sampling, compiled unmodified) and
// the drop-in adapters of qwenium_b200/adapter (CudaTemperatureSampler,
// CudaGreedySampler, GPU through libqsamp.so) side by side on the same
// inputs, with both engines seeded alike, and checks after every call that
//   * the returned ids are equal,
//   * the logits vectors left behind are bit-identical (the reference mutates
//     them in place: pruning, grammar mask, penalty, /T),
//   * the two std::mt19937 engines are in the same state (a draw consumed u
//     in both or in neither).
// Cases: full-vocabulary top-p, top-k + top-p with a growing history,
// greedy, a pruning keep-set, a JSON grammar walk (GBNF text from argv[1]),
// and empty logits (both throw). Prints one line per case; exit 0 iff all
// agree. Built by oracle/Makefile into oracle/_ref/adapter_check.
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <random>
#include <sstream>
#include <stdexcept>
#include <string>
#include <unordered_set>
#include <vector>

#include "../qwenium_b200/adapter/cuda_sampler.h"
#include "grammar_vocab.h"
#include "ref_access.h"
#include "sampling.h"

namespace {

int g_fail = 0;

bool same_bits(const std::vector<float>& a, const std::vector<float>& b) {
    return a.size() == b.size() && std::memcmp(a.data(), b.data(), a.size() * sizeof(float)) == 0;
}

std::vector<float> make_logits(uint32_t seed, int V, float sigma) {
    std::mt19937 g(seed);
    std::normal_distribution<float> n(0.0f, sigma);
    std::vector<float> x((size_t)V);
    for (float& v : x) v = n(g);
    return x;
}

bool engines_equal(qwenium::TemperatureSampler& r, qwenium_b200::CudaTemperatureSampler& c) {
    return qwref_access::engine_of(r) == c.engine();
}
bool engines_equal(qwenium::GreedySampler&, qwenium_b200::CudaGreedySampler&) { return true; }

template <typename RefS, typename CudaS>
void run_steps(const char* name, RefS& ref, CudaS& cuda, int V, int steps, uint32_t seed,
               const std::vector<std::string>& vocab, qwenium::GrammarVocab* gref, qwenium::GrammarVocab* gcuda) {
    std::vector<int32_t> hist;
    int bad = 0;
    for (int t = 0; t < steps; ++t) {
        std::vector<float> a = make_logits(seed + (uint32_t)t, V, 3.0f);
        std::vector<float> b = a;
        const int ia = ref.sample(a, hist, vocab);
        const int ib = cuda.sample(b, hist, vocab);
        const bool ok_id = ia == ib;
        const bool ok_lo = same_bits(a, b);
        const bool ok_eng = engines_equal(ref, cuda);
        if (!ok_id || !ok_lo || !ok_eng) {
            if (bad < 3)
                std::printf("  %s step %d: ref %d cuda %d, logits %s, engines %s\n", name, t, ia, ib,
                            ok_lo ? "same" : "DIFFER", ok_eng ? "same" : "DIFFER");
            ++bad;
        }
        hist.push_back(ia);
        if (gref) gref->accept_token(ia, vocab);
        if (gcuda) gcuda->accept_token(ia, vocab);
    }
    std::printf("%-28s %d steps, %d mismatches\n", name, steps, bad);
    g_fail += bad;
}

std::string read_file(const char* path) {
    std::ifstream f(path);
    std::stringstream ss;
    ss << f.rdbuf();
    return ss.str();
}

// A small vocabulary for the grammar walk: the 256 single bytes, JSON-ish
// multi-byte tokens, random printable strings and the two EOS strings.
std::vector<std::string> grammar_vocab(int V) {
    std::vector<std::string> v;
    for (int i = 0; i < 256; ++i) v.emplace_back(1, (char)i);
    const char* pieces[] = {"{\"", "\":", "\": ", "\"}", "\",", ", \"", "true", "false", "null", "[1", "2]", "{}",
                            "[]", "\"a", "bc\"", "12", ".5", "-3", " {", "}\n", "\"key\"", "\"v\"", "  "};
    for (const char* p : pieces) v.emplace_back(p);
    std::mt19937 g(99);
    std::uniform_int_distribution<int> len(2, 8), ch(0x20, 0x7e);
    while ((int)v.size() < V - 2) {
        std::string s;
        const int n = len(g);
        for (int i = 0; i < n; ++i) s.push_back((char)ch(g));
        v.push_back(s);
    }
    v.emplace_back("<|endoftext|>");
    v.emplace_back("<|im_end|>");
    return v;
}

// --time N: per-call latency of the drop-in samplers and of the reference's,
// one row per call as Sampler::sample is called (C1: V=151936 logits ~N(0,3^2)
// plus 20 ids boosted by +8, a 64-id history, repetition penalty 1.1 over 64;
// T 0.8, top-k 40, top-p 0.95, and GreedySampler's defaults). Prints one
// JSON object of mean milliseconds per call.
template <typename S>
double time_calls(S& s, const std::vector<std::vector<float>>& rows, const std::vector<int32_t>& hist, int n) {
    const std::vector<std::string> none;
    volatile int sink = 0;
    auto t0 = std::chrono::steady_clock::now();
    for (int i = 0; i < n; ++i) {
        std::vector<float> x = rows[(size_t)i % rows.size()];
        sink = sink + s.sample(x, hist, none);
    }
    const double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    return ms / n;
}

int time_mode(int n) {
    const int V = 151936;
    std::vector<std::vector<float>> rows;
    for (uint32_t r = 0; r < 4; ++r) {
        std::vector<float> x = make_logits(700 + r, V, 3.0f);
        std::mt19937 g(800 + r);
        std::uniform_int_distribution<int> id(0, V - 1);
        for (int j = 0; j < 20; ++j) x[(size_t)id(g)] += 8.0f;
        rows.push_back(std::move(x));
    }
    std::vector<int32_t> hist;
    std::mt19937 g(900);
    std::uniform_int_distribution<int> id(0, V - 1);
    for (int j = 0; j < 64; ++j) hist.push_back(id(g));
    qwenium_b200::CudaTemperatureSampler ct(0.8f, 1.1f, 64, 40, 0.95f);
    qwenium_b200::CudaGreedySampler cg;
    qwenium::TemperatureSampler rt(0.8f, 1.1f, 64, 40, 0.95f);
    qwenium::GreedySampler rg;
    time_calls(ct, rows, hist, 3);  // context creation and first-call set-up
    time_calls(cg, rows, hist, 3);
    const double a = time_calls(ct, rows, hist, n), b = time_calls(cg, rows, hist, n);
    const double c = time_calls(rt, rows, hist, n < 20 ? n : 20), d = time_calls(rg, rows, hist, n);
    std::printf("{\"calls\": %d, \"cuda_temperature_ms\": %.4f, \"cuda_greedy_ms\": %.4f, "
                "\"reference_temperature_ms\": %.4f, \"reference_greedy_ms\": %.4f}\n", n, a, b, c, d);
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    const int V = 151936;
    const std::vector<std::string> none;
    if (argc > 2 && std::strcmp(argv[1], "--time") == 0) return time_mode(std::atoi(argv[2]));
    try {
        {  // full vocabulary, top-p only
            qwenium::TemperatureSampler ref(1.0f, 1.1f, 64, 0, 0.9f);
            qwenium_b200::CudaTemperatureSampler cuda(1.0f, 1.1f, 64, 0, 0.9f);
            qwref_access::engine_of(ref).seed(11);
            cuda.seed(11);
            run_steps("full vocab top-p 0.9", ref, cuda, V, 8, 100, none, nullptr, nullptr);
        }
        {  // top-k + top-p, the reference's defaults
            qwenium::TemperatureSampler ref;
            qwenium_b200::CudaTemperatureSampler cuda;
            qwref_access::engine_of(ref).seed(12);
            cuda.seed(12);
            run_steps("defaults (T .7 k 40 p .95)", ref, cuda, V, 24, 200, none, nullptr, nullptr);
        }
        {  // greedy
            qwenium::GreedySampler ref;
            qwenium_b200::CudaGreedySampler cuda;
            run_steps("greedy (rep 1.2 / 32)", ref, cuda, V, 16, 300, none, nullptr, nullptr);
        }
        {  // pruning keep-set
            std::unordered_set<int32_t> keep;
            std::mt19937 g(5);
            std::uniform_int_distribution<int> id(0, V - 1);
            while ((int)keep.size() < 5000) keep.insert(id(g));
            qwenium::TemperatureSampler ref(0.9f, 1.1f, 64, 50, 0.9f);
            qwenium_b200::CudaTemperatureSampler cuda(0.9f, 1.1f, 64, 50, 0.9f);
            ref.set_pruned_vocab(&keep);
            cuda.set_pruned_vocab(&keep);
            qwref_access::engine_of(ref).seed(13);
            cuda.seed(13);
            run_steps("pruned vocab (5000 ids)", ref, cuda, V, 12, 400, none, nullptr, nullptr);
        }
        if (argc > 1) {  // grammar walk
            const std::string gbnf = read_file(argv[1]);
            const int GV = 20000;
            const std::vector<std::string> vocab = grammar_vocab(GV);
            auto gr = qwenium::GrammarVocab::parse_impl(gbnf);
            auto gc = qwenium::GrammarVocab::parse_impl(gbnf);
            if (!gr || !gc) throw std::runtime_error("GBNF parse failed");
            qwenium::TemperatureSampler ref(0.8f, 1.0f, 64, 0, 0.95f);
            qwenium_b200::CudaTemperatureSampler cuda(0.8f, 1.0f, 64, 0, 0.95f);
            ref.set_grammar(gr.get());
            cuda.set_grammar(gc.get());
            ref.set_eos_token_id(GV - 1);
            cuda.set_eos_token_id(GV - 1);
            qwref_access::engine_of(ref).seed(14);
            cuda.seed(14);
            run_steps("JSON grammar walk", ref, cuda, GV, 30, 500, vocab, gr.get(), gc.get());
        }
        {  // empty logits: both throw
            qwenium::TemperatureSampler ref;
            qwenium_b200::CudaTemperatureSampler cuda;
            std::vector<float> e;
            int thrown = 0;
            try { ref.sample(e, {}, none); } catch (const std::runtime_error&) { ++thrown; }
            try { cuda.sample(e, {}, none); } catch (const std::runtime_error&) { ++thrown; }
            std::printf("%-28s %s\n", "empty logits", thrown == 2 ? "both throw" : "MISMATCH");
            if (thrown != 2) ++g_fail;
        }
    } catch (const std::exception& ex) {
        std::printf("error: %s\n", ex.what());
        return 2;
    }
    std::printf("%s\n", g_fail ? "FAIL" : "ALL AGREE");
    return g_fail ? 1 : 0;
}
