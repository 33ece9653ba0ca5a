// cuda_sampler.h -- drop-in qwenium::Sampler implementations over libqsamp.
//
// CudaTemperatureSampler / CudaGreedySampler derive from the reference's
// qwenium::Sampler (src/sampling/sampling.h:15-51) and keep its contract:
//   * sample(logits, last_tokens, token_strs) returns the token id and
//     throws std::runtime_error on empty logits (sampling.cpp:101,140);
//   * set_grammar / set_pruned_vocab / set_eos_token_id / build_token_trie
//     are the base class's own (non-owning grammar and keep-set, owned trie);
//   * the selection runs on the GPU (qsamp_sample_host: prune and grammar
//     allow-mask, stuck-grammar EOS forcing, repetition penalty, /T, sort,
//     top-k, top-p, softmax, draw), bit-identical to the reference evaluated
//     in source order;
//   * the sampler's own std::mt19937 is advanced exactly when the reference's
//     std::discrete_distribution would draw (two or more survivors);
//   * on return, `logits` holds what the reference leaves in it: pruned and
//     grammar-masked ids at -inf (the stuck-grammar rule applied), the
//     repetition penalty applied, divided by T when T > 0.
// Like the reference, an instance is not thread-safe. Each instance owns a
// qsamp context on `device`, created on the first sample() call.
#pragma once

#include <cstdint>
#include <random>
#include <string>
#include <vector>

#include "qsamp.h"
#include "sampling.h"

namespace qwenium_b200 {

class CudaSamplerBase : public qwenium::Sampler {
public:
    ~CudaSamplerBase() override;

protected:
    CudaSamplerBase(int device, float temperature, float repetition_penalty, int repetition_lookback, int top_k,
                    float top_p);
    // One row through qsamp_sample_host; u < 0: no draw (greedy).
    int select(std::vector<float>& logits, const std::vector<int32_t>& last_tokens,
               const std::vector<std::string>& token_strs, std::mt19937* gen);

private:
    void ensure_ctx();
    int32_t eos_string_id(const std::vector<std::string>& token_strs);
    void apply_host_side_effects(std::vector<float>& logits, const std::vector<int32_t>& last_tokens,
                                 int32_t force) const;

    int device_;
    float temperature_, repetition_penalty_, top_p_;
    int repetition_lookback_, top_k_;
    qsamp_ctx* ctx_ = nullptr;
    std::vector<uint32_t> mask_, gmask_;
    const std::string* eos_cache_vocab_ = nullptr;
    size_t eos_cache_size_ = 0;
    int32_t eos_cache_id_ = -1;
};

// qwenium::TemperatureSampler on the GPU (defaults of sampling.h:73-77).
class CudaTemperatureSampler : public CudaSamplerBase {
public:
    explicit CudaTemperatureSampler(float temperature = 0.7f, float repetition_penalty = 1.1f,
                                    int repetition_lookback = 64, int top_k = 40, float top_p = 0.95f,
                                    int device = 0);
    int sample(std::vector<float>& logits, const std::vector<int32_t>& last_tokens,
               const std::vector<std::string>& token_strs) override;
    // The engine is seeded from std::random_device like the reference's
    // (sampling.cpp:120-121); this reseeds it (tests, reproducible runs).
    void seed(uint32_t s) { gen_.seed(s); }
    const std::mt19937& engine() const { return gen_; }

private:
    std::mt19937 gen_;
};

// qwenium::GreedySampler on the GPU (defaults of sampling.h:55-56).
class CudaGreedySampler : public CudaSamplerBase {
public:
    explicit CudaGreedySampler(float repetition_penalty = 1.2f, int repetition_lookback = 32, int device = 0);
    int sample(std::vector<float>& logits, const std::vector<int32_t>& last_tokens,
               const std::vector<std::string>& token_strs = {}) override;
};

}  // namespace qwenium_b200
