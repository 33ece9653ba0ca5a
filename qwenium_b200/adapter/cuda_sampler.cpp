// cuda_sampler.cpp -- see cuda_sampler.h.
#include "cuda_sampler.h"

#include <cstring>
#include <iostream>
#include <limits>
#include <stdexcept>
#include <unordered_set>

namespace qwenium_b200 {

namespace {
void check(qsamp_ctx* ctx, qsamp_status s, const char* what) {
    if (s == QSAMP_OK) return;
    throw std::runtime_error(std::string(what) + ": " + (ctx ? qsamp_last_error(ctx) : "qsamp error"));
}
}  // namespace

CudaSamplerBase::CudaSamplerBase(int device, float temperature, float repetition_penalty, int repetition_lookback,
                                 int top_k, float top_p)
    : device_(device),
      temperature_(temperature),
      repetition_penalty_(repetition_penalty),
      top_p_(top_p),
      repetition_lookback_(repetition_lookback),
      top_k_(top_k) {}

CudaSamplerBase::~CudaSamplerBase() { qsamp_destroy(ctx_); }

void CudaSamplerBase::ensure_ctx() {
    if (ctx_) return;
    const qsamp_status s = qsamp_create(device_, &ctx_);
    if (s != QSAMP_OK) {
        ctx_ = nullptr;
        throw std::runtime_error("qsamp_create failed on device " + std::to_string(device_) + " (status " +
                                 std::to_string((int)s) + ")");
    }
}

// The first "<|endoftext|>" / "<|im_end|>" entry (sampling.cpp:53-58,67-71),
// cached per vocabulary.
int32_t CudaSamplerBase::eos_string_id(const std::vector<std::string>& token_strs) {
    if (eos_cache_vocab_ == token_strs.data() && eos_cache_size_ == token_strs.size()) return eos_cache_id_;
    int32_t id = -1;
    for (size_t i = 0; i < token_strs.size(); ++i)
        if (token_strs[i] == "<|endoftext|>" || token_strs[i] == "<|im_end|>") {
            id = (int32_t)i;
            break;
        }
    eos_cache_vocab_ = token_strs.data();
    eos_cache_size_ = token_strs.size();
    eos_cache_id_ = id;
    return id;
}

int CudaSamplerBase::select(std::vector<float>& logits, const std::vector<int32_t>& last_tokens,
                            const std::vector<std::string>& token_strs, std::mt19937* gen) {
    if (logits.empty()) throw std::runtime_error("Cannot sample from empty logits");
    ensure_ctx();
    const int32_t V = (int32_t)logits.size();
    const int64_t words = (V + 31) / 32;

    // allow-mask: the pruning keep-set (sampling.cpp:12-18), then the grammar
    // (sampling.cpp:25-81); a stuck grammar forces the EOS string.
    bool masked = false;
    int32_t force = -1;
    if (pruned_vocab_) {
        std::vector<int32_t> keep(pruned_vocab_->begin(), pruned_vocab_->end());
        mask_.assign((size_t)words, 0u);
        check(ctx_, qsamp_pack_ids(keep.data(), (int64_t)keep.size(), V, mask_.data()), "qsamp_pack_ids");
        masked = true;
    }
    if (grammar_ && !token_strs.empty()) {
        if (!token_trie_) build_token_trie(token_strs);
        grammar_->set_token_trie(token_trie_.get());
        const std::vector<int32_t> valid = grammar_->get_valid_tokens(token_strs);
        gmask_.assign((size_t)words, 0u);
        check(ctx_,
              qsamp_grammar_mask(valid.data(), (int64_t)valid.size(), grammar_->is_accepting_state() ? 1 : 0,
                                 eos_string_id(token_strs), eos_token_id_, V, gmask_.data(), &force),
              "qsamp_grammar_mask");
        if (force >= 0) {
            std::cerr << "[GrammarVocab] ERROR: Grammar is stuck! No valid tokens found in vocabulary.\n"
                      << "  Action: Forcing EOS to prevent crash.\n";
        } else if (masked) {
            check(ctx_, qsamp_mask_and(mask_.data(), gmask_.data(), words, mask_.data()), "qsamp_mask_and");
        } else {
            mask_.swap(gmask_);
            masked = true;
        }
    }

    qsamp_row_params p = {};
    p.temperature = temperature_;
    p.top_k = top_k_;
    p.top_p = top_p_;
    p.repetition_penalty = repetition_penalty_;
    p.repetition_lookback = repetition_lookback_;
    p.force_token = force;
    // The reference's engine: generate_canonical<double,53> on a copy, kept
    // only if the discrete distribution drew (two or more weights).
    std::mt19937 probe;
    double u = 0.0;
    if (gen) {
        probe = *gen;
        u = std::generate_canonical<double, 53>(probe);
    }
    const int32_t hl = (int32_t)last_tokens.size();
    qsamp_batch b = {};
    b.logits = logits.data();
    b.dtype = QSAMP_F32;
    b.B = 1;
    b.V = V;
    b.row_stride = V;
    b.params = &p;
    b.hist = hl > 0 ? last_tokens.data() : nullptr;
    b.hist_stride = hl > 0 ? hl : 1;
    b.hist_len = hl > 0 ? &hl : nullptr;
    b.masks = (masked && force < 0) ? mask_.data() : nullptr;
    b.mask_stride = 0;
    b.u = gen ? &u : nullptr;
    int32_t id = -1;
    qsamp_row_result res = {};
    b.out_ids = &id;
    b.out_results = &res;
    check(ctx_, qsamp_sample_host(ctx_, &b), "qsamp_sample_host");
    if (gen && res.drew) *gen = probe;
    apply_host_side_effects(logits, last_tokens, force);
    return id;
}

// What the reference leaves in `logits` (sampling.cpp:12-18, 25-81, 85-96 /
// 124-135, 154-156): masked ids at -inf, the penalty, then /T.
void CudaSamplerBase::apply_host_side_effects(std::vector<float>& logits, const std::vector<int32_t>& last_tokens,
                                              int32_t force) const {
    const float ninf = -std::numeric_limits<float>::infinity();
    const size_t V = logits.size();
    if (force >= 0) {
        for (size_t i = 0; i < V; ++i) logits[i] = ninf;
        logits[(size_t)force] = 0.0f;
    } else if (!mask_.empty() && (pruned_vocab_ || (grammar_ != nullptr))) {
        for (size_t i = 0; i < V; ++i)
            if (!((mask_[i >> 5] >> (i & 31)) & 1u)) logits[i] = ninf;
    }
    if (repetition_penalty_ != 1.0f && !last_tokens.empty()) {
        const size_t lookback = std::min((size_t)repetition_lookback_, last_tokens.size());
        const std::unordered_set<int32_t> recent(last_tokens.end() - lookback, last_tokens.end());
        for (int32_t id : recent)
            if (id >= 0 && (size_t)id < V)
                logits[id] = logits[id] < 0 ? logits[id] * repetition_penalty_ : logits[id] / repetition_penalty_;
    }
    if (temperature_ > 0.0f)
        for (size_t i = 0; i < V; ++i) logits[i] /= temperature_;
}

CudaTemperatureSampler::CudaTemperatureSampler(float temperature, float repetition_penalty, int repetition_lookback,
                                               int top_k, float top_p, int device)
    : CudaSamplerBase(device, temperature, repetition_penalty, repetition_lookback, top_k, top_p) {
    std::random_device rd;
    gen_ = std::mt19937(rd());
}

int CudaTemperatureSampler::sample(std::vector<float>& logits, const std::vector<int32_t>& last_tokens,
                                   const std::vector<std::string>& token_strs) {
    return select(logits, last_tokens, token_strs, &gen_);
}

CudaGreedySampler::CudaGreedySampler(float repetition_penalty, int repetition_lookback, int device)
    : CudaSamplerBase(device, 0.0f, repetition_penalty, repetition_lookback, 0, 1.0f) {}

int CudaGreedySampler::sample(std::vector<float>& logits, const std::vector<int32_t>& last_tokens,
                              const std::vector<std::string>& token_strs) {
    return select(logits, last_tokens, token_strs, nullptr);
}

}  // namespace qwenium_b200
