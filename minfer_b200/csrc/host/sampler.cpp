#include "sampler.hpp"

#include <algorithm>
#include <cmath>
#include <numeric>
#include <stdexcept>

namespace minfer {

Sampler::Sampler(const SamplerParams& p)
    : p_(p), logits_(p.vocab_size), probs_(p.vocab_size), idx_(p.vocab_size), rng_(p.seed), dist_(0.0f, 1.0f) {
    // parameter ranges checked by the reference's constructor (src/base/sampler.cpp:24-27)
    if (p.top_k == 0 || p.top_k > p.vocab_size) throw std::invalid_argument("top_k must be in [1, vocab_size]");
    if (!(p.top_p >= 0.0f && p.top_p <= 1.0f)) throw std::invalid_argument("top_p must be in [0, 1]");
    if (!(p.min_p >= 0.0f && p.min_p <= 1.0f)) throw std::invalid_argument("min_p must be in [0, 1]");
    if (!(p.penalty_pres >= 0.0f && p.penalty_pres <= 2.0f)) throw std::invalid_argument("penalty_pres must be in [0, 2]");
}

void Sampler::add_token(uint32_t token) { seen_.insert(token); }

std::vector<float> Sampler::peek_draws(size_t n) const {
    std::mt19937_64 rng = rng_;
    std::uniform_real_distribution<float> dist = dist_;
    std::vector<float> out(n);
    for (float& r : out) r = dist(rng);
    return out;
}

void Sampler::skip_draws(size_t n) {
    for (size_t i = 0; i < n; ++i) (void)dist_(rng_);
}

uint32_t Sampler::sample(const float* logits) {
    const size_t V = p_.vocab_size;
    if (p_.temp == 0.0f) return (uint32_t)(std::max_element(logits, logits + V) - logits);

    for (size_t i = 0; i < V; ++i) logits_[i] = logits[i] - float(seen_.count((uint32_t)i)) * p_.penalty_pres;
    std::iota(idx_.begin(), idx_.end(), 0u);
    auto by_logit = [&](size_t a, size_t b) { return logits_[a] > logits_[b]; };
    std::nth_element(idx_.begin(), idx_.begin() + p_.top_k, idx_.end(), by_logit);
    std::sort(idx_.begin(), idx_.begin() + p_.top_k, by_logit);
    for (size_t i = 0; i < p_.top_k; ++i) probs_[i] = logits_[idx_[i]];  // candidate logits, in order
    return pick(idx_.data(), probs_.data(), p_.top_k);
}

uint32_t Sampler::sample_candidates(const uint32_t* ids, const float* logits, size_t k) {
    if (k != p_.top_k || p_.penalty_pres != 0.0f) throw std::invalid_argument("candidate list does not match top_k");
    if (p_.temp == 0.0f) return ids[0];
    return pick(ids, logits, k);
}

bool Sampler::candidates_decisive(const float* vals, size_t n) {
    for (size_t i = 0; i + 1 < n; ++i)
        if (!(vals[i] != vals[i + 1])) return false;  // equal (or NaN): order undefined
    return true;
}

// src/base/sampler.cpp:52-117 from the sorted top-k list: softmax over the
// top-k, top-p cut, min-p cut, temperature softmax over the kept prefix, draw.
uint32_t Sampler::pick(const uint32_t* ids, const float* lg, size_t k) {
    std::vector<float>& pr = pick_probs_;
    pr.resize(k);
    size_t cut = k;
    const float top = lg[0];
    float acc = 0.0f;
    for (size_t i = 0; i < cut; ++i) {
        pr[i] = std::exp(lg[i] - top);
        acc += pr[i];
    }
    for (size_t i = 0; i < cut; ++i) pr[i] /= acc;

    acc = 0.0f;
    for (size_t i = 0; i < cut; ++i) {
        acc += pr[i];
        if (acc >= p_.top_p) {
            cut = i + 1;
            break;
        }
    }
    if (p_.min_p > 0.0f) {
        const float thr = top + std::log(p_.min_p);
        for (size_t i = 0; i < cut; ++i) {
            if (lg[i] < thr) {
                cut = i;
                break;
            }
        }
    }
    if (cut == 0) throw std::runtime_error("sampling filters removed every token");

    acc = 0.0f;
    for (size_t i = 0; i < cut; ++i) {
        pr[i] = std::exp((lg[i] - top) / p_.temp);
        acc += pr[i];
    }
    for (size_t i = 0; i < cut; ++i) pr[i] /= acc;

    const float r = dist_(rng_);
    acc = 0.0f;
    for (size_t i = 0; i < cut; ++i) {
        acc += pr[i];
        if (acc >= r) return ids[i];
    }
    return ids[cut - 1];
}

}  // namespace minfer
