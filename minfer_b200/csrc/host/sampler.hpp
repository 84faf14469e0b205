// Host-side token sampler of the token loop. Same algorithm and the same
// libstdc++ primitives as the reference's Sampler (src/base/sampler.cpp:10-117),
// so identical logits give identical ids:
//   temp == 0  -> first maximum (std::max_element);
//   otherwise  -> presence penalty, nth_element + sort for the top-k,
//                 softmax over the top-k, top-p cut, min-p cut, temperature
//                 softmax, one std::uniform_real_distribution<float> draw from
//                 std::mt19937_64(seed).
#pragma once

#include <cstddef>
#include <cstdint>
#include <random>
#include <unordered_set>
#include <vector>

namespace minfer {

struct SamplerParams {
    size_t vocab_size = 0;
    size_t top_k = 1;
    float temp = 0.0f;
    float top_p = 1.0f;
    float min_p = 0.0f;
    float penalty_pres = 0.0f;
    int seed = 0;
};

class Sampler {
public:
    explicit Sampler(const SamplerParams& p);
    void add_token(uint32_t token);
    uint32_t sample(const float* logits);
    // The same draw from the top-k candidates alone: ids[i], logits[i] sorted by
    // logit, largest first (ties: lower id first), k == top_k. Valid when the
    // presence penalty is 0 (the candidates are then exactly the list sample()
    // builds); consumes one random number like sample().
    uint32_t sample_candidates(const uint32_t* ids, const float* logits, size_t k);
    // Whether a candidate list decides the draw on its own. `vals` holds the
    // top_k + 1 largest logits, largest first. sample() orders equal logits
    // the way nth_element + sort leaves them, which a list built with another
    // tie rule need not reproduce; so any two equal values among them (inside
    // the top-k, or the k-th equal to the next one, which makes the top-k set
    // itself ambiguous) mean the whole-vocabulary sample() must decide.
    static bool candidates_decisive(const float* vals, size_t n);
    // the next n draws of the random stream, without consuming them
    std::vector<float> peek_draws(size_t n) const;
    // consume n draws (as n sample() calls would)
    void skip_draws(size_t n);
    bool greedy() const { return p_.temp == 0.0f; }
    size_t top_k() const { return p_.top_k; }
    float penalty_pres() const { return p_.penalty_pres; }

private:
    // top-p / min-p cuts, temperature softmax and the draw over a sorted candidate list
    uint32_t pick(const uint32_t* ids, const float* lg, size_t k);

    SamplerParams p_;
    std::vector<float> logits_, probs_, pick_probs_;
    std::vector<uint32_t> idx_;
    std::unordered_set<uint32_t> seen_;
    std::mt19937_64 rng_;
    std::uniform_real_distribution<float> dist_;
};

}  // namespace minfer
