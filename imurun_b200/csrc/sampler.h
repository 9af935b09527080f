// sampler.h — host token sampler with the reference's semantics
// (model/fish/src/sampler.cpp:42-175): repetition penalty over the recent
// window, then greedy (temperature <= 0: first index of the maximum) or
// temperature, top-k, softmax over the kept set, nucleus cut, draw with a
// mt19937_64 stream.
#pragma once

#include <cstdint>
#include <random>
#include <vector>

namespace fb {

struct SampleParams {
    float temperature = 0.7f;
    int top_k = 40;
    float top_p = 0.9f;
    float repeat_penalty = 1.1f;
    int repeat_last_n = 64;
};

class Sampler {
public:
    explicit Sampler(uint64_t seed = 0) { reseed(seed); }
    void reseed(uint64_t seed);
    // logits are modified in place (penalty, temperature)
    int32_t sample(float* logits, int n_vocab, const SampleParams& p, const std::vector<int32_t>& recent);
    // the penalty step alone (used before an on-device greedy argmax)
    static void penalise(float* logits, int n_vocab, const SampleParams& p, const std::vector<int32_t>& recent);
    // The distribution sample() draws from, as probabilities over the whole
    // vocabulary (speculative decoding compares the target's and the
    // draft's): penalty, then a one-hot of the first maximum (temperature
    // <= 0) or temperature, top-k, softmax and the nucleus cut renormalised
    // (reference sampler.cpp:42-89). logits are modified in place.
    void distribution(float* logits, int n_vocab, const SampleParams& p, const std::vector<int32_t>& recent,
                      std::vector<float>& probs);
    // An index drawn in proportion to the positive weights (-1 when none).
    int32_t draw(const float* w, int n);
    // A uniform draw in [0, 1) from the same stream.
    double uniform();
    // Speculative verification of one draft token d drawn from q against the
    // target's distribution p (reference c_api.cpp:719-741): d is kept with
    // probability min(1, p(d)/q(d)); otherwise the replacement is drawn from
    // max(0, p - q), or from p when that is all zero. Returns -1 when d is
    // kept, else the replacement; the result is distributed as p. The accept
    // test draws from this sampler's seeded stream.
    int32_t verify_draft(const std::vector<float>& p, const std::vector<float>& q, int32_t d,
                         std::vector<float>& residual);

private:
    std::mt19937_64 rng_;
    struct Cand { float v; int32_t id; };
    std::vector<Cand> buf_;
};

}  // namespace fb
