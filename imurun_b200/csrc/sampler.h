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

private:
    std::mt19937_64 rng_;
    struct Cand { float v; int32_t id; };
    std::vector<Cand> buf_;
};

}  // namespace fb
