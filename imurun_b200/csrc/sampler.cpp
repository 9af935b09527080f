// sampler.cpp — see sampler.h.
#include "sampler.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <limits>

namespace fb {

void Sampler::reseed(uint64_t seed) {
    if (seed == 0) seed = (uint64_t)std::chrono::high_resolution_clock::now().time_since_epoch().count();
    rng_.seed(seed);
}

void Sampler::penalise(float* logits, int n_vocab, const SampleParams& p, const std::vector<int32_t>& recent) {
    if (!(p.repeat_penalty > 0.0f) || p.repeat_penalty == 1.0f || recent.empty()) return;
    const int window = p.repeat_last_n > 0 ? p.repeat_last_n : 64;
    const int start = std::max(0, (int)recent.size() - window);
    for (int i = start; i < (int)recent.size(); ++i) {
        const int32_t id = recent[i];
        if (id < 0 || id >= n_vocab) continue;
        float& v = logits[id];
        v = v > 0.0f ? v / p.repeat_penalty : v * p.repeat_penalty;
    }
}

int32_t Sampler::sample(float* logits, int n_vocab, const SampleParams& p, const std::vector<int32_t>& recent) {
    if (!logits || n_vocab <= 0) return 0;
    penalise(logits, n_vocab, p, recent);
    if (p.temperature <= 0.0f) {
        int32_t best = 0;
        float bv = -std::numeric_limits<float>::infinity();
        for (int i = 0; i < n_vocab; ++i) if (logits[i] > bv) { bv = logits[i]; best = i; }
        return best;
    }
    const float inv_t = 1.0f / p.temperature;
    for (int i = 0; i < n_vocab; ++i) logits[i] *= inv_t;
    const int k = p.top_k > 0 ? std::min(p.top_k, n_vocab) : n_vocab;
    if ((int)buf_.size() < n_vocab) buf_.resize(n_vocab);
    for (int i = 0; i < n_vocab; ++i) buf_[i] = {logits[i], i};
    std::partial_sort(buf_.begin(), buf_.begin() + k, buf_.begin() + n_vocab,
                      [](const Cand& a, const Cand& b) { return a.v > b.v; });
    const float mx = buf_[0].v;
    double sum = 0.0;
    for (int i = 0; i < k; ++i) { const float e = std::exp(buf_[i].v - mx); buf_[i].v = e; sum += e; }
    if (sum <= 0.0) return buf_[0].id;
    double cum = 0.0;
    int keep = k;
    for (int i = 0; i < k; ++i) {
        cum += buf_[i].v / sum;
        if (cum >= p.top_p) { keep = i + 1; break; }
    }
    double norm = 0.0;
    for (int i = 0; i < keep; ++i) norm += buf_[i].v;
    if (norm <= 0.0) return buf_[0].id;
    std::uniform_real_distribution<double> dist(0.0, norm);
    const double r = dist(rng_);
    double acc = 0.0;
    for (int i = 0; i < keep; ++i) {
        acc += buf_[i].v;
        if (r <= acc) return buf_[i].id;
    }
    return buf_[keep - 1].id;
}

}  // namespace fb
