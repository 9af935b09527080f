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

void Sampler::distribution(float* logits, int n_vocab, const SampleParams& p, const std::vector<int32_t>& recent,
                           std::vector<float>& probs) {
    probs.assign((size_t)std::max(0, n_vocab), 0.0f);
    if (!logits || n_vocab <= 0) return;
    penalise(logits, n_vocab, p, recent);
    if (p.temperature <= 0.0f) {
        int32_t best = 0;
        float bv = -std::numeric_limits<float>::infinity();
        for (int i = 0; i < n_vocab; ++i) if (logits[i] > bv) { bv = logits[i]; best = i; }
        probs[best] = 1.0f;
        return;
    }
    const float inv_t = 1.0f / p.temperature;
    const int k = p.top_k > 0 ? std::min(p.top_k, n_vocab) : n_vocab;
    if ((int)buf_.size() < n_vocab) buf_.resize(n_vocab);
    for (int i = 0; i < n_vocab; ++i) buf_[i] = {logits[i] * inv_t, i};
    std::partial_sort(buf_.begin(), buf_.begin() + k, buf_.begin() + n_vocab,
                      [](const Cand& a, const Cand& b) { return a.v > b.v; });
    const float mx = buf_[0].v;
    double sum = 0.0;
    for (int i = 0; i < k; ++i) { const float e = std::exp(buf_[i].v - mx); buf_[i].v = e; sum += e; }
    if (sum <= 0.0) { probs[buf_[0].id] = 1.0f; return; }
    double cum = 0.0;
    int keep = k;
    for (int i = 0; i < k; ++i) {
        cum += buf_[i].v / sum;
        if (cum >= p.top_p) { keep = i + 1; break; }
    }
    double norm = 0.0;
    for (int i = 0; i < keep; ++i) norm += buf_[i].v;
    for (int i = 0; i < keep; ++i) probs[buf_[i].id] = (float)(buf_[i].v / norm);
}

int32_t Sampler::draw(const float* w, int n) {
    double total = 0.0;
    for (int i = 0; i < n; ++i) if (w[i] > 0.0f) total += w[i];
    if (!(total > 0.0)) return -1;
    std::uniform_real_distribution<double> dist(0.0, total);
    const double r = dist(rng_);
    double acc = 0.0;
    int32_t last = -1;
    for (int i = 0; i < n; ++i) {
        if (w[i] <= 0.0f) continue;
        acc += w[i];
        last = i;
        if (r <= acc) return i;
    }
    return last;
}

double Sampler::uniform() {
    std::uniform_real_distribution<double> dist(0.0, 1.0);
    return dist(rng_);
}

int32_t Sampler::verify_draft(const std::vector<float>& p, const std::vector<float>& q, int32_t d,
                              std::vector<float>& residual) {
    const float pd = p[(size_t)d], qd = q[(size_t)d];
    bool accept = pd >= qd;
    if (!accept && qd > 0.0f && pd > 0.0f) accept = uniform() < (double)(pd / qd);
    if (accept) return -1;
    residual.resize(p.size());
    float total = 0.0f;
    for (size_t i = 0; i < p.size(); ++i) {
        const float r = p[i] - q[i];
        residual[i] = r > 0.0f ? r : 0.0f;
        total += residual[i];
    }
    return total > 0.0f ? draw(residual.data(), (int)p.size()) : draw(p.data(), (int)p.size());
}

}  // namespace fb
