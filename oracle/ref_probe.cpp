/*
 * ref_probe.cpp — a thin C entry-point layer over the REFERENCE FISH engine.
 *
 * TEST INFRASTRUCTURE ONLY. This file is compiled together with the unmodified
 * reference sources (read from the reference checkout by oracle/Makefile) into
 * oracle/_ref/libfish_ref.so. It exposes the reference's internal C++ API
 * (include/fish/quant.h, model.h) as plain C functions so the tests can pin the
 * oracle restatement, generate golden vectors, and time the reference CPU path
 * as the CPU baseline. It contains no arithmetic of its own.
 */
#include <fish/model.h>
#include <fish/quant.h>
#include <fish/ops.h>
#include <fish/threadpool.h>
#include <fish/sampler.h>
#include <fish/gguf.h>
#include <cstdio>

#include <cstring>
#include <memory>
#include <string>
#include <vector>

using namespace fish;

extern "C" {

__attribute__((visibility("default"))) const char* ref_kernel_name(void) { return quant_kernels().name; }

__attribute__((visibility("default"))) void ref_quantize_acts(const float* x, uint64_t n, void* out) {
    quantize_acts(x, n, static_cast<Q8Act*>(out));
}
__attribute__((visibility("default"))) void ref_quantize_acts_k(const float* x, uint64_t n, void* out) {
    quantize_acts_k(x, n, static_cast<Q8ActK*>(out));
}
/* scalar table (quant.cpp:436-456), to pin the AVX2 table the build installs. */
__attribute__((visibility("default"))) void ref_quantize_acts_scalar(const float* x, uint64_t n, void* out) {
    scalar_kernels().quantize(x, n, static_cast<Q8Act*>(out));
}
__attribute__((visibility("default"))) void ref_quantize_acts_k_scalar(const float* x, uint64_t n, void* out) {
    scalar_kernels().quantize_k(x, n, static_cast<Q8ActK*>(out));
}
__attribute__((visibility("default"))) int ref_vec_dot_q8(int type, const void* row, const void* x, uint64_t n, float* out) {
    return vec_dot_q8(static_cast<GgmlType>(type), row, static_cast<const Q8Act*>(x), n, out) ? 1 : 0;
}
__attribute__((visibility("default"))) int ref_vec_dot_q8k(int type, const void* row, const void* x, uint64_t n, float* out) {
    return vec_dot_q8k(static_cast<GgmlType>(type), row, static_cast<const Q8ActK*>(x), n, out) ? 1 : 0;
}
__attribute__((visibility("default"))) int ref_dequant_row(int type, const void* src, float* dst, uint64_t n) {
    return dequant_row(static_cast<GgmlType>(type), src, dst, n) ? 1 : 0;
}
__attribute__((visibility("default"))) int ref_quantize_row(int type, const float* x, void* dst, uint64_t n) {
    return quantize_row(static_cast<GgmlType>(type), x, dst, n) ? 1 : 0;
}
__attribute__((visibility("default"))) void ref_rmsnorm(float* out, const float* x, const float* w, int n, float eps) {
    rmsnorm(out, x, w, n, eps);
}
__attribute__((visibility("default"))) void ref_act(float* x, int n, int gelu) {
    if (gelu) gelu_inplace(x, n);
    else silu_inplace(x, n);
}
__attribute__((visibility("default"))) void ref_attention(const float* q, const float* k, const float* v, int n_ctx,
                                                          int n_head, int n_head_kv, int head_dim, int pos0, int n_tok,
                                                          float* out, float scale) {
    attention_batch(q, k, v, n_ctx, n_head, n_head_kv, head_dim, pos0, n_tok, out, scale, 0.0f, 0);
}
/* The same with gemma2's score soft cap and sliding window. */
__attribute__((visibility("default"))) void ref_attention_capped(const float* q, const float* k, const float* v,
                                                                 int n_ctx, int n_head, int n_head_kv, int head_dim,
                                                                 int pos0, int n_tok, float* out, float scale,
                                                                 float softcap, int window) {
    attention_batch(q, k, v, n_ctx, n_head, n_head_kv, head_dim, pos0, n_tok, out, scale, softcap, window);
}
__attribute__((visibility("default"))) void ref_rope_table(int n_ctx, int head_dim, int rot_dim, int neox,
                                                           float freq_base, float* cos_out, float* sin_out) {
    RopeParams p;
    p.head_dim = head_dim;
    p.rot_dim = rot_dim;
    p.freq_base = freq_base;
    p.neox = neox != 0;
    RopeCache c;
    rope_build(c, n_ctx, p);
    std::memcpy(cos_out, c.cos_.data(), c.cos_.size() * sizeof(float));
    std::memcpy(sin_out, c.sin_.data(), c.sin_.size() * sizeof(float));
}
__attribute__((visibility("default"))) void ref_set_threads(int n) { ThreadPool::instance().set_active_threads(n); }
__attribute__((visibility("default"))) int ref_threads(void) { return ThreadPool::instance().active_threads(); }

struct RefModel { std::unique_ptr<LlamaModel> m; std::string err; };

__attribute__((visibility("default"))) void* ref_model_load(const char* path, int n_ctx, char* err, int cap) {
    auto* h = new RefModel();
    LlamaModel::LoadOptions o;
    o.gpu_layers = 0;
    o.allow_span = false;
    h->m = LlamaModel::load(path, n_ctx, o, &h->err);
    if (!h->m) {
        if (err && cap > 0) std::snprintf(err, static_cast<size_t>(cap), "%s", h->err.c_str());
        delete h;
        return nullptr;
    }
    return h;
}
__attribute__((visibility("default"))) void ref_model_free(void* h) { delete static_cast<RefModel*>(h); }
__attribute__((visibility("default"))) int ref_model_vocab(void* h) { return static_cast<RefModel*>(h)->m->config().vocab; }
__attribute__((visibility("default"))) int ref_model_n_ctx(void* h) { return static_cast<RefModel*>(h)->m->config().n_ctx; }
__attribute__((visibility("default"))) int ref_model_max_batch(void* h) { return static_cast<RefModel*>(h)->m->max_batch(); }
/* LlamaModel::forward (model.cpp:1603-1811); logits of the last token copied out,
 * and with logits_all non-null every token's (all_logits=true). */
__attribute__((visibility("default"))) int ref_model_forward(void* h, const int32_t* tokens, int n, int pos0,
                                                             float* logits, float* logits_all) {
    LlamaModel& m = *static_cast<RefModel*>(h)->m;
    if (!m.forward(tokens, n, pos0, logits_all != nullptr)) return 0;
    const int V = m.config().vocab;
    if (logits) std::memcpy(logits, m.logits(), sizeof(float) * static_cast<size_t>(V));
    if (logits_all) std::memcpy(logits_all, m.logits_at(0), sizeof(float) * static_cast<size_t>(V) * n);
    return 1;
}
__attribute__((visibility("default"))) int ref_model_argmax(void* h) { return static_cast<RefModel*>(h)->m->argmax(); }
__attribute__((visibility("default"))) void ref_model_set_kv_len(void* h, int n) { static_cast<RefModel*>(h)->m->set_kv_len(n); }
__attribute__((visibility("default"))) void ref_model_reset(void* h) { static_cast<RefModel*>(h)->m->reset_kv(); }
__attribute__((visibility("default"))) unsigned long long ref_model_weights_bytes(void* h) {
    return static_cast<RefModel*>(h)->m->weights_bytes();
}
/* Sampler::sample (include/fish/sampler.h:26-33) n_draws times with one
 * Sampler seeded with `seed`, each draw on a fresh copy of the logits (the
 * call modifies them in place); the ids go to out. */
__attribute__((visibility("default"))) void ref_sample(const float* logits, int n_vocab, float temperature, int top_k,
                                                       float top_p, float repeat_penalty, int repeat_last_n,
                                                       const int32_t* recent, int n_recent, unsigned long long seed,
                                                       int n_draws, int32_t* out) {
    SampleParams p;
    p.temperature = temperature;
    p.top_k = top_k;
    p.top_p = top_p;
    p.repeat_penalty = repeat_penalty;
    p.repeat_last_n = repeat_last_n;
    p.seed = seed;
    Sampler s(seed);
    std::vector<int32_t> rec(recent, recent + n_recent);
    std::vector<float> work(static_cast<size_t>(n_vocab));
    for (int i = 0; i < n_draws; ++i) {
        std::memcpy(work.data(), logits, sizeof(float) * static_cast<size_t>(n_vocab));
        out[i] = s.sample(work.data(), n_vocab, p, rec);
    }
}
/* The reference's Sampler::distribution and Sampler::draw behind the same
 * arguments as the library's fbx_sample_distribution / fbx_sample_draw. */
__attribute__((visibility("default"))) void ref_distribution(const float* logits, int n_vocab, float temperature,
                                                             int top_k, float top_p, float repeat_penalty,
                                                             int repeat_last_n, const int32_t* recent, int n_recent,
                                                             float* probs) {
    SampleParams p;
    p.temperature = temperature;
    p.top_k = top_k;
    p.top_p = top_p;
    p.repeat_penalty = repeat_penalty;
    p.repeat_last_n = repeat_last_n;
    Sampler s(1);
    std::vector<int32_t> rec(recent, recent + n_recent);
    std::vector<float> work(logits, logits + n_vocab), out;
    s.distribution(work.data(), n_vocab, p, rec, out);
    std::memcpy(probs, out.data(), sizeof(float) * static_cast<size_t>(n_vocab));
}
__attribute__((visibility("default"))) void ref_draw(const float* weights, int n, unsigned long long seed,
                                                     int n_draws, int32_t* out) {
    Sampler s(seed);
    for (int i = 0; i < n_draws; ++i) out[i] = s.draw(weights, n);
}
/* The same digest as the library's fbx_gguf_digest, from the reference's own
 * GgufFile reader (include/fish/gguf.h:77-116): tensor directory and the
 * requested metadata keys, arrays reduced to counts and an FNV-1a digest. */
static unsigned long long ref_fnv1a(unsigned long long h, const void* p, size_t n) {
    const unsigned char* b = static_cast<const unsigned char*>(p);
    for (size_t i = 0; i < n; ++i) h = (h ^ b[i]) * 1099511628211ull;
    return h;
}
__attribute__((visibility("default"))) int ref_gguf_digest(const char* path, const char* const* keys, int n_keys,
                                                           char* out, int cap) {
    std::string err;
    auto g = GgufFile::open(path, &err);
    if (!g) return -1;
    std::string d;
    char line[256];
    for (const TensorInfo& t : g->tensors()) {
        d += "T " + t.name + " " + std::to_string(static_cast<unsigned>(t.type)) + " ";
        for (size_t i = 0; i < t.ne.size(); ++i) d += (i ? "," : "") + std::to_string(t.ne[i]);
        const unsigned long long off = static_cast<unsigned long long>(t.data - g->data_base()) + g->data_offset();
        std::snprintf(line, sizeof(line), " %llu %llu\n", off, static_cast<unsigned long long>(t.nbytes));
        d += line;
    }
    for (int k = 0; k < n_keys; ++k) {
        const MetaValue* m = g->meta(keys[k]);
        d += std::string("K ") + keys[k] + " ";
        if (!m) { d += "missing\n"; continue; }
        d += std::to_string(static_cast<int>(m->kind)) + " ";
        switch (m->kind) {
            case MetaValue::UINT: d += std::to_string(m->u); break;
            case MetaValue::INT: d += std::to_string(m->i); break;
            case MetaValue::FLOAT: std::snprintf(line, sizeof(line), "%.17g", m->f); d += line; break;
            case MetaValue::BOOL: d += m->b ? "1" : "0"; break;
            case MetaValue::STRING: d += m->s; break;
            default: {
                unsigned long long h = 1469598103934665603ull;
                for (const std::string& s : m->sarr) h = ref_fnv1a(h, s.c_str(), s.size() + 1);
                h = ref_fnv1a(h, m->iarr.data(), m->iarr.size() * sizeof(int32_t));
                h = ref_fnv1a(h, m->farr.data(), m->farr.size() * sizeof(float));
                const size_t n = m->sarr.size() + m->iarr.size() + m->farr.size() + m->arr.size();
                std::snprintf(line, sizeof(line), "n=%zu s=%zu i=%zu f=%zu h=%016llx", n, m->sarr.size(),
                              m->iarr.size(), m->farr.size(), h);
                d += line;
            }
        }
        d += "\n";
    }
    const int need = static_cast<int>(d.size());
    if (out && cap > 0) {
        const int n = need < cap - 1 ? need : cap - 1;
        std::memcpy(out, d.data(), static_cast<size_t>(n));
        out[n] = '\0';
    }
    return need;
}

}  // extern "C"
