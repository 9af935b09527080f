// c_api.cpp — the FISH C ABI (include/fish/c_api.h) over the B200 engine.
//
// The ABI-4 entry points keep the reference's contracts
// (model/fish/src/c_api.cpp): one mutex per context, negative error codes
// plus fish_last_error, "required size" string results, and the generation
// loop of generate_ids_locked (c_api.cpp:504-794): head+tail prompt fit with
// a sticky cut, the one-slot KV prefix cache (longest common prefix >= 8,
// identical prompt -> n-1), prefill in chunks of <= 256, sampled decode with
// UTF-8-complete streaming callbacks, cancel between forwards, stats.
#include <fish/c_api.h>
#include <fish/fish_kernels.h>

#include <sys/resource.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "engine.h"
#include "prompt_fit.h"
#include "sampler.h"
#include "tokenizer.h"

struct fish_ctx {
    std::mutex mu;
    std::unique_ptr<fb::Engine> eng;
    std::unique_ptr<fb::Tokenizer> tok;
    fb::Sampler sampler{0};
    std::string err;
    std::atomic<bool> cancel{false};
    fish_stats stats{};
    std::vector<int32_t> cache_ids;
    fb::PromptCut cut;
    std::string adapter_path;
    float adapter_scale = 1.0f;
    std::string model_path;
    int n_ctx_req = 0;
    std::vector<float> logits;
    int tp_rank = 0, tp_world = 1;       // set by fish_tp_init for the next fish_load
    unsigned char tp_id[128] = {};
    // speculative decoding: the draft engine, the ids its sequence 0 holds,
    // the longest draft per round
    std::unique_ptr<fb::Engine> draft;
    std::vector<int32_t> draft_ids;
    int draft_k = 5;
    std::vector<int32_t> last_ids;       // the ids the last generation emitted
};

namespace {

double now_s() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

double peak_rss_mb() {
    struct rusage ru {};
    return getrusage(RUSAGE_SELF, &ru) == 0 ? (double)ru.ru_maxrss / 1024.0 : 0.0;
}

// Emit only complete UTF-8 sequences (c_api.cpp:81-101).
void emit_utf8(fish_token_cb cb, void* user, const std::string& bytes, int id, std::string& pending, std::string& sink) {
    pending += bytes;
    size_t i = 0, done = 0;
    while (i < pending.size()) {
        const unsigned char c = (unsigned char)pending[i];
        size_t len = 1;
        if ((c & 0xE0) == 0xC0) len = 2;
        else if ((c & 0xF0) == 0xE0) len = 3;
        else if ((c & 0xF8) == 0xF0) len = 4;
        if (i + len > pending.size()) break;
        i += len;
        done = i;
    }
    if (!done) return;
    const std::string ready = pending.substr(0, done);
    pending.erase(0, done);
    sink += ready;
    if (cb) cb(ready.c_str(), id, user);
}

// Send what is still pending when generation ends (c_api.cpp:774-779).
void flush_utf8(fish_token_cb cb, void* user, std::string& pending, std::string& sink) {
    if (pending.empty()) return;
    sink += pending;
    if (cb) cb(pending.c_str(), -1, user);
    pending.clear();
}

int write_string(const std::string& s, char* out, int cap) {
    const int need = (int)s.size();
    if (out && cap > 0) {
        const int n = std::min(need, cap - 1);
        std::memcpy(out, s.data(), (size_t)n);
        out[n] = '\0';
    }
    return need;
}

fb::Messages to_messages(const char* const* roles, const char* const* contents, int n) {
    fb::Messages m;
    for (int i = 0; i < n; ++i)
        m.emplace_back(roles && roles[i] ? roles[i] : "user", contents && contents[i] ? contents[i] : "");
    return m;
}

void fill_load_stats(fish_ctx* ctx, double t_load) {
    fb::Engine& e = *ctx->eng;
    fish_stats& s = ctx->stats;
    s = fish_stats{};
    s.load_seconds = t_load;
    s.weights_bytes = e.weights_bytes();
    s.kv_bytes = e.kv_bytes();
    s.context_size = e.cfg().n_ctx;
    s.n_threads = 1;
    s.gpu_layers = e.cfg().n_layers;
    s.gpu_bytes = e.device_weight_bytes() + e.kv_bytes();
    std::snprintf(s.gpu_name, sizeof(s.gpu_name), "%s (cuda sm_100a)", e.device_name().c_str());
    std::snprintf(s.gpu_mix, sizeof(s.gpu_mix), "all %d layers resident at file precision; paged %s KV, %d-position pages",
                  e.cfg().n_layers, std::getenv("FISH_KV_F32") ? "f32" : "fp16", e.page_size());
    std::snprintf(s.placement, sizeof(s.placement), "whole model on GPU %d", e.device());
    std::snprintf(s.load_profile, sizeof(s.load_profile), "total %.2f s (upload %.2f s)", t_load, e.load_seconds_upload);
    size_t fr = 0, tot = 0;
    cudaMemGetInfo(&fr, &tot);
    s.vram_total = tot;
    s.vram_free = fr;
}

int load_locked(fish_ctx* ctx, const char* path, int n_ctx) {
    const double t0 = now_s();
    if (!ctx->adapter_path.empty()) {
        ctx->err = "adapter: LoRA merging is not supported by the B200 engine";
        ctx->adapter_path.clear();
        ctx->adapter_scale = 1.0f;
        return -4;
    }
    ctx->draft.reset();          // a draft belongs to one target vocabulary
    ctx->draft_ids.clear();
    ctx->eng.reset();
    ctx->tok.reset();
    auto eng = std::make_unique<fb::Engine>();
    std::string err;
    if (ctx->tp_world > 1) {   // the group id is used once: a reload needs a new fish_tp_init
        const bool ok = eng->set_tp(ctx->tp_rank, ctx->tp_world, ctx->tp_id, &err);
        ctx->tp_world = 1;
        ctx->tp_rank = 0;
        if (!ok) { ctx->err = err; return -2; }
    }
    if (!eng->load(path, n_ctx > 0 ? n_ctx : 4096, &err)) { ctx->err = err; return -2; }
    auto tok = fb::Tokenizer::create(eng->gguf(), &err);
    if (!tok) { ctx->err = err; return -3; }
    ctx->eng = std::move(eng);
    ctx->tok = std::move(tok);
    ctx->model_path = path;
    ctx->n_ctx_req = n_ctx;
    ctx->cache_ids.clear();
    ctx->logits.assign((size_t)ctx->eng->cfg().vocab, 0.0f);
    fill_load_stats(ctx, now_s() - t0);
    ctx->err.clear();
    return 0;
}

// Forward ids[0..n) on the context's sequence in chunks of <= 256
// (LlamaModel::forward's batch limit); last logits into ctx->logits.
bool prefill_chunks(fish_ctx* ctx, const int32_t* ids, int n, bool stop_on_cancel, int* done) {
    fb::Engine& e = *ctx->eng;
    const int batch = std::min(fb::kMaxBatch, e.cfg().n_ctx);
    int pos = 0;
    while (pos < n) {
        const int m = std::min(batch, n - pos);
        std::string err;
        if (!e.forward(0, ids + pos, m, ctx->logits.data(), nullptr, nullptr, &err)) {
            ctx->err = err;
            if (done) *done = pos;
            return false;
        }
        pos += m;
        if (stop_on_cancel && ctx->cancel) break;
    }
    if (done) *done = pos;
    return true;
}

int generate_ids_locked(fish_ctx* ctx, std::vector<int32_t> ids, int max_tokens, float temperature, int top_k,
                        float top_p, float repeat_penalty, fish_token_cb cb, void* user, std::string* collected) {
    if (!ctx->eng || !ctx->tok) { ctx->err = "no model loaded"; return -1; }
    if (ids.empty()) { ctx->err = "empty prompt"; return -1; }
    fb::Engine& e = *ctx->eng;
    const fb::Config& c = e.cfg();
    if (max_tokens <= 0) max_tokens = c.n_ctx;
    ctx->stats.truncated = fb::fit_prompt(ids, c.n_ctx, max_tokens, ctx->cut) ? 1 : 0;
    ctx->cancel = false;
    const int prefix = fb::cached_prefix(ids, ctx->cache_ids);
    ctx->stats.cached_tokens = prefix;
    const double t0 = now_s();
    e.seq_truncate(0, prefix);
    ctx->cache_ids.resize((size_t)prefix);
    int done = 0;
    if (!prefill_chunks(ctx, ids.data() + prefix, (int)ids.size() - prefix, true, &done)) {
        ctx->err = "prefill failed: " + ctx->err;
        ctx->cache_ids.clear();
        e.seq_truncate(0, 0);
        return -1;
    }
    int pos = prefix + done;
    if (ctx->cancel) ctx->cache_ids.assign(ids.begin(), ids.begin() + pos);
    else ctx->cache_ids = ids;
    const double t1 = now_s();
    const int prefilled = pos - prefix;

    fb::SampleParams sp;
    sp.temperature = temperature;
    sp.top_k = top_k;
    sp.top_p = top_p;
    sp.repeat_penalty = repeat_penalty;
    std::string pending, sink;
    std::vector<int32_t> recent;
    const size_t recent_cap = 128;
    for (size_t i = ids.size() > recent_cap ? ids.size() - recent_cap : 0; i < ids.size(); ++i) recent.push_back(ids[i]);
    ctx->last_ids.clear();
    auto remember = [&](int32_t t) {
        ctx->last_ids.push_back(t);
        recent.push_back(t);
        if (recent.size() > recent_cap) recent.erase(recent.begin());
    };
    // the sampler's penalty window (repeat_last_n of the capped history)
    const int window = std::min<int>(sp.repeat_last_n > 0 ? sp.repeat_last_n : 64, (int)recent_cap);
    int generated = 0;
    int next = -1;
    if (!ctx->cancel) next = ctx->sampler.sample(ctx->logits.data(), c.vocab, sp, recent);

    // Speculative decoding (reference c_api.cpp:630-773). Each round the
    // draft proposes up to k tokens, the target verifies [next, drafts] in
    // one forward, and the drafts are accepted left to right by the rejection
    // rule (accept d with probability min(1, p(d)/q(d)); on a rejection the
    // replacement is drawn from max(0, p - q)), which leaves the target's
    // sampling distribution unchanged; both caches are cut back to what was
    // committed. k adapts: +1 after a fully accepted round, else accepted+1.
    // The verify forward is the batched decode step over consecutive
    // positions of one sequence, so each row's logits are the bits plain
    // decode gives at that position. Greedy (temperature <= 0) makes p and q
    // one-hot: a draft is accepted iff it is the target's penalised argmax,
    // the engines return argmaxes and no logits cross to the host, and the
    // ids equal plain greedy decoding's. The accept test draws from the
    // sampler's own seeded stream, so a seeded run is reproducible.
    fb::Engine* D = ctx->draft.get();
    const int k_max = ctx->draft_k;
    int k = std::max(1, std::min(k_max, 3));
    ctx->stats.draft_proposed = 0;
    ctx->stats.draft_accepted = 0;
    const bool greedy = sp.temperature <= 0.0f;
    std::vector<std::vector<float>> q(D ? (size_t)k_max : 0);
    std::vector<float> p, residual, dlogits, vlogits;
    std::vector<int32_t> drafts, verify, hist, vam;
    bool stopped = false;

    while (!stopped && next >= 0 && generated < max_tokens && pos < c.n_ctx) {
        if (ctx->cancel) break;
        if (ctx->tok->is_eog(next)) break;
        emit_utf8(cb, user, ctx->tok->token_text(next), next, pending, sink);
        remember(next);
        ++generated;
        std::string err;

        if (D && generated < max_tokens && pos + k_max + 2 <= c.n_ctx) {
            // 0. the draft's sequence holds its longest common prefix with
            //    the committed ids; forward the rest
            size_t common = 0;
            while (common < ctx->draft_ids.size() && common < (size_t)pos && ctx->draft_ids[common] == ctx->cache_ids[common])
                ++common;
            bool ok = D->seq_truncate(0, (int)common);
            ctx->draft_ids.resize(ok ? common : 0);
            while (ok && (int)ctx->draft_ids.size() < pos) {
                const int dp = (int)ctx->draft_ids.size();
                const int n = std::min(fb::kMaxBatch, pos - dp);
                // a few committed tokens (the usual catch-up after a
                // rejection) through the captured decode step, a prompt
                // through the prefill kernels
                ok = n <= 16 ? D->verify(0, ctx->cache_ids.data() + dp, n, nullptr, 0, 0, 1.0f, nullptr, nullptr, &err)
                             : D->forward(0, ctx->cache_ids.data() + dp, n, nullptr, nullptr, nullptr, &err);
                if (ok) ctx->draft_ids.insert(ctx->draft_ids.end(), ctx->cache_ids.begin() + dp, ctx->cache_ids.begin() + dp + n);
            }
            // 1. the draft proposes up to k tokens
            drafts.clear();
            std::vector<int32_t> recent_d = recent;
            int32_t cur = next;
            for (int j = 0; ok && j < k; ++j) {
                int32_t d = -1;
                if (greedy) {
                    const int nw = std::min<int>(window, (int)recent_d.size());
                    ok = D->decode_argmax(0, cur, recent_d.data() + recent_d.size() - nw, nw, sp.repeat_penalty, &d, &err);
                } else {
                    dlogits.resize((size_t)c.vocab);
                    ok = D->forward(0, &cur, 1, dlogits.data(), nullptr, nullptr, &err);
                    if (ok) {
                        ctx->sampler.distribution(dlogits.data(), c.vocab, sp, recent_d, q[(size_t)j]);
                        d = ctx->sampler.draw(q[(size_t)j].data(), c.vocab);
                    }
                }
                if (!ok) break;
                ctx->draft_ids.push_back(cur);
                if (d < 0) break;
                drafts.push_back(d);
                recent_d.push_back(d);
                if (recent_d.size() > recent_cap) recent_d.erase(recent_d.begin());
                cur = d;
                if (ctx->tok->is_eog(d)) break;   // nothing useful can follow
            }
            if (!ok) {   // the draft engine failed: plain decode from here on
                ctx->draft.reset();
                ctx->draft_ids.clear();
                D = nullptr;
                ctx->stats.draft_active = 0;
            }
            if (!drafts.empty()) {
                ctx->stats.draft_proposed += (int)drafts.size();
                const int n = (int)drafts.size();
                verify.assign(1, next);
                verify.insert(verify.end(), drafts.begin(), drafts.end());
                // 2. the target verifies [next, d_0 .. d_{n-1}] in one forward
                if (greedy) {
                    hist = recent;
                    hist.insert(hist.end(), drafts.begin(), drafts.end());
                    vam.resize((size_t)n + 1);
                    ok = e.verify(0, verify.data(), n + 1, hist.data(), (int)recent.size(), window, sp.repeat_penalty,
                                  vam.data(), nullptr, &err);
                } else {
                    vlogits.resize((size_t)(n + 1) * c.vocab);
                    ok = e.verify(0, verify.data(), n + 1, nullptr, 0, 0, 1.0f, nullptr, vlogits.data(), &err);
                }
                if (!ok) {
                    ctx->err = "decode failed: " + err;
                    ctx->cache_ids.clear();
                    break;
                }
                ctx->cache_ids.push_back(next);
                ++pos;
                // 3. accept / reject left to right
                int accepted = 0;
                int32_t replacement = -1;
                for (int j = 0; j < n; ++j) {
                    const int32_t d = drafts[(size_t)j];
                    if (greedy) {
                        if (vam[(size_t)j] != d) { replacement = vam[(size_t)j]; break; }
                    } else {
                        ctx->sampler.distribution(vlogits.data() + (size_t)j * c.vocab, c.vocab, sp, recent, p);
                        replacement = ctx->sampler.verify_draft(p, q[(size_t)j], d, residual);
                        if (replacement >= 0) break;
                    }
                    // accepted: d is committed at position pos
                    ++accepted;
                    ++ctx->stats.draft_accepted;
                    if (ctx->tok->is_eog(d)) { stopped = true; break; }
                    emit_utf8(cb, user, ctx->tok->token_text(d), d, pending, sink);
                    remember(d);
                    ++generated;
                    ctx->cache_ids.push_back(d);
                    ++pos;
                    if (generated >= max_tokens) { stopped = true; break; }
                }
                // 4. cut the target's cache back to the committed length
                e.seq_truncate(0, pos);
                k = accepted == n ? std::min(k_max, k + 1) : std::max(1, accepted + 1);
                if (stopped) break;
                if (replacement >= 0) {
                    next = replacement;
                } else if (greedy) {
                    next = vam[(size_t)n];   // the bonus token after the last accepted draft
                } else {
                    next = ctx->sampler.sample(vlogits.data() + (size_t)n * c.vocab, c.vocab, sp, recent);
                }
                continue;
            }
        }

        if (greedy) {
            // greedy: penalty and argmax on the device, only the id comes back
            // (the sampler's window: the last repeat_last_n ids of `recent`)
            const size_t start = recent.size() > (size_t)window ? recent.size() - window : 0;
            int32_t am = 0;
            if (!e.decode_argmax(0, next, recent.data() + start, (int)(recent.size() - start), sp.repeat_penalty, &am,
                                 &err)) {
                ctx->err = "decode failed: " + err;
                ctx->cache_ids.clear();
                break;
            }
            ctx->cache_ids.push_back(next);
            ++pos;
            next = am;
            continue;
        }
        if (!e.forward(0, &next, 1, ctx->logits.data(), nullptr, nullptr, &err)) {
            ctx->err = "decode failed: " + err;
            ctx->cache_ids.clear();
            break;
        }
        ctx->cache_ids.push_back(next);
        ++pos;
        next = ctx->sampler.sample(ctx->logits.data(), c.vocab, sp, recent);
    }
    flush_utf8(cb, user, pending, sink);
    const double t2 = now_s();
    ctx->stats.prefill_seconds = t1 - t0;
    ctx->stats.decode_seconds = t2 - t1;
    ctx->stats.prompt_tokens = (int)ids.size();
    ctx->stats.generated_tokens = generated;
    ctx->stats.context_used = pos;
    ctx->stats.tokens_per_second = ctx->stats.decode_seconds > 0 ? generated / ctx->stats.decode_seconds : 0.0;
    ctx->stats.prefill_tokens_per_second = ctx->stats.prefill_seconds > 0 ? prefilled / ctx->stats.prefill_seconds : 0.0;
    if (collected) *collected = sink;
    return generated;
}

bool need_model(fish_ctx* ctx) {
    if (!ctx->eng) { ctx->err = "no model loaded"; return false; }
    return true;
}

}  // namespace

extern "C" {

const char* fish_version(void) { return "fish-b200 0.1.0"; }
int fish_abi_version(void) { return FISH_ABI_VERSION; }
const char* fish_supported_archs(void) { return "llama,qwen2,qwen2moe,qwen3,qwen3moe,gemma2,phi3"; }
const char* fish_kernel_name(void) { return "cuda-sm100a"; }

fish_ctx* fish_create(void) { return new (std::nothrow) fish_ctx(); }

void fish_destroy(fish_ctx* ctx) {
    if (!ctx) return;
    ctx->cancel = true;
    {
        std::lock_guard<std::mutex> lock(ctx->mu);
        ctx->draft.reset();
        ctx->eng.reset();
        ctx->tok.reset();
    }
    delete ctx;
}

int fish_load(fish_ctx* ctx, const char* path, int n_ctx) {
    if (!ctx || !path) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    return load_locked(ctx, path, n_ctx);
}

int fish_loaded(fish_ctx* ctx) {
    if (!ctx) return 0;
    std::lock_guard<std::mutex> lock(ctx->mu);
    return (ctx->eng && ctx->tok) ? 1 : 0;
}

const char* fish_last_error(fish_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

int fish_model_info_of(fish_ctx* ctx, fish_model_info* out) {
    if (!ctx || !out) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (!ctx->eng || !ctx->tok) return -1;
    const fb::Config& c = ctx->eng->cfg();
    std::memset(out, 0, sizeof(*out));
    std::snprintf(out->arch, sizeof(out->arch), "%s", c.arch.c_str());
    out->n_layers = c.n_layers;
    out->n_embd = c.n_embd;
    out->n_ff = c.n_ff_model;   // the model's own shape, also under tensor parallelism
    out->n_head = c.n_head_model;
    out->n_head_kv = c.n_head_kv_model;
    out->head_dim = c.head_dim;
    out->n_ctx = c.n_ctx;
    out->vocab = c.vocab;
    out->tied_output = c.tied_output ? 1 : 0;
    out->n_experts = c.n_experts;
    out->n_experts_per_tok = c.n_experts_per_tok;
    out->n_ctx_train = c.n_ctx_train;
    std::snprintf(out->chat_format, sizeof(out->chat_format), "%s", fb::chat_format_name(ctx->tok->format()));
    std::snprintf(out->tokenizer, sizeof(out->tokenizer), "%s", ctx->tok->spm() ? "spm" : "bpe");
    std::vector<std::pair<const char*, int>> counts;
    for (const auto& t : ctx->eng->gguf().tensors()) {
        const char* n = fb::ggml_type_name(t.type);
        bool f = false;
        for (auto& kv : counts) if (std::strcmp(kv.first, n) == 0) { ++kv.second; f = true; break; }
        if (!f) counts.emplace_back(n, 1);
    }
    std::sort(counts.begin(), counts.end(), [](const auto& a, const auto& b) { return a.second > b.second; });
    std::string mix;
    for (size_t i = 0; i < counts.size() && i < 4; ++i) {
        if (!mix.empty()) mix += " ";
        mix += std::string(counts[i].first) + ":" + std::to_string(counts[i].second);
    }
    std::snprintf(out->quant, sizeof(out->quant), "%s", mix.c_str());
    return 0;
}

int fish_tokenize(fish_ctx* ctx, const char* text, int add_bos, int32_t* out, int cap) {
    if (!ctx || !text) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (!ctx->tok) return -1;
    const auto ids = ctx->tok->encode(text, add_bos != 0, true);
    if (!out || cap <= 0) return (int)ids.size();
    const int n = std::min((int)ids.size(), cap);
    std::memcpy(out, ids.data(), sizeof(int32_t) * (size_t)n);
    return n;
}

int fish_detokenize(fish_ctx* ctx, const int32_t* ids, int n, char* out, int cap) {
    if (!ctx || !ids || n < 0) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (!ctx->tok) return -1;
    return write_string(ctx->tok->decode(std::vector<int32_t>(ids, ids + n)), out, cap);
}

int fish_chat_prompt(fish_ctx* ctx, const char* const* roles, const char* const* contents, int n, char* out, int cap) {
    if (!ctx || n < 0) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (!ctx->tok) return -1;
    return write_string(ctx->tok->apply_chat(to_messages(roles, contents, n), ctx->tok->format()), out, cap);
}

int fish_count_chat_tokens(fish_ctx* ctx, const char* const* roles, const char* const* contents, int n) {
    if (!ctx || n < 0) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (!ctx->tok) return -1;
    return (int)ctx->tok->encode_chat(to_messages(roles, contents, n)).size();
}

const char* fish_chat_format(fish_ctx* ctx) {
    if (!ctx) return "none";
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (!ctx->tok) return "none";
    return fb::chat_format_name(ctx->tok->format());
}

// ------------------------------------------------ tokenizer without a model
// The tokenizer fish_load would build for the GGUF at `path`, from its
// metadata alone (no weights read, no device touched).
static std::unique_ptr<fb::Tokenizer> tokenizer_of(const char* path, std::unique_ptr<fb::Gguf>* g) {
    if (!path) return nullptr;
    std::string err;
    *g = fb::Gguf::open(path, &err);
    if (!*g) return nullptr;
    return fb::Tokenizer::create(**g, &err);
}

int fbx_tokenize_gguf(const char* gguf_path, const char* text, int add_bos, int32_t* out, int cap) {
    std::unique_ptr<fb::Gguf> g;
    auto tok = tokenizer_of(gguf_path, &g);
    if (!tok || !text) return -1;
    const auto ids = tok->encode(text, add_bos != 0, true);
    if (!out || cap <= 0) return (int)ids.size();
    const int n = std::min((int)ids.size(), cap);
    std::memcpy(out, ids.data(), sizeof(int32_t) * (size_t)n);
    return n;
}

int fbx_detokenize_gguf(const char* gguf_path, const int32_t* ids, int n, char* out, int cap) {
    std::unique_ptr<fb::Gguf> g;
    auto tok = tokenizer_of(gguf_path, &g);
    if (!tok || !ids || n < 0) return -1;
    return write_string(tok->decode(std::vector<int32_t>(ids, ids + n)), out, cap);
}

int fbx_chat_prompt_gguf(const char* gguf_path, const char* const* roles, const char* const* contents, int n,
                         char* out, int cap) {
    std::unique_ptr<fb::Gguf> g;
    auto tok = tokenizer_of(gguf_path, &g);
    if (!tok || n < 0) return -1;
    return write_string(tok->apply_chat(to_messages(roles, contents, n), tok->format()), out, cap);
}

int fbx_chat_info_gguf(const char* gguf_path, const char* const* roles, const char* const* contents, int n,
                       char* format, int cap) {
    std::unique_ptr<fb::Gguf> g;
    auto tok = tokenizer_of(gguf_path, &g);
    if (!tok || n < 0) return -1;
    write_string(fb::chat_format_name(tok->format()), format, cap);
    return (int)tok->encode_chat(to_messages(roles, contents, n)).size();
}

int fbx_stream_gguf(const char* gguf_path, const int32_t* ids, int n, char* out, int cap) {
    std::unique_ptr<fb::Gguf> g;
    auto tok = tokenizer_of(gguf_path, &g);
    if (!tok || n < 0 || (n > 0 && !ids)) return -1;
    std::string rec, pending, sink;
    const fish_token_cb cb = [](const char* text, int id, void* user) {
        *static_cast<std::string*>(user) += std::to_string(id) + " " + std::to_string(std::strlen(text)) + "\n" + text;
    };
    for (int i = 0; i < n; ++i) emit_utf8(cb, &rec, tok->token_text(ids[i]), ids[i], pending, sink);
    flush_utf8(cb, &rec, pending, sink);
    return write_string(rec, out, cap);
}

// FNV-1a over bytes, for the digest of metadata arrays
static uint64_t fnv1a(uint64_t h, const void* p, size_t n) {
    const uint8_t* b = static_cast<const uint8_t*>(p);
    for (size_t i = 0; i < n; ++i) h = (h ^ b[i]) * 1099511628211ull;
    return h;
}

struct fbx_prompt_state {
    fb::PromptCut cut;
    std::vector<int32_t> cache_ids;
};

fbx_prompt_state* fbx_prompt_state_create(void) { return new (std::nothrow) fbx_prompt_state(); }
void fbx_prompt_state_destroy(fbx_prompt_state* s) { delete s; }

int fbx_prompt_plan(fbx_prompt_state* s, const int32_t* ids, int n, int n_ctx, int max_tokens, int32_t* kept, int cap,
                    int* cached, int* truncated) {
    if (!s || !ids || n <= 0 || n_ctx <= 0 || !kept || !cached || !truncated) return -1;
    if (max_tokens <= 0) max_tokens = n_ctx;
    std::vector<int32_t> v(ids, ids + n);
    *truncated = fb::fit_prompt(v, n_ctx, max_tokens, s->cut) ? 1 : 0;
    *cached = fb::cached_prefix(v, s->cache_ids);
    if ((int)v.size() > cap) return -1;
    std::copy(v.begin(), v.end(), kept);
    return (int)v.size();
}

int fbx_prompt_commit(fbx_prompt_state* s, const int32_t* ids, int n) {
    if (!s || n < 0 || (n > 0 && !ids)) return -1;
    s->cache_ids.assign(ids, ids + n);
    return 0;
}

int fbx_gguf_digest(const char* gguf_path, const char* const* keys, int n_keys, char* out, int cap) {
    if (!gguf_path || n_keys < 0 || (n_keys > 0 && !keys)) return -1;
    std::string err;
    auto g = fb::Gguf::open(gguf_path, &err);
    if (!g) return -1;
    std::string d;
    char line[256];
    for (const fb::Tensor& t : g->tensors()) {
        d += "T " + t.name + " " + std::to_string(t.type) + " ";
        for (size_t i = 0; i < t.ne.size(); ++i) d += (i ? "," : "") + std::to_string(t.ne[i]);
        std::snprintf(line, sizeof(line), " %llu %llu\n", (unsigned long long)(t.data - g->map_base()),
                      (unsigned long long)t.nbytes);
        d += line;
    }
    for (int k = 0; k < n_keys; ++k) {
        const fb::MetaValue* m = keys[k] ? g->meta(keys[k]) : nullptr;
        d += std::string("K ") + (keys[k] ? keys[k] : "") + " ";
        if (!m) { d += "missing\n"; continue; }
        d += std::to_string((int)m->kind) + " ";
        switch (m->kind) {
            case fb::MetaValue::UINT: d += std::to_string(m->u); break;
            case fb::MetaValue::INT: d += std::to_string(m->i); break;
            case fb::MetaValue::FLOAT: std::snprintf(line, sizeof(line), "%.17g", m->f); d += line; break;
            case fb::MetaValue::BOOL: d += m->b ? "1" : "0"; break;
            case fb::MetaValue::STRING: d += m->s; break;
            default: {
                uint64_t h = 1469598103934665603ull;
                for (const std::string& s : m->sarr) h = fnv1a(h, s.c_str(), s.size() + 1);
                h = fnv1a(h, m->iarr.data(), m->iarr.size() * sizeof(int32_t));
                h = fnv1a(h, m->farr.data(), m->farr.size() * sizeof(float));
                std::snprintf(line, sizeof(line), "n=%llu s=%zu i=%zu f=%zu h=%016llx", (unsigned long long)m->count,
                              m->sarr.size(), m->iarr.size(), m->farr.size(), (unsigned long long)h);
                d += line;
            }
        }
        d += "\n";
    }
    return write_string(d, out, cap);
}

int fbx_sample(const float* logits, int n_vocab, float temperature, int top_k, float top_p, float repeat_penalty,
               int repeat_last_n, const int32_t* recent, int n_recent, uint64_t seed, int n_draws, int32_t* out) {
    if (!logits || n_vocab <= 0 || n_draws < 0 || (n_draws > 0 && !out) || n_recent < 0 || (n_recent > 0 && !recent))
        return -1;
    fb::SampleParams p;
    p.temperature = temperature;
    p.top_k = top_k;
    p.top_p = top_p;
    p.repeat_penalty = repeat_penalty;
    p.repeat_last_n = repeat_last_n;
    fb::Sampler s(seed);
    const std::vector<int32_t> rec(recent, recent + n_recent);
    std::vector<float> work((size_t)n_vocab);
    for (int i = 0; i < n_draws; ++i) {
        std::memcpy(work.data(), logits, sizeof(float) * (size_t)n_vocab);
        out[i] = s.sample(work.data(), n_vocab, p, rec);
    }
    return 0;
}

int fbx_sample_distribution(const float* logits, int n_vocab, float temperature, int top_k, float top_p,
                            float repeat_penalty, int repeat_last_n, const int32_t* recent, int n_recent, float* probs) {
    if (!logits || n_vocab <= 0 || !probs || n_recent < 0 || (n_recent > 0 && !recent)) return -1;
    fb::SampleParams p;
    p.temperature = temperature;
    p.top_k = top_k;
    p.top_p = top_p;
    p.repeat_penalty = repeat_penalty;
    p.repeat_last_n = repeat_last_n;
    fb::Sampler s(1);
    const std::vector<int32_t> rec(recent, recent + n_recent);
    std::vector<float> work(logits, logits + n_vocab), out;
    s.distribution(work.data(), n_vocab, p, rec, out);
    std::memcpy(probs, out.data(), sizeof(float) * (size_t)n_vocab);
    return 0;
}

int fbx_sample_draw(const float* weights, int n, uint64_t seed, int n_draws, int32_t* out) {
    if (!weights || n <= 0 || n_draws < 0 || (n_draws > 0 && !out)) return -1;
    fb::Sampler s(seed);
    for (int i = 0; i < n_draws; ++i) out[i] = s.draw(weights, n);
    return 0;
}

int fbx_last_generated(fish_ctx* ctx, int32_t* out, int cap) {
    if (!ctx || cap < 0 || (cap > 0 && !out)) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    const int n = (int)ctx->last_ids.size();
    std::copy(ctx->last_ids.begin(), ctx->last_ids.begin() + std::min(n, cap), out);
    return n;
}

int fbx_speculative_draws(const float* p, const float* q, int n, uint64_t seed, int n_trials, int32_t* out) {
    if (!p || !q || n <= 0 || n_trials < 0 || (n_trials > 0 && !out)) return -1;
    fb::Sampler s(seed);
    const std::vector<float> pv(p, p + n), qv(q, q + n);
    std::vector<float> residual;
    for (int i = 0; i < n_trials; ++i) {
        const int32_t d = s.draw(q, n);
        if (d < 0) { out[i] = -1; continue; }
        const int32_t r = s.verify_draft(pv, qv, d, residual);
        out[i] = r < 0 ? d : r;
    }
    return 0;
}

int fish_generate(fish_ctx* ctx, const char* prompt, int add_bos, int max_tokens, float temperature, int top_k,
                  float top_p, float repeat_penalty, fish_token_cb cb, void* user) {
    if (!ctx || !prompt) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (!ctx->tok) { ctx->err = "no model loaded"; return -1; }
    return generate_ids_locked(ctx, ctx->tok->encode(prompt, add_bos != 0, true), max_tokens, temperature, top_k,
                               top_p, repeat_penalty, cb, user, nullptr);
}

int fish_generate_chat(fish_ctx* ctx, const char* const* roles, const char* const* contents, int n, int max_tokens,
                       float temperature, int top_k, float top_p, float repeat_penalty, fish_token_cb cb, void* user) {
    if (!ctx || n <= 0) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (!ctx->tok) { ctx->err = "no model loaded"; return -1; }
    return generate_ids_locked(ctx, ctx->tok->encode_chat(to_messages(roles, contents, n)), max_tokens, temperature,
                               top_k, top_p, repeat_penalty, cb, user, nullptr);
}

int fish_generate_to(fish_ctx* ctx, const char* prompt, int add_bos, int max_tokens, float temperature, int top_k,
                     float top_p, float repeat_penalty, char* out, int cap) {
    if (!ctx || !prompt) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (!ctx->tok) { ctx->err = "no model loaded"; return -1; }
    std::string collected;
    const int n = generate_ids_locked(ctx, ctx->tok->encode(prompt, add_bos != 0, true), max_tokens, temperature,
                                      top_k, top_p, repeat_penalty, nullptr, nullptr, &collected);
    if (n < 0) return n;
    return write_string(collected, out, cap);
}

void fish_cancel(fish_ctx* ctx) { if (ctx) ctx->cancel = true; }

void fish_reset(fish_ctx* ctx) {
    if (!ctx) return;
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (ctx->eng) ctx->eng->seq_truncate(0, 0);
    if (ctx->draft) ctx->draft->seq_truncate(0, 0);
    ctx->cache_ids.clear();
    ctx->draft_ids.clear();
}

void fish_get_stats(fish_ctx* ctx, fish_stats* out) {
    if (!ctx || !out) return;
    std::lock_guard<std::mutex> lock(ctx->mu);
    *out = ctx->stats;
    out->peak_rss_mb = peak_rss_mb();
    if (ctx->eng) {
        out->context_used = ctx->eng->seq_len(0);
        size_t fr = 0, tot = 0;
        if (cudaMemGetInfo(&fr, &tot) == cudaSuccess) out->vram_free = fr;
    }
    out->n_threads = 1;
}

int fish_set_threads(fish_ctx* ctx, int n) {
    if (!ctx) return -1;
    (void)n;   // host threads do not take part in the device forward
    std::lock_guard<std::mutex> lock(ctx->mu);
    ctx->stats.n_threads = 1;
    return 0;
}

const char* fish_specs_json(fish_ctx* ctx) {
    thread_local std::string buf;
    int ndev = 0;
    cudaGetDeviceCount(&ndev);
    std::string gpus = "[";
    for (int i = 0; i < ndev; ++i) {
        cudaDeviceProp p{};
        cudaGetDeviceProperties(&p, i);
        char b[256];
        std::snprintf(b, sizeof(b), "%s{\"name\":\"%s\",\"memory_bytes\":%zu,\"sms\":%d,\"cc\":\"%d.%d\"}",
                      i ? "," : "", p.name, (size_t)p.totalGlobalMem, p.multiProcessorCount, p.major, p.minor);
        gpus += b;
    }
    gpus += "]";
    std::string plan = "null";
    if (ctx) {
        std::lock_guard<std::mutex> lock(ctx->mu);
        if (ctx->eng) {
            char b[256];
            std::snprintf(b, sizeof(b), "{\"n_ctx\":%d,\"gpu_layers\":%d,\"kv_bytes\":%llu}", ctx->eng->cfg().n_ctx,
                          ctx->eng->cfg().n_layers, (unsigned long long)ctx->eng->kv_bytes());
            plan = b;
        }
    }
    buf = "{\"hardware\":{\"gpus\":" + gpus + "},\"plan\":" + plan + ",\"threads\":1,\"pool_threads\":1,\"kernel\":\"" +
          std::string(fish_kernel_name()) + "\"}";
    return buf.c_str();
}

// The draft model for speculative decoding (reference c_api.cpp:410-447):
// same vocabulary, BOS and token table as the target (-3 otherwise), k
// tokens proposed per round at most (default 5, capped at 16). The draft is
// a second engine on the target's GPU with the target's context length.
int fish_set_draft(fish_ctx* ctx, const char* path, int k) {
    if (!ctx || !path) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (!ctx->eng || !ctx->tok) { ctx->err = "load the target model first"; return -1; }
    if (ctx->eng->tp_world() > 1) {
        ctx->err = "draft: speculative decoding with a tensor-parallel target is not supported";
        return -2;
    }
    ctx->draft.reset();
    ctx->draft_ids.clear();
    ctx->stats.draft_active = 0;
    auto d = std::make_unique<fb::Engine>();
    std::string err;
    if (!d->load(path, ctx->eng->cfg().n_ctx, &err)) { ctx->err = "draft: " + err; return -2; }
    const fb::Config& t = ctx->eng->cfg();
    const fb::Config& c = d->cfg();
    if (c.vocab != t.vocab || c.bos != t.bos) {
        ctx->err = "draft model has a different vocabulary (" + std::to_string(c.vocab) + " vs " +
                   std::to_string(t.vocab) + ")";
        return -3;
    }
    const fb::MetaValue* tt = ctx->eng->gguf().meta("tokenizer.ggml.tokens");
    const fb::MetaValue* dt = d->gguf().meta("tokenizer.ggml.tokens");
    if (tt && dt && (tt->sarr.size() != dt->sarr.size() || (tt->sarr.size() > 1000 && tt->sarr[1000] != dt->sarr[1000]))) {
        ctx->err = "draft model tokenizer differs from the target";
        return -3;
    }
    ctx->draft = std::move(d);
    ctx->draft_k = k > 0 ? std::min(k, 16) : 5;
    ctx->stats.draft_active = 1;
    ctx->err.clear();
    return 0;
}

void fish_clear_draft(fish_ctx* ctx) {
    if (!ctx) return;
    std::lock_guard<std::mutex> lock(ctx->mu);
    ctx->draft.reset();
    ctx->draft_ids.clear();
    ctx->stats.draft_active = 0;
}

int fish_set_adapter(fish_ctx* ctx, const char* path, float scale) {
    if (!ctx || !path || !*path || !(scale == scale)) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (!ctx->eng) {
        ctx->adapter_path = path;
        ctx->adapter_scale = scale;
        return 0;
    }
    ctx->err = "adapter: LoRA merging is not supported by the B200 engine";
    return -2;
}

int fish_clear_adapter(fish_ctx* ctx) {
    if (!ctx) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    ctx->adapter_path.clear();
    ctx->adapter_scale = 1.0f;
    return 0;
}

int fish_adapter_info_of(fish_ctx* ctx, fish_adapter_info* out) {
    if (!ctx || !out) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    std::memset(out, 0, sizeof(*out));
    if (!ctx->adapter_path.empty()) {
        out->pending = 1;
        const std::string& p = ctx->adapter_path;
        const size_t sl = p.find_last_of("/\\");
        std::snprintf(out->name, sizeof(out->name), "%s", (sl == std::string::npos ? p : p.substr(sl + 1)).c_str());
        out->scale = ctx->adapter_scale;
    }
    return 0;
}

// ------------------------------------------------------------------ ABI 5

int fish_prefill_ids(fish_ctx* ctx, const int32_t* ids, int n, int pos0, float* logits) {
    if (!ctx || !ids || n <= 0 || pos0 < 0) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (!need_model(ctx)) return -1;
    fb::Engine& e = *ctx->eng;
    if (pos0 > e.seq_len(0)) { ctx->err = "pos0 beyond the cached length"; return -1; }
    e.seq_truncate(0, pos0);
    ctx->cache_ids.resize(std::min(ctx->cache_ids.size(), (size_t)pos0));
    if (!prefill_chunks(ctx, ids, n, false, nullptr)) return -2;
    ctx->cache_ids.insert(ctx->cache_ids.end(), ids, ids + n);
    if (logits) std::memcpy(logits, ctx->logits.data(), sizeof(float) * ctx->logits.size());
    return 0;
}

int fish_decode_ids(fish_ctx* ctx, const int32_t* ids, int n, int pos0, float* logits_all, int32_t* argmax_out) {
    if (!ctx || !ids || n <= 0 || pos0 < 0 || n > fb::kMaxBatch) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (!need_model(ctx)) return -1;
    fb::Engine& e = *ctx->eng;
    if (pos0 > e.seq_len(0)) { ctx->err = "pos0 beyond the cached length"; return -1; }
    e.seq_truncate(0, pos0);
    ctx->cache_ids.resize(std::min(ctx->cache_ids.size(), (size_t)pos0));
    std::string err;
    // only what the caller asked for crosses back (the last row of logits is
    // 513 KB for a 128k vocabulary; no later call reads it from the context)
    if (!e.forward(0, ids, n, nullptr, logits_all, argmax_out, &err)) { ctx->err = err; return -2; }
    ctx->cache_ids.insert(ctx->cache_ids.end(), ids, ids + n);
    return 0;
}

int fbx_layer_probe(fish_ctx* ctx, int layer, int pos0, const float* x_in, int n_tok, float* x_out,
                    fbx_layer_probe_out* out) {
    if (!ctx || !x_in || !x_out || !out || n_tok <= 0) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (!need_model(ctx)) return -1;
    fb::Engine& e = *ctx->eng;
    fb::LayerProbe p;
    std::string err;
    if (!e.layer_probe(layer, pos0, x_in, n_tok, x_out, &p, &err)) { ctx->err = err; return -1; }
    ctx->cache_ids.clear();   // the sequence's KV no longer matches any id list
    for (int st = 0; st < 4; ++st) {
        out->rows[st] = p.rows[st];
        out->K[st] = p.K[st];
        out->has_k[st] = p.has_k[st] ? 1 : 0;
        out->has_32[st] = p.has_32[st] ? 1 : 0;
        if (out->f[st] && !p.f[st].empty()) std::memcpy(out->f[st], p.f[st].data(), sizeof(float) * p.f[st].size());
        if (out->qk[st] && !p.rk[st].empty()) std::memcpy(out->qk[st], p.rk[st].data(), p.rk[st].size());
        if (out->q32[st] && !p.r32[st].empty()) std::memcpy(out->q32[st], p.r32[st].data(), p.r32[st].size());
    }
    out->silu_in_prologue = p.f[4].empty() ? 0 : 1;
    if (out->silu_in_prologue) {
        if (out->gate3) std::memcpy(out->gate3, p.f[4].data(), sizeof(float) * p.f[4].size());
        if (out->up3) std::memcpy(out->up3, p.f[5].data(), sizeof(float) * p.f[5].size());
    }
    return 0;
}

int fish_tp_unique_id(void* out, int cap) {
    if (!out || cap < (int)sizeof(ncclUniqueId)) return (int)sizeof(ncclUniqueId);
    const fb::NcclApi* nc = fb::nccl_api(nullptr);
    ncclUniqueId id;
    if (!nc || nc->get_unique_id(&id) != ncclSuccess) return -1;
    std::memcpy(out, &id, sizeof(id));
    return (int)sizeof(id);
}

int fish_tp_init(fish_ctx* ctx, int rank, int world, const void* id, int id_bytes) {
    if (!ctx || world < 1 || rank < 0 || rank >= world) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (world > 1 && (!id || id_bytes != (int)sizeof(ncclUniqueId))) { ctx->err = "tensor parallelism: bad group id"; return -1; }
    ctx->tp_rank = rank;
    ctx->tp_world = world;
    if (world > 1) std::memcpy(ctx->tp_id, id, sizeof(ncclUniqueId));
    return 0;
}

int fish_decode_greedy(fish_ctx* ctx, int32_t first, int n_steps, int32_t* out_ids) {
    if (!ctx || !out_ids || n_steps < 0) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (!need_model(ctx)) return -1;
    std::string err;
    const int n = ctx->eng->decode_greedy(0, first, n_steps, out_ids, &err);
    if (n < 0) { ctx->err = err; return -2; }
    ctx->cache_ids.push_back(first);
    for (int i = 0; i + 1 < n; ++i) ctx->cache_ids.push_back(out_ids[i]);
    return n;
}

int fish_trace_decode(fish_ctx* ctx, int32_t first, int n_steps, uint64_t* out, int cap) {
    if (!ctx || !out || cap <= 0 || n_steps <= 0) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (!need_model(ctx)) return -1;
    std::vector<int32_t> ids(n_steps);
    std::string err;
    int n = 0, got = 0;
    if (ctx->eng->step_ready()) {
        // persistent step kernel: phase boundaries of the first and the last
        // CTA, as records (ns, tag 5, event, step * 2 + which CTA)
        const size_t vals = (size_t)n_steps * fb::kStepTraceEvents * 2;
        unsigned long long* dev = nullptr;
        if (cudaMalloc(&dev, vals * sizeof(unsigned long long)) != cudaSuccess) { ctx->err = "trace buffer"; return -2; }
        cudaMemset(dev, 0, vals * sizeof(unsigned long long));
        ctx->eng->set_step_trace(dev);
        n = ctx->eng->decode_greedy(0, first, n_steps, ids.data(), &err);
        ctx->eng->set_step_trace(nullptr);
        std::vector<unsigned long long> h(vals);
        cudaMemcpy(h.data(), dev, vals * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
        cudaFree(dev);
        for (size_t i = 0; i < vals && got < cap; ++i) {
            if (!h[i]) continue;
            const size_t step = i / (2 * fb::kStepTraceEvents), ev = (i / 2) % fb::kStepTraceEvents, which = i % 2;
            uint64_t* r = out + 4 * (size_t)got++;
            r[0] = h[i];
            r[1] = 5;
            r[2] = ev;
            r[3] = step * 2 + which;
        }
    } else {
        if (fbk_trace_enable(cap)) { ctx->err = "trace buffer"; return -2; }
        n = ctx->eng->decode_greedy(0, first, n_steps, ids.data(), &err);
        got = fbk_trace_dump(reinterpret_cast<unsigned long long*>(out), cap);
        fbk_trace_enable(0);
    }
    if (n < 0) { ctx->err = err; return -2; }
    ctx->cache_ids.push_back(first);
    for (int i = 0; i + 1 < n; ++i) ctx->cache_ids.push_back(ids[i]);
    return got;
}

int fish_kv_len(fish_ctx* ctx) {
    if (!ctx) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    return ctx->eng ? ctx->eng->seq_len(0) : -1;
}

int fish_set_kv_len(fish_ctx* ctx, int n) {
    if (!ctx || n < 0) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (!need_model(ctx)) return -1;
    ctx->eng->seq_truncate(0, n);
    ctx->cache_ids.resize(std::min(ctx->cache_ids.size(), (size_t)n));
    return 0;
}

int fish_session_open(fish_ctx* ctx) {
    if (!ctx) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (!need_model(ctx)) return -1;
    const int s = ctx->eng->seq_open();
    if (s < 0) ctx->err = "too many sessions";
    return s;
}

int fish_session_fork(fish_ctx* ctx, int parent, int prefix_len) {
    if (!ctx) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (!need_model(ctx)) return -1;
    std::string err;
    const int s = ctx->eng->seq_fork(parent, prefix_len, &err);
    if (s < 0) ctx->err = err;
    return s;
}

int fish_session_close(fish_ctx* ctx, int session) {
    if (!ctx) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (!need_model(ctx)) return -1;
    if (!ctx->eng->seq_close(session)) { ctx->err = "bad session"; return -1; }
    if (session == 0) ctx->cache_ids.clear();
    return 0;
}

int fish_session_len(fish_ctx* ctx, int session) {
    if (!ctx) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    return ctx->eng ? ctx->eng->seq_len(session) : -1;
}

int fish_session_prefill(fish_ctx* ctx, int session, const int32_t* ids, int n, float* logits) {
    if (!ctx || !ids || n <= 0) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (!need_model(ctx)) return -1;
    fb::Engine& e = *ctx->eng;
    int pos = 0;
    while (pos < n) {
        const int m = std::min(fb::kMaxBatch, n - pos);
        std::string err;
        if (!e.forward(session, ids + pos, m, ctx->logits.data(), nullptr, nullptr, &err)) { ctx->err = err; return -2; }
        pos += m;
    }
    if (session == 0) ctx->cache_ids.insert(ctx->cache_ids.end(), ids, ids + n);
    if (logits) std::memcpy(logits, ctx->logits.data(), sizeof(float) * ctx->logits.size());
    return 0;
}

int fish_decode_batch(fish_ctx* ctx, const int* sessions, const int32_t* ids, int n, int32_t* argmax_out, float* logits) {
    if (!ctx || !sessions || !ids || n <= 0) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (!need_model(ctx)) return -1;
    std::string err;
    if (!ctx->eng->decode_batch(sessions, ids, n, argmax_out, logits, &err)) { ctx->err = err; return -2; }
    for (int i = 0; i < n; ++i) if (sessions[i] == 0) ctx->cache_ids.push_back(ids[i]);
    return 0;
}

int fish_session_pages(fish_ctx* ctx, int session, int32_t* out, int cap) {
    if (!ctx) return -1;
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (!need_model(ctx)) return -1;
    const std::vector<int> p = ctx->eng->seq_pages(session);
    if (out && cap >= (int)p.size()) for (size_t i = 0; i < p.size(); ++i) out[i] = p[i];
    return (int)p.size();
}

int fish_kv_page_size(fish_ctx* ctx) {
    (void)ctx;
    return fb::kPageSize;
}

const char* fish_engine_json(fish_ctx* ctx) {
    thread_local std::string buf;
    if (!ctx) return "{}";
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (!ctx->eng) return "{}";
    fb::Engine& e = *ctx->eng;
    long long wr[128] = {0};
    const int kerr = fbk_take_error_flag();
    const int nwr = fbk_take_wait_record(wr);
    std::string recs = "[";
    for (int i = 0; i < std::min(nwr, 8); ++i) {
        if (i) recs += ",";
        recs += "[";
        for (int j = 0; j < 16; ++j) recs += (j ? "," : "") + std::to_string(wr[i * 16 + j]);
        recs += "]";
    }
    recs += "]";
    char b[1024];
    std::snprintf(b, sizeof(b),
                  "{\"device\":\"%s\",\"kv_page_size\":%d,\"kv_free_pages\":%d,\"kv_bytes\":%llu,"
                  "\"weights_device_bytes\":%llu,\"greedy_graph_kernels\":%d,\"step_graph_kernels\":%d,"
                  "\"last_decode_device_ms\":%.6f,\"kernel_error\":%d,\"wait_failures\":%d,"
                  "\"step_kernel\":%d,\"step_grid\":%d,\"step_ring_slots\":%d,\"step_slot_bytes\":%d,"
                  "\"step_weight_bytes\":%.0f,\"last_step_ms\":%.6f,\"last_batch_device_ms\":%.6f,"
                  "\"last_batch_prefix_blocks\":%d,\"tp_world\":%d,\"wait_records\":",
                  e.device_name().c_str(), e.page_size(), e.free_pages(), (unsigned long long)e.kv_bytes(),
                  (unsigned long long)e.device_weight_bytes(), e.graph_kernels(0), e.graph_kernels(1),
                  (double)e.last_greedy_ms(), kerr, nwr, e.step_ready() ? 1 : 0, e.step_grid(), e.step_stages(),
                  e.step_slot_bytes(), e.step_weight_bytes(), (double)e.last_step_ms(), (double)e.last_batch_ms(),
                  e.last_prefix_blocks(), e.tp_world());
    buf = std::string(b) + recs + ",\"step_unavailable\":\"" + e.step_why() + "\"}";
    return buf.c_str();
}

const char* fish_profile_decode_json(fish_ctx* ctx, int32_t first, int n_steps) {
    thread_local std::string buf;
    if (!ctx || n_steps <= 0) return nullptr;
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (!need_model(ctx)) return nullptr;
    std::vector<fb::Engine::ProfClass> cls;
    std::string err;
    if (!ctx->eng->profile_decode(0, first, n_steps, &cls, &err)) { ctx->err = err; return nullptr; }
    buf = "{\"steps\":" + std::to_string(n_steps) + ",\"classes\":[";
    for (size_t i = 0; i < cls.size(); ++i) {
        char b[256];
        std::snprintf(b, sizeof(b), "%s{\"name\":\"%s\",\"launches\":%d,\"ms\":%.6f,\"bytes\":%.0f}", i ? "," : "",
                      cls[i].name.c_str(), cls[i].launches, cls[i].ms, cls[i].bytes);
        buf += b;
    }
    buf += "]}";
    return buf.c_str();
}

}  // extern "C"
