// gguf_synth.cpp — seeded synthetic GGUF models for parity tests and benchmarks.
//
// Writes a llama/qwen2-architecture GGUF v3 file whose weights are N(0, std)
// random values quantised with this file's own Q8_0 / Q4_K / Q6_K encoders, so
// the workloads named by the benchmark configs (tiny Q8_0 llama, Llama-3-8B-,
// Qwen2.5-7B-, Mixtral-8x7B- and Llama-3-70B-shaped Q4_K_M files) can be made
// on any machine without a download. Both engines under test read the same
// file bytes, so parity never depends on how the encoder rounds.
//
// Randomness is counter based (splitmix64 of seed, tensor name and element
// index), so the bytes do not depend on the thread count.
//
// Layouts written (GGUF block specification, as read by the reference at
// include/fish/quant.h:28-52 and src/quant.cpp:129-216):
//   Q8_0  fp16 d, int8 qs[32]
//   Q4_K  fp16 d, fp16 dmin, 12 B packed 6-bit scales/mins, qs[128]
//   Q6_K  ql[128], qh[64], int8 scales[16], fp16 d
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>
#include <map>
#include <vector>

namespace {

constexpr uint32_t T_F32 = 0, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14;

uint16_t f2h(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const int32_t e = static_cast<int32_t>((x >> 23) & 0xFF);
    uint32_t m = x & 0x7FFFFFu;
    if (e == 255) return static_cast<uint16_t>(sign | 0x7C00u | (m ? 0x200u : 0));
    const int32_t he = e - 127 + 15;
    if (he >= 31) return static_cast<uint16_t>(sign | 0x7C00u);
    if (he <= 0) {
        if (he < -10) return static_cast<uint16_t>(sign);
        m |= 0x800000u;
        const int shift = 14 - he;
        uint32_t hm = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (hm & 1u))) ++hm;
        return static_cast<uint16_t>(sign | hm);
    }
    const uint32_t hm = m >> 13, rem = m & 0x1FFFu;
    uint32_t out = sign | (static_cast<uint32_t>(he) << 10) | hm;
    if (rem > 0x1000u || (rem == 0x1000u && (hm & 1u))) ++out;
    return static_cast<uint16_t>(out);
}

float h2f(uint16_t h) {
    const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu, mant = h & 0x3FFu, bits;
    if (exp == 0) {
        if (mant == 0) bits = sign;
        else {
            int e = 113;
            while (!(mant & 0x400u)) { mant <<= 1; --e; }
            bits = sign | (static_cast<uint32_t>(e) << 23) | ((mant & 0x3FFu) << 13);
        }
    } else if (exp == 31) bits = sign | 0x7F800000u | (mant << 13);
    else bits = sign | ((exp + 112) << 23) | (mant << 13);
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

inline uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t name_seed(uint64_t base, const std::string& name) {
    uint64_t h = 1469598103934665603ull ^ base;
    for (unsigned char c : name) h = (h ^ c) * 1099511628211ull;
    return mix64(h);
}

// Standard normal values for elements [i0, i0+n) of a tensor stream (Box-Muller
// over counter-hashed uniform pairs; element 2k and 2k+1 share a pair).
void normals(uint64_t seed, uint64_t i0, size_t n, float stddev, float* out) {
    const double two_pi = 6.283185307179586;
    size_t k = 0;
    uint64_t i = i0;
    while (k < n) {
        const uint64_t pair = i >> 1;
        const uint64_t h1 = mix64(seed ^ (pair * 2 + 0x1234567ull));
        const uint64_t h2 = mix64(seed + (pair * 2 + 1) * 0x9E3779B97F4A7C15ull);
        const double u1 = (static_cast<double>(h1 >> 11) + 0.5) * (1.0 / 9007199254740992.0);
        const double u2 = static_cast<double>(h2 >> 11) * (1.0 / 9007199254740992.0);
        const double r = std::sqrt(-2.0 * std::log(u1));
        const double z = (i & 1) ? r * std::sin(two_pi * u2) : r * std::cos(two_pi * u2);
        out[k++] = static_cast<float>(z) * stddev;
        ++i;
    }
}

inline int nearest_int(float v) { return static_cast<int>(std::lrintf(v)); }

void enc_q8_0(const float* x, uint8_t* out) {
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = std::max(amax, std::fabs(x[i]));
    const uint16_t dh = f2h(amax / 127.0f);
    const float d = h2f(dh);
    std::memcpy(out, &dh, 2);
    int8_t* q = reinterpret_cast<int8_t*>(out + 2);
    for (int i = 0; i < 32; ++i)
        q[i] = static_cast<int8_t>(d > 0 ? std::max(-127, std::min(127, nearest_int(x[i] / d))) : 0);
}

// Q4_K: per 32-wide sub-block an affine grid (scale, min) with 6-bit codes
// relative to the two fp16 super-block factors d and dmin.
void enc_q4_K(const float* x, uint8_t* out) {
    float scale[8], minv[8];
    for (int g = 0; g < 8; ++g) {
        float lo = x[32 * g], hi = x[32 * g];
        for (int l = 1; l < 32; ++l) { lo = std::min(lo, x[32 * g + l]); hi = std::max(hi, x[32 * g + l]); }
        if (lo > 0.0f) lo = 0.0f;
        scale[g] = (hi - lo) / 15.0f;
        minv[g] = -lo;
    }
    float smax = 0.0f, mmax = 0.0f;
    for (int g = 0; g < 8; ++g) { smax = std::max(smax, scale[g]); mmax = std::max(mmax, minv[g]); }
    const uint16_t dh = f2h(smax / 63.0f), mh = f2h(mmax / 63.0f);
    const float d = h2f(dh), dmin = h2f(mh);
    int sc[8], mc[8];
    for (int g = 0; g < 8; ++g) {
        sc[g] = d > 0 ? std::max(0, std::min(63, nearest_int(scale[g] / d))) : 0;
        mc[g] = dmin > 0 ? std::max(0, std::min(63, nearest_int(minv[g] / dmin))) : 0;
    }
    std::memcpy(out, &dh, 2);
    std::memcpy(out + 2, &mh, 2);
    uint8_t* s = out + 4;
    for (int j = 0; j < 4; ++j) {
        s[j] = static_cast<uint8_t>((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = static_cast<uint8_t>((mc[j] & 63) | ((mc[j + 4] >> 4) << 6));
        s[j + 8] = static_cast<uint8_t>((sc[j + 4] & 0x0F) | ((mc[j + 4] & 0x0F) << 4));
    }
    uint8_t* qs = out + 16;
    for (int p = 0; p < 4; ++p) {
        for (int l = 0; l < 32; ++l) {
            int qv[2];
            for (int h = 0; h < 2; ++h) {
                const int g = 2 * p + h;
                const float step = d * static_cast<float>(sc[g]);
                const float off = dmin * static_cast<float>(mc[g]);
                qv[h] = step > 0 ? std::max(0, std::min(15, nearest_int((x[32 * g + l] + off) / step))) : 0;
            }
            qs[32 * p + l] = static_cast<uint8_t>(qv[0] | (qv[1] << 4));
        }
    }
}

// Q6_K: 16 groups of 16 values, signed 8-bit group scales, 6-bit codes - 32.
void enc_q6_K(const float* x, uint8_t* out) {
    float gs[16];
    float amax_all = 0.0f;
    for (int j = 0; j < 16; ++j) {
        float a = 0.0f;
        for (int k = 0; k < 16; ++k) a = std::max(a, std::fabs(x[16 * j + k]));
        gs[j] = a / 31.0f;
        amax_all = std::max(amax_all, gs[j]);
    }
    const uint16_t dh = f2h(amax_all / 127.0f);
    const float d = h2f(dh);
    int sc[16];
    for (int j = 0; j < 16; ++j) sc[j] = d > 0 ? std::max(-128, std::min(127, nearest_int(gs[j] / d))) : 0;
    uint8_t* ql = out;
    uint8_t* qh = out + 128;
    int8_t* scales = reinterpret_cast<int8_t*>(out + 192);
    std::memset(out, 0, 210);
    for (int i = 0; i < 256; ++i) {
        const int half = i / 128, r = i % 128, quad = r / 32, l = r % 32;
        const int j = 8 * half + 2 * quad + l / 16;
        const float step = d * static_cast<float>(sc[j]);
        const int q = (step != 0.0f ? std::max(-32, std::min(31, nearest_int(x[i] / step))) : 0) + 32;
        uint8_t* qlp = ql + 64 * half + l + ((quad & 1) ? 32 : 0);
        if (quad < 2) *qlp = static_cast<uint8_t>((*qlp & 0xF0) | (q & 0x0F));
        else *qlp = static_cast<uint8_t>((*qlp & 0x0F) | ((q & 0x0F) << 4));
        qh[32 * half + l] = static_cast<uint8_t>(qh[32 * half + l] | (((q >> 4) & 3) << (2 * quad)));
    }
    for (int j = 0; j < 16; ++j) scales[j] = static_cast<int8_t>(sc[j]);
    std::memcpy(out + 208, &dh, 2);
}

size_t block_elems(uint32_t t) { return t == T_F32 ? 1 : (t == T_Q8_0 ? 32 : 256); }
size_t block_bytes(uint32_t t) { return t == T_F32 ? 4 : (t == T_Q8_0 ? 34 : (t == T_Q4_K ? 144 : 210)); }

struct TensorSpec {
    std::string name;
    std::vector<uint64_t> ne;
    uint32_t type;
    int fill;          // 0 random normal, 1 constant one, 2 one plus random normal
    float stddev;
    uint64_t offset = 0;
    uint64_t nbytes = 0;
};

struct Writer {
    std::vector<uint8_t> buf;
    void u32(uint32_t v) { const uint8_t* p = reinterpret_cast<uint8_t*>(&v); buf.insert(buf.end(), p, p + 4); }
    void u64(uint64_t v) { const uint8_t* p = reinterpret_cast<uint8_t*>(&v); buf.insert(buf.end(), p, p + 8); }
    void f32(float v) { const uint8_t* p = reinterpret_cast<uint8_t*>(&v); buf.insert(buf.end(), p, p + 4); }
    void i32(int32_t v) { u32(static_cast<uint32_t>(v)); }
    void str(const std::string& s) { u64(s.size()); buf.insert(buf.end(), s.begin(), s.end()); }
    void kv_str(const std::string& k, const std::string& v) { str(k); u32(8); str(v); }
    void kv_u32(const std::string& k, uint32_t v) { str(k); u32(4); u32(v); }
    void kv_i32(const std::string& k, int32_t v) { str(k); u32(5); i32(v); }
    void kv_f32(const std::string& k, float v) { str(k); u32(6); f32(v); }
    void kv_bool(const std::string& k, bool v) { str(k); u32(7); buf.push_back(v ? 1 : 0); }
};

// ---- byte-level BPE test vocabulary

// GPT-2's byte alphabet: printable Latin-1 bytes keep their value, the
// others map to 256, 257, ... in byte order (as UTF-8 text).
std::string byte_char(int b) {
    static std::vector<std::string> table = [] {
        std::vector<std::string> t(256);
        uint32_t next = 256;
        for (int i = 0; i < 256; ++i) {
            const bool keep = (i >= 0x21 && i <= 0x7E) || (i >= 0xA1 && i <= 0xAC) || (i >= 0xAE && i <= 0xFF);
            const uint32_t cp = keep ? static_cast<uint32_t>(i) : next++;
            std::string& o = t[i];
            if (cp < 0x80) o += static_cast<char>(cp);
            else { o += static_cast<char>(0xC0 | (cp >> 6)); o += static_cast<char>(0x80 | (cp & 0x3F)); }
        }
        return t;
    }();
    return table[b & 0xFF];
}

// Text the merges are learned from: words, numbers, contractions,
// punctuation runs, code and a few non-Latin scripts.
const char* kBpeCorpus =
    "The quick brown fox jumps over the lazy dog. It's the 2024 edition, and we're told they'll ship 123456 units; "
    "don't worry, I'm sure you've heard the news. Numbers like 3.14159 and 1,000,000 appear in the text, "
    "as do dates such as 2023-11-05. Punctuation!!! Questions??? Ellipses... and dashes -- everywhere.\n"
    "def train(model, data):\n    for batch in data:\n        loss = model(batch)\n        loss.backward()\n"
    "    return model\n\n"
    "Caf\xC3\xA9 na\xC3\xAFve r\xC3\xA9sum\xC3\xA9 \xC3\xBCber stra\xC3\x9F" "e; "
    "\xD0\x9F\xD1\x80\xD0\xB8\xD0\xB2\xD0\xB5\xD1\x82 \xD0\xBC\xD0\xB8\xD1\x80; "
    "\xE6\x97\xA5\xE6\x9C\xAC\xE8\xAA\x9E\xE3\x81\xAE\xE3\x83\x86\xE3\x82\xAD\xE3\x82\xB9\xE3\x83\x88. "
    "the theory of the thing: there, then, those, these, this, that, than, thank. interesting internal international "
    "information. running jumping swimming reading writing. hello world, hello there, hello again.\n";

struct BpeVocab {
    std::vector<std::string> tokens;
    std::vector<int32_t> types;
    std::vector<std::string> merges;
    int bos = 0, eos = 0;
};

// 256 byte characters, then merges learned greedily on the corpus (the most
// frequent adjacent pair, ties to the lower pair of ids; spaces attach to the
// following word), then a few control tokens, then filler up to `vocab`.
BpeVocab build_bpe_vocab(int vocab, int n_merges) {
    BpeVocab v;
    std::map<std::string, int> id;
    auto add = [&](const std::string& t, int type) {
        id.emplace(t, static_cast<int>(v.tokens.size()));
        v.tokens.push_back(t);
        v.types.push_back(type);
    };
    for (int b = 0; b < 256; ++b) add(byte_char(b), 1);
    std::vector<std::vector<int>> words;
    {
        const std::string text = kBpeCorpus;
        std::vector<int> cur;
        for (size_t i = 0; i < text.size(); ++i) {
            const unsigned char ch = static_cast<unsigned char>(text[i]);
            if ((ch == ' ' || ch == '\n') && !cur.empty()) { words.push_back(cur); cur.clear(); }
            cur.push_back(ch);
        }
        if (!cur.empty()) words.push_back(cur);
    }
    for (int m = 0; m < n_merges; ++m) {
        std::map<std::pair<int, int>, int> count;
        for (const auto& w : words)
            for (size_t i = 0; i + 1 < w.size(); ++i) ++count[{w[i], w[i + 1]}];
        std::pair<int, int> best{-1, -1};
        int bc = 1;
        for (const auto& [pr, c] : count)
            if (c > bc) { bc = c; best = pr; }
        if (best.first < 0) break;
        const std::string joined = v.tokens[best.first] + v.tokens[best.second];
        if (id.count(joined)) break;
        v.merges.push_back(v.tokens[best.first] + " " + v.tokens[best.second]);
        const int nid = static_cast<int>(v.tokens.size());
        add(joined, 1);
        for (auto& w : words) {
            std::vector<int> o;
            for (size_t i = 0; i < w.size(); ++i) {
                if (i + 1 < w.size() && w[i] == best.first && w[i + 1] == best.second) { o.push_back(nid); ++i; }
                else o.push_back(w[i]);
            }
            w.swap(o);
        }
    }
    v.bos = static_cast<int>(v.tokens.size());
    for (const char* sp : {"<|begin_of_text|>", "<|end_of_text|>", "<|start_header_id|>", "<|end_header_id|>",
                           "<|eot_id|>", "<|im_start|>", "<|im_end|>"})
        add(sp, 3);
    v.eos = v.bos + 1;
    for (int i = static_cast<int>(v.tokens.size()); i < vocab; ++i) add("<filler " + std::to_string(i) + ">", 1);
    return v;
}

}  // namespace

extern "C" {

// Shape and encoding of a synthetic model. wtype: 8 = every matrix Q8_0;
// 12 = "Q4_K_M" mixture (token_embd Q4_K, output Q6_K, attn_v / ffn_down in
// Q6_K on even layers and Q4_K on odd ones, every other matrix Q4_K).
typedef struct fish_synth_config {
    const char* arch;            // "llama", "qwen2" or "qwen3"
    int n_layers, n_embd, n_ff, n_head, n_head_kv, vocab, n_ctx_train;
    float eps, freq_base;
    int n_experts, n_experts_per_tok;
    int qkv_bias;
    int wtype;
    unsigned long long seed;
    float wstd;                  // weight std (0.02)
    float router_std;            // MoE router std (1/64: logits on a unit-RMS input of width 4096 ~ N(0, 1))
    const char* chat_template;   // tokenizer.chat_template; nullptr or "" writes none
    const char* bpe_pre;         // nullptr / "": SentencePiece dummy vocabulary; else a byte-level BPE
                                 // vocabulary with this tokenizer.ggml.pre name (merges learned from
                                 // a built-in text)
    int qk_norm;                 // 1: per-head q/k RMSNorm weights (attn_q_norm / attn_k_norm, qwen3),
                                 // 1 + N(0, 0.1) so they are not the identity
    // gemma2: attention-score and final-logit soft caps (0: the format's
    // defaults 50 / 30) and the sliding window of the even layers (0: 4096)
    float attn_softcap, final_softcap;
    int sliding_window;
    // phi3 longrope: rope.scaling.original_context_length (0: n_ctx_train)
    // and rope.scaling.attn_factor (0: 1)
    int rope_orig_ctx;
    float rope_attn_factor;
    // MoE: rows of a shared expert every token takes (0: none), with a
    // one-row F32 sigmoid gate (qwen2moe)
    int n_ff_shexp;
    int o_bias;                  // 1: attn_output.bias
    int no_bos;                  // 1: tokenizer.ggml.add_bos_token = false (Qwen-style files)
} fish_synth_config;

__attribute__((visibility("default")))
int fish_synth_write(const char* path, const fish_synth_config* c, int n_threads, char* err, int cap) {
    auto fail = [&](const char* why) { if (err && cap > 0) std::snprintf(err, static_cast<size_t>(cap), "%s", why); return -1; };
    if (!path || !c || c->n_layers <= 0 || c->n_embd <= 0 || c->n_head <= 0 || c->vocab < 300)
        return fail("bad synth config");
    if (n_threads <= 0) n_threads = static_cast<int>(std::max(1u, std::thread::hardware_concurrency()));
    const std::string arch = c->arch ? c->arch : "llama";
    const int E = c->n_embd, F = c->n_ff, H = c->n_head, HKV = c->n_head_kv > 0 ? c->n_head_kv : c->n_head;
    const int D = E / H;
    const bool q8 = c->wtype == 8;
    const uint32_t tm = q8 ? T_Q8_0 : T_Q4_K;
    const float wstd = c->wstd > 0 ? c->wstd : 0.02f;

    std::vector<TensorSpec> ts;
    auto add = [&](const std::string& n, std::vector<uint64_t> ne, uint32_t t, int fill, float sd) {
        ts.push_back(TensorSpec{n, std::move(ne), t, fill, sd});
    };
    // gemma2 stores its norm weights as w with 1 + w applied (so N(0, 0.1)
    // here is 1 + N(0, 0.1)), adds post-attention / post-FFN norms and ties
    // the output to the embedding; phi3 fuses q|k|v and gate|up and carries
    // longrope factor vectors
    const bool gemma2 = arch == "gemma2", phi3 = arch == "phi3";
    const int nfill = gemma2 ? 0 : 1;
    const float nsd = gemma2 ? 0.1f : 0.0f;
    add("token_embd.weight", {static_cast<uint64_t>(E), static_cast<uint64_t>(c->vocab)}, tm, 0, wstd);
    if (phi3) {
        add("rope_factors_short.weight", {static_cast<uint64_t>(D / 2)}, T_F32, 2, 0.05f);
        add("rope_factors_long.weight", {static_cast<uint64_t>(D / 2)}, T_F32, 2, 0.25f);
    }
    for (int i = 0; i < c->n_layers; ++i) {
        const std::string p = "blk." + std::to_string(i) + ".";
        const uint32_t tv = q8 ? T_Q8_0 : ((i % 2) == 0 ? T_Q6_K : T_Q4_K);
        add(p + "attn_norm.weight", {static_cast<uint64_t>(E)}, T_F32, nfill, nsd);
        if (phi3) {
            add(p + "attn_qkv.weight", {static_cast<uint64_t>(E), static_cast<uint64_t>((H + 2 * HKV) * D)}, tm, 0, wstd);
            if (c->qkv_bias) add(p + "attn_qkv.bias", {static_cast<uint64_t>((H + 2 * HKV) * D)}, T_F32, 0, wstd);
            add(p + "attn_output.weight", {static_cast<uint64_t>(H * D), static_cast<uint64_t>(E)}, tm, 0, wstd);
            if (c->o_bias) add(p + "attn_output.bias", {static_cast<uint64_t>(E)}, T_F32, 0, wstd);
            add(p + "ffn_norm.weight", {static_cast<uint64_t>(E)}, T_F32, 1, 0);
            add(p + "ffn_up.weight", {static_cast<uint64_t>(E), static_cast<uint64_t>(2 * F)}, tm, 0, wstd);
            add(p + "ffn_down.weight", {static_cast<uint64_t>(F), static_cast<uint64_t>(E)}, tv, 0, wstd);
            continue;
        }
        add(p + "attn_q.weight", {static_cast<uint64_t>(E), static_cast<uint64_t>(H * D)}, tm, 0, wstd);
        add(p + "attn_k.weight", {static_cast<uint64_t>(E), static_cast<uint64_t>(HKV * D)}, tm, 0, wstd);
        add(p + "attn_v.weight", {static_cast<uint64_t>(E), static_cast<uint64_t>(HKV * D)}, tv, 0, wstd);
        if (c->qkv_bias) {
            add(p + "attn_q.bias", {static_cast<uint64_t>(H * D)}, T_F32, 0, wstd);
            add(p + "attn_k.bias", {static_cast<uint64_t>(HKV * D)}, T_F32, 0, wstd);
            add(p + "attn_v.bias", {static_cast<uint64_t>(HKV * D)}, T_F32, 0, wstd);
        }
        if (c->qk_norm) {
            add(p + "attn_q_norm.weight", {static_cast<uint64_t>(D)}, T_F32, 2, 0.1f);
            add(p + "attn_k_norm.weight", {static_cast<uint64_t>(D)}, T_F32, 2, 0.1f);
        }
        add(p + "attn_output.weight", {static_cast<uint64_t>(H * D), static_cast<uint64_t>(E)}, tm, 0, wstd);
        if (c->o_bias) add(p + "attn_output.bias", {static_cast<uint64_t>(E)}, T_F32, 0, wstd);
        if (gemma2) add(p + "post_attention_norm.weight", {static_cast<uint64_t>(E)}, T_F32, nfill, nsd);
        add(p + "ffn_norm.weight", {static_cast<uint64_t>(E)}, T_F32, nfill, nsd);
        if (gemma2) add(p + "post_ffw_norm.weight", {static_cast<uint64_t>(E)}, T_F32, nfill, nsd);
        if (c->n_experts > 0) {
            const uint64_t NE = static_cast<uint64_t>(c->n_experts);
            add(p + "ffn_gate_inp.weight", {static_cast<uint64_t>(E), NE}, T_F32, 0,
                c->router_std > 0 ? c->router_std : 0.015625f);
            add(p + "ffn_gate_exps.weight", {static_cast<uint64_t>(E), static_cast<uint64_t>(F), NE}, tm, 0, wstd);
            add(p + "ffn_up_exps.weight", {static_cast<uint64_t>(E), static_cast<uint64_t>(F), NE}, tm, 0, wstd);
            add(p + "ffn_down_exps.weight", {static_cast<uint64_t>(F), static_cast<uint64_t>(E), NE}, tv, 0, wstd);
            if (c->n_ff_shexp > 0) {
                const uint64_t FS = static_cast<uint64_t>(c->n_ff_shexp);
                add(p + "ffn_gate_inp_shexp.weight", {static_cast<uint64_t>(E)}, T_F32, 0,
                    c->router_std > 0 ? c->router_std : 0.015625f);
                add(p + "ffn_gate_shexp.weight", {static_cast<uint64_t>(E), FS}, tm, 0, wstd);
                add(p + "ffn_up_shexp.weight", {static_cast<uint64_t>(E), FS}, tm, 0, wstd);
                add(p + "ffn_down_shexp.weight", {FS, static_cast<uint64_t>(E)}, tv, 0, wstd);
            }
        } else {
            add(p + "ffn_gate.weight", {static_cast<uint64_t>(E), static_cast<uint64_t>(F)}, tm, 0, wstd);
            add(p + "ffn_up.weight", {static_cast<uint64_t>(E), static_cast<uint64_t>(F)}, tm, 0, wstd);
            add(p + "ffn_down.weight", {static_cast<uint64_t>(F), static_cast<uint64_t>(E)}, tv, 0, wstd);
        }
    }
    add("output_norm.weight", {static_cast<uint64_t>(E)}, T_F32, nfill, nsd);
    if (!gemma2)
        add("output.weight", {static_cast<uint64_t>(E), static_cast<uint64_t>(c->vocab)}, q8 ? T_Q8_0 : T_Q6_K, 0, wstd);

    for (auto& t : ts) {
        if (t.ne[0] % block_elems(t.type)) return fail("row not a whole number of blocks");
        uint64_t rows = 1;
        for (size_t d = 1; d < t.ne.size(); ++d) rows *= t.ne[d];
        t.nbytes = t.ne[0] / block_elems(t.type) * block_bytes(t.type) * rows;
    }
    const uint64_t align = 32;
    uint64_t off = 0;
    for (auto& t : ts) { t.offset = off; off = (off + t.nbytes + align - 1) / align * align; }

    Writer w;
    w.u32(0x46554747u);
    w.u32(3);
    w.u64(ts.size());
    const uint64_t n_kv_pos = w.buf.size();
    w.u64(0);
    uint64_t n_kv = 0;
    auto k = [&](const std::string& s) { return arch + "." + s; };
    w.kv_str("general.architecture", arch); ++n_kv;
    w.kv_str("general.name", "fish-b200 synthetic"); ++n_kv;
    w.kv_str("general.description", q8 ? "synthetic N(0,std) weights, every matrix Q8_0"
                                        : "synthetic N(0,std) weights, Q4_K_M mixture: output Q6_K; attn_v and ffn_down Q6_K on even layers, Q4_K on odd; all other matrices Q4_K"); ++n_kv;
    w.kv_u32("general.alignment", static_cast<uint32_t>(align)); ++n_kv;
    w.kv_u32(k("block_count"), static_cast<uint32_t>(c->n_layers)); ++n_kv;
    w.kv_u32(k("context_length"), static_cast<uint32_t>(c->n_ctx_train > 0 ? c->n_ctx_train : 8192)); ++n_kv;
    w.kv_u32(k("embedding_length"), static_cast<uint32_t>(E)); ++n_kv;
    w.kv_u32(k("feed_forward_length"), static_cast<uint32_t>(F)); ++n_kv;
    w.kv_u32(k("attention.head_count"), static_cast<uint32_t>(H)); ++n_kv;
    w.kv_u32(k("attention.head_count_kv"), static_cast<uint32_t>(HKV)); ++n_kv;
    w.kv_f32(k("attention.layer_norm_rms_epsilon"), c->eps > 0 ? c->eps : 1e-5f); ++n_kv;
    w.kv_f32(k("rope.freq_base"), c->freq_base > 0 ? c->freq_base : 10000.0f); ++n_kv;
    w.kv_u32(k("vocab_size"), static_cast<uint32_t>(c->vocab)); ++n_kv;
    if (gemma2) {
        w.kv_f32(k("attn_logit_softcapping"), c->attn_softcap > 0 ? c->attn_softcap : 50.0f); ++n_kv;
        w.kv_f32(k("final_logit_softcapping"), c->final_softcap > 0 ? c->final_softcap : 30.0f); ++n_kv;
        w.kv_u32(k("attention.sliding_window"), static_cast<uint32_t>(c->sliding_window > 0 ? c->sliding_window : 4096)); ++n_kv;
    }
    if (phi3) {
        w.kv_str(k("rope.scaling.type"), "longrope"); ++n_kv;
        w.kv_u32(k("rope.scaling.original_context_length"),
                 static_cast<uint32_t>(c->rope_orig_ctx > 0 ? c->rope_orig_ctx : (c->n_ctx_train > 0 ? c->n_ctx_train : 8192))); ++n_kv;
        w.kv_f32(k("rope.scaling.attn_factor"), c->rope_attn_factor > 0 ? c->rope_attn_factor : 1.0f); ++n_kv;
    }
    if (c->n_experts > 0) {
        w.kv_u32(k("expert_count"), static_cast<uint32_t>(c->n_experts)); ++n_kv;
        w.kv_u32(k("expert_used_count"), static_cast<uint32_t>(c->n_experts_per_tok)); ++n_kv;
        w.kv_u32(k("expert_feed_forward_length"), static_cast<uint32_t>(F)); ++n_kv;
        if (c->n_ff_shexp > 0) {
            w.kv_u32(k("expert_shared_feed_forward_length"), static_cast<uint32_t>(c->n_ff_shexp)); ++n_kv;
        }
    }
    if (c->bpe_pre && c->bpe_pre[0]) {
        // byte-level BPE vocabulary (see build_bpe_vocab)
        const BpeVocab bv = build_bpe_vocab(c->vocab, 400);
        if (static_cast<int>(bv.tokens.size()) != c->vocab) return fail("vocabulary too small for the BPE tokens");
        w.kv_str("tokenizer.ggml.model", "gpt2"); ++n_kv;
        w.kv_str("tokenizer.ggml.pre", c->bpe_pre); ++n_kv;
        w.str("tokenizer.ggml.tokens"); w.u32(9); w.u32(8); w.u64(bv.tokens.size());
        for (const auto& t : bv.tokens) w.str(t);
        ++n_kv;
        w.str("tokenizer.ggml.token_type"); w.u32(9); w.u32(5); w.u64(bv.types.size());
        for (int32_t t : bv.types) w.i32(t);
        ++n_kv;
        w.str("tokenizer.ggml.merges"); w.u32(9); w.u32(8); w.u64(bv.merges.size());
        for (const auto& m : bv.merges) w.str(m);
        ++n_kv;
        w.kv_u32("tokenizer.ggml.bos_token_id", static_cast<uint32_t>(bv.bos)); ++n_kv;
        w.kv_u32("tokenizer.ggml.eos_token_id", static_cast<uint32_t>(bv.eos)); ++n_kv;
        w.kv_bool("tokenizer.ggml.add_bos_token", !c->no_bos); ++n_kv;
    } else {
    // SentencePiece dummy vocabulary: <unk> <s> </s>, 256 byte tokens, then
    // "▁t<i>" pieces up to the vocabulary size.
    w.kv_str("tokenizer.ggml.model", "llama"); ++n_kv;
    w.str("tokenizer.ggml.tokens"); w.u32(9); w.u32(8); w.u64(static_cast<uint64_t>(c->vocab));
    for (int i = 0; i < c->vocab; ++i) {
        if (i == 0) w.str("<unk>");
        else if (i == 1) w.str("<s>");
        else if (i == 2) w.str("</s>");
        else if (i < 259) { char b[8]; std::snprintf(b, sizeof(b), "<0x%02X>", i - 3); w.str(b); }
        else w.str("\xE2\x96\x81t" + std::to_string(i));
    }
    ++n_kv;
    w.str("tokenizer.ggml.scores"); w.u32(9); w.u32(6); w.u64(static_cast<uint64_t>(c->vocab));
    for (int i = 0; i < c->vocab; ++i) w.f32(i < 259 ? 0.0f : -static_cast<float>(i));
    ++n_kv;
    w.str("tokenizer.ggml.token_type"); w.u32(9); w.u32(5); w.u64(static_cast<uint64_t>(c->vocab));
    for (int i = 0; i < c->vocab; ++i) w.i32(i == 0 ? 2 : (i < 3 ? 3 : (i < 259 ? 6 : 1)));
    ++n_kv;
    w.kv_u32("tokenizer.ggml.bos_token_id", 1); ++n_kv;
    w.kv_u32("tokenizer.ggml.eos_token_id", 2); ++n_kv;
    w.kv_u32("tokenizer.ggml.unknown_token_id", 0); ++n_kv;
    w.kv_bool("tokenizer.ggml.add_bos_token", !c->no_bos); ++n_kv;
    }
    if (c->chat_template && c->chat_template[0]) { w.kv_str("tokenizer.chat_template", c->chat_template); ++n_kv; }
    std::memcpy(w.buf.data() + n_kv_pos, &n_kv, 8);

    for (const auto& t : ts) {
        w.str(t.name);
        w.u32(static_cast<uint32_t>(t.ne.size()));
        for (uint64_t d : t.ne) w.u64(d);
        w.u32(t.type);
        w.u64(t.offset);
    }
    while (w.buf.size() % align) w.buf.push_back(0);

    FILE* f = std::fopen(path, "wb");
    if (!f) return fail("cannot create output file");
    if (std::fwrite(w.buf.data(), 1, w.buf.size(), f) != w.buf.size()) { std::fclose(f); return fail("write failed"); }

    std::vector<uint8_t> data;
    uint64_t written = 0;
    for (const auto& t : ts) {
        while (written < t.offset) { std::fputc(0, f); ++written; }
        data.assign(static_cast<size_t>(t.nbytes), 0);
        const uint64_t be = block_elems(t.type), bb = block_bytes(t.type);
        const uint64_t n_blocks = t.nbytes / bb;
        const uint64_t seed = name_seed(c->seed, t.name);
        std::atomic<uint64_t> next{0};
        const uint64_t chunk = 4096;
        auto work = [&]() {
            std::vector<float> vals(static_cast<size_t>(be * chunk));
            for (;;) {
                const uint64_t b0 = next.fetch_add(chunk);
                if (b0 >= n_blocks) break;
                const uint64_t nb = std::min(chunk, n_blocks - b0);
                if (t.fill == 1) std::fill(vals.begin(), vals.begin() + static_cast<long>(nb * be), 1.0f);
                else normals(seed, b0 * be, static_cast<size_t>(nb * be), t.stddev, vals.data());
                if (t.fill == 2)
                    for (uint64_t i = 0; i < nb * be; ++i) vals[static_cast<size_t>(i)] += 1.0f;
                for (uint64_t b = 0; b < nb; ++b) {
                    uint8_t* o = data.data() + (b0 + b) * bb;
                    const float* x = vals.data() + b * be;
                    switch (t.type) {
                        case T_F32: std::memcpy(o, x, 4); break;
                        case T_Q8_0: enc_q8_0(x, o); break;
                        case T_Q4_K: enc_q4_K(x, o); break;
                        default: enc_q6_K(x, o); break;
                    }
                }
            }
        };
        std::vector<std::thread> th;
        for (int i = 1; i < n_threads; ++i) th.emplace_back(work);
        work();
        for (auto& x : th) x.join();
        if (std::fwrite(data.data(), 1, data.size(), f) != data.size()) { std::fclose(f); return fail("write failed"); }
        written += t.nbytes;
    }
    std::fclose(f);
    return 0;
}

}  // extern "C"
