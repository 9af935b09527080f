// tokenizer.cpp — see tokenizer.h.
//
// The observable rules are the reference's (model/fish/src/tokenizer.cpp) —
// they decide which ids a prompt becomes, so they must be the same:
//   * vocabulary set-up from the GGUF metadata (bos / eos / unk ids, the
//     end-of-generation set, digit grouping by `tokenizer.ggml.pre`, merge
//     ranks, special tokens, SPM byte-fallback ids, chat-format detection);
//   * the byte-level BPE pre-split of the llama3 / qwen2 split expressions
//     (contractions | [^\r\n L N]? L+ | N{1,k} |  ?[^\s L N]+[\r\n]* |
//     \s*[\r\n]+ | \s+(?!\S) | \s+, with the reference's character classes);
//   * BPE: repeatedly merge the adjacent pair of lowest merge rank, the
//     leftmost one on ties; SentencePiece: repeatedly merge the adjacent pair
//     whose joined piece has the highest score, the leftmost on ties, then
//     <0xNN> byte fallback;
//   * specials matched longest first at code-point boundaries;
//   * the chat templates' exact strings.
// The code is this library's own: text is decoded once into classified code
// points, the pre-split is a table of rules tried in order, both merge loops
// run on a linked list with a priority queue of candidate pairs (stale
// candidates dropped when popped), specials are found with a byte trie, and
// token texts are decoded once at load.
#include "tokenizer.h"

#include <algorithm>
#include <cstring>
#include <queue>

namespace fb {

namespace {

const char kSpaceMark[] = "\xE2\x96\x81";   // U+2581, SentencePiece's word boundary

// ------------------------------------------------------------ UTF-8

// One code point at p (n bytes left): its value and byte length. A lead byte
// whose sequence runs past the end, or a byte that cannot lead, stands for
// itself as a one-byte unit; continuation bytes are not checked.
uint32_t utf8_at(const unsigned char* p, size_t n, size_t* len) {
    const unsigned char c = p[0];
    const size_t L = c < 0x80 ? 1 : (c >> 5) == 0x6 ? 2 : (c >> 4) == 0xE ? 3 : (c >> 3) == 0x1E ? 4 : 1;
    if (L == 1 || L > n) {
        *len = 1;
        return c;
    }
    uint32_t v = c & (0x7Fu >> L);
    for (size_t k = 1; k < L; ++k) v = (v << 6) | (p[k] & 0x3Fu);
    *len = L;
    return v;
}

void append_utf8(std::string& o, uint32_t cp) {
    char b[4];
    int n;
    if (cp < 0x80) { b[0] = (char)cp; n = 1; }
    else if (cp < 0x800) { b[0] = (char)(0xC0 | (cp >> 6)); b[1] = (char)(0x80 | (cp & 0x3F)); n = 2; }
    else if (cp < 0x10000) {
        b[0] = (char)(0xE0 | (cp >> 12)); b[1] = (char)(0x80 | ((cp >> 6) & 0x3F)); b[2] = (char)(0x80 | (cp & 0x3F));
        n = 3;
    } else {
        b[0] = (char)(0xF0 | (cp >> 18)); b[1] = (char)(0x80 | ((cp >> 12) & 0x3F));
        b[2] = (char)(0x80 | ((cp >> 6) & 0x3F)); b[3] = (char)(0x80 | (cp & 0x3F));
        n = 4;
    }
    o.append(b, (size_t)n);
}

// ------------------------------------------------------------ character classes

enum : uint8_t { K_LETTER = 1, K_DIGIT = 2, K_SPACE = 4, K_NEWLINE = 8 };

struct Span { uint32_t lo, hi; };

const Span kDigits[] = {{0x30, 0x39}, {0xB2, 0xB3}, {0xB9, 0xB9}, {0xBC, 0xBE}, {0x660, 0x669}, {0x6F0, 0x6F9},
                        {0x966, 0x96F}, {0x9E6, 0x9EF}, {0xFF10, 0xFF19}};
const Span kSpaces[] = {{0x09, 0x0D}, {0x20, 0x20}, {0x85, 0x85}, {0xA0, 0xA0}, {0x1680, 0x1680}, {0x2000, 0x200A},
                        {0x2028, 0x2029}, {0x202F, 0x202F}, {0x205F, 0x205F}, {0x3000, 0x3000}};
// Above U+00BF every code point counts as a letter except these (and the digits).
const Span kNotLetters[] = {{0xD7, 0xD7}, {0xF7, 0xF7}, {0x2000, 0x2BFF}, {0x3000, 0x303F}, {0xE000, 0xF8FF},
                            {0xFE00, 0xFE0F}, {0xFF00, 0xFF20}, {0x1F000, 0x1FAFF}};

template <size_t N>
bool in_spans(const Span (&t)[N], uint32_t c) {
    for (const Span& s : t)
        if (c >= s.lo && c <= s.hi) return true;
    return false;
}

uint8_t classify(uint32_t c) {
    uint8_t k = 0;
    const bool digit = in_spans(kDigits, c);
    if (digit) k |= K_DIGIT;
    if (in_spans(kSpaces, c)) k |= K_SPACE;
    if (c == '\n' || c == '\r') k |= K_NEWLINE;
    bool letter;
    if (c < 0x80) letter = (c | 0x20) >= 'a' && (c | 0x20) <= 'z';
    else if (c < 0xC0) letter = c == 0xAA || c == 0xB5 || c == 0xBA;
    else letter = !digit && !in_spans(kNotLetters, c);
    if (letter) k |= K_LETTER;
    return k;
}

struct Cp {
    uint32_t v;
    uint32_t at;    // byte offset
    uint8_t kind;
};

std::vector<Cp> decode_text(const std::string& s) {
    std::vector<Cp> out;
    out.reserve(s.size());
    const unsigned char* p = reinterpret_cast<const unsigned char*>(s.data());
    for (size_t i = 0; i < s.size();) {
        size_t len;
        const uint32_t v = utf8_at(p + i, s.size() - i, &len);
        out.push_back({v, (uint32_t)i, classify(v)});
        i += len;
    }
    return out;
}

// ------------------------------------------------------------ byte-level BPE alphabet

// GPT-2's reversible byte -> printable code point map: printable Latin-1
// bytes keep their value, the rest take 256, 257, ... in byte order.
struct ByteAlphabet {
    std::string to_text[256];
    std::unordered_map<uint32_t, uint8_t> to_byte;
    ByteAlphabet() {
        uint32_t next = 256;
        for (int b = 0; b < 256; ++b) {
            const bool keep = (b >= 0x21 && b <= 0x7E) || (b >= 0xA1 && b <= 0xAC) || (b >= 0xAE && b <= 0xFF);
            const uint32_t cp = keep ? (uint32_t)b : next++;
            append_utf8(to_text[b], cp);
            to_byte[cp] = (uint8_t)b;
        }
    }
};
const ByteAlphabet& byte_alphabet() {
    static const ByteAlphabet a;
    return a;
}

// ------------------------------------------------------------ pre-split rules

// Each rule looks at code point i of the text and returns the end (one past
// the last code point) of the piece it takes there, or 0 when it does not
// apply. The splitter tries them in table order; the last always applies.
struct SplitCtx {
    const std::vector<Cp>& c;
    int max_digits;   // 0: digit runs of any length
    size_t n() const { return c.size(); }
    bool is(size_t i, uint8_t k) const { return i < c.size() && (c[i].kind & k); }
};
using Rule = size_t (*)(const SplitCtx&, size_t);

size_t rule_contraction(const SplitCtx& x, size_t i) {
    // an apostrophe and one of the English contraction tails, any case
    if (x.c[i].v != '\'') return 0;
    static const char* const kTails[] = {"s", "t", "re", "ve", "m", "ll", "d"};
    for (const char* t : kTails) {
        const size_t L = std::strlen(t);
        if (i + 1 + L > x.n()) continue;
        bool eq = true;
        for (size_t k = 0; k < L && eq; ++k) {
            const uint32_t v = x.c[i + 1 + k].v;
            eq = v < 0x80 && (char)((v >= 'A' && v <= 'Z') ? v + 32 : v) == t[k];
        }
        if (eq) return i + 1 + L;
    }
    return 0;
}

size_t run_of(const SplitCtx& x, size_t j, uint8_t k) {
    while (j < x.n() && (x.c[j].kind & k)) ++j;
    return j;
}

size_t rule_letters(const SplitCtx& x, size_t i) {
    // L+, or one code point that is neither a newline nor a digit, then L+
    if (x.is(i, K_LETTER)) return run_of(x, i, K_LETTER);
    if (!(x.c[i].kind & (K_NEWLINE | K_DIGIT)) && x.is(i + 1, K_LETTER)) return run_of(x, i + 1, K_LETTER);
    return 0;
}

size_t rule_digits(const SplitCtx& x, size_t i) {
    if (!x.is(i, K_DIGIT)) return 0;
    size_t j = i;
    while (j < x.n() && (x.c[j].kind & K_DIGIT) && (x.max_digits == 0 || (int)(j - i) < x.max_digits)) ++j;
    return j;
}

size_t rule_punct(const SplitCtx& x, size_t i) {
    // an optional space, a run of code points that are not space / letter /
    // digit, then any newlines
    const size_t st = x.c[i].v == ' ' ? i + 1 : i;
    const uint8_t word = K_SPACE | K_LETTER | K_DIGIT;
    if (st >= x.n() || (x.c[st].kind & word)) return 0;
    size_t j = st;
    while (j < x.n() && !(x.c[j].kind & word)) ++j;
    return run_of(x, j, K_NEWLINE);
}

size_t rule_spaces(const SplitCtx& x, size_t i) {
    if (!x.is(i, K_SPACE)) return 0;
    const size_t e = run_of(x, i, K_SPACE);
    size_t after_nl = 0;
    for (size_t j = i; j < e; ++j)
        if (x.c[j].kind & K_NEWLINE) after_nl = j + 1;
    if (after_nl) return after_nl;              // \s*[\r\n]+
    if (e < x.n() && e - 1 > i) return e - 1;   // \s+(?!\S): the last space stays with the next piece
    return e;                                   // \s+
}

size_t rule_single(const SplitCtx&, size_t i) { return i + 1; }

const Rule kSplitRules[] = {rule_contraction, rule_letters, rule_digits, rule_punct, rule_spaces, rule_single};

// ------------------------------------------------------------ merge loops

// Symbols of a piece in a doubly linked list; merging keeps the left one.
struct Node {
    int prev, next;
    int32_t id;       // BPE: token id
    uint32_t at, len; // SPM: byte span in the text
};

struct Candidate {
    double key;   // smaller is merged first
    int left, right;
    uint32_t stamp_l, stamp_r;
    bool operator<(const Candidate& o) const {   // std::priority_queue keeps the largest on top
        if (key != o.key) return key > o.key;
        return left > o.left;
    }
};

// ------------------------------------------------------------ chat templates

struct ChatBuilder {
    std::vector<std::pair<std::string, bool>>& out;   // (text, parse specials)
    void tag(const std::string& s) const { if (!s.empty()) out.emplace_back(s, true); }
    void text(const std::string& s) const { if (!s.empty()) out.emplace_back(s, false); }
};

// chat format by the markers its template or vocabulary holds, in the
// reference's order of precedence
struct FormatMarker {
    ChatFormat f;
    const char* a;
    const char* b;   // both must be present (nullptr: one marker)
};
const FormatMarker kTemplateMarkers[] = {
    {ChatFormat::Llama3, "<|start_header_id|>", nullptr},
    {ChatFormat::ChatML, "<|im_start|>", nullptr},
    {ChatFormat::Gemma, "<start_of_turn>", nullptr},
    {ChatFormat::Phi3, "<|user|>", "<|end|>"},
    {ChatFormat::DeepSeek, "User\xEF\xBD\x9C>", nullptr},
    {ChatFormat::Mistral, "[INST]", nullptr},
};
const FormatMarker kVocabMarkers[] = {
    {ChatFormat::Llama3, "<|start_header_id|>", "<|end_header_id|>"},
    {ChatFormat::ChatML, "<|im_start|>", nullptr},
    {ChatFormat::Phi3, "<|user|>", "<|end|>"},
    {ChatFormat::Gemma, "<start_of_turn>", nullptr},
    {ChatFormat::DeepSeek, "<\xEF\xBD\x9C" "User\xEF\xBD\x9C>", nullptr},
    {ChatFormat::Mistral, "[INST]", nullptr},
};

// digit-group length of the byte-level pre-split by `tokenizer.ggml.pre`
int digits_for(const std::string& pre) {
    static const char* const kSingle[] = {"qwen2", "qwen35", "deepseek-llm", "deepseek-coder", "deepseek-v3",
                                          "stablelm2", "command-r", "olmo", "dbrx", "chatglm-bpe", "glm4"};
    static const char* const kUnbounded[] = {"gpt-2", "starcoder", "refact", "jina-v2-en"};
    for (const char* p : kSingle)
        if (pre == p) return 1;
    for (const char* p : kUnbounded)
        if (pre == p) return 0;
    return 3;
}

}  // namespace

const char* chat_format_name(ChatFormat f) {
    static const char* const kNames[] = {"llama3", "chatml", "phi3", "gemma", "mistral", "deepseek", "plain"};
    const int i = (int)f;
    return i >= 0 && i < 7 ? kNames[i] : "plain";
}

// ------------------------------------------------------------ set-up

bool Tokenizer::load_vocab(const Gguf& g, std::string* err) {
    const MetaValue* toks = g.meta("tokenizer.ggml.tokens");
    if (!toks || toks->sarr.empty()) { *err = "tokenizer.ggml.tokens missing"; return false; }
    tokens_ = toks->sarr;
    index_.reserve(tokens_.size() * 2);
    for (size_t i = 0; i < tokens_.size(); ++i) index_.emplace(tokens_[i], (int32_t)i);
    const std::string model = g.str("tokenizer.ggml.model", "gpt2");
    spm_ = model == "llama";
    if (!spm_ && model != "gpt2" && model != "bpe") { *err = "unsupported tokenizer model: " + model; return false; }
    const int64_t nv = (int64_t)tokens_.size();
    auto valid_id = [&](const char* key, int32_t fallback) {
        const int64_t v = g.i64(key, fallback);
        return v >= 0 && v < nv ? (int32_t)v : fallback;
    };
    bos_ = valid_id("tokenizer.ggml.bos_token_id", spm_ ? 1 : -1);
    eos_ = valid_id("tokenizer.ggml.eos_token_id", spm_ ? 2 : -1);
    unk_ = valid_id("tokenizer.ggml.unknown_token_id", 0);
    add_bos_ = bos_ >= 0 && g.flag("tokenizer.ggml.add_bos_token", bos_ >= 0);
    space_prefix_ = g.flag("tokenizer.ggml.add_space_prefix", true);
    types_.assign(tokens_.size(), 1);
    const MetaValue* types = g.meta("tokenizer.ggml.token_type");
    if (types) std::copy_n(types->iarr.begin(), std::min(types->iarr.size(), types_.size()), types_.begin());
    scores_.clear();
    if (const MetaValue* s = g.meta("tokenizer.ggml.scores")) scores_ = s->farr;
    if (spm_ && scores_.size() != tokens_.size()) scores_.assign(tokens_.size(), 0.0f);
    // the end-of-generation set: eos, the eot / eom ids, and the usual
    // end-of-turn texts where the vocabulary has them
    if (eos_ >= 0) eog_.insert(eos_);
    for (const char* key : {"tokenizer.ggml.eot_token_id", "tokenizer.ggml.eom_token_id"}) {
        const int32_t id = valid_id(key, -1);
        if (id >= 0) eog_.insert(id);
    }
    for (const char* s : {"<|eot_id|>", "<|end_of_text|>", "<|im_end|>", "<|end|>", "<|endoftext|>", "<end_of_turn>",
                          "<|eom_id|>", "<\xEF\xBD\x9C" "end\xE2\x96\x81" "of\xE2\x96\x81" "sentence\xEF\xBD\x9C>"}) {
        const int32_t id = lookup(s);
        if (id >= 0) eog_.insert(id);
    }
    // specials: control / user-defined types, or, in a vocabulary without
    // types, every "<|...|>" text
    for (size_t i = 0; i < tokens_.size(); ++i) {
        const std::string& s = tokens_[i];
        bool special = types_[i] == 3 || types_[i] == 4;
        if (!special && !types && s.size() >= 4 && s.compare(0, 2, "<|") == 0 && s.compare(s.size() - 2, 2, "|>") == 0)
            special = true;
        if (special && !s.empty()) trie_insert(s, (int32_t)i);
    }
    // texts of every token, as decode emits them
    const ByteAlphabet& ab = byte_alphabet();
    texts_.resize(tokens_.size());
    for (size_t i = 0; i < tokens_.size(); ++i) {
        const std::string& tok = tokens_[i];
        std::string& o = texts_[i];
        const int ty = types_[i];
        if (ty == 3 || ty == 4) { o = tok; continue; }
        if (spm_) {
            if (ty == 6 && tok.size() == 6 && tok.compare(0, 3, "<0x") == 0) {
                o.assign(1, (char)std::strtol(tok.c_str() + 3, nullptr, 16));
                continue;
            }
            for (size_t k = 0; k < tok.size();) {
                if (tok.compare(k, 3, kSpaceMark) == 0) { o += ' '; k += 3; }
                else o += tok[k++];
            }
            continue;
        }
        const unsigned char* p = reinterpret_cast<const unsigned char*>(tok.data());
        for (size_t k = 0; k < tok.size();) {
            size_t len;
            const uint32_t cp = utf8_at(p + k, tok.size() - k, &len);
            auto it = ab.to_byte.find(cp);
            if (it != ab.to_byte.end()) o += (char)it->second;
            else o.append(tok, k, len);
            k += len;
        }
    }
    return true;
}

bool Tokenizer::load_merges(const Gguf& g, std::string* err) {
    if (spm_) {
        byte_ids_.assign(256, -1);
        for (int b = 0; b < 256; ++b) {
            char name[8];
            std::snprintf(name, sizeof(name), "<0x%02X>", b);
            byte_ids_[b] = lookup(name);
        }
        return true;
    }
    digits_ = digits_for(g.str("tokenizer.ggml.pre", ""));
    if (const MetaValue* m = g.meta("tokenizer.ggml.merges")) {
        ranks_.reserve(m->sarr.size() * 2);
        for (size_t r = 0; r < m->sarr.size(); ++r) {
            const std::string& line = m->sarr[r];
            const size_t cut = line.find(' ');
            if (cut == std::string::npos) continue;
            const int32_t a = lookup(line.substr(0, cut)), b = lookup(line.substr(cut + 1));
            if (a < 0 || b < 0) continue;
            std::string joined = line.substr(0, cut);
            joined.append(line, cut + 1, std::string::npos);
            const int32_t ab = lookup(joined);
            if (ab < 0) continue;
            ranks_.emplace(pair_key(a, b), MergeTo{(int)r, ab});   // the first rank of a pair counts
        }
    }
    if (ranks_.empty()) { *err = "tokenizer.ggml.merges missing for a BPE vocabulary"; return false; }
    return true;
}

void Tokenizer::detect_format(const Gguf& g) {
    const std::string tmpl = g.str("tokenizer.chat_template", "");
    auto in_template = [&](const char* s) { return s == nullptr || tmpl.find(s) != std::string::npos; };
    auto in_vocab = [&](const char* s) { return s == nullptr || lookup(s) >= 0; };
    for (const FormatMarker& m : kTemplateMarkers)
        if (in_template(m.a) && in_template(m.b)) { format_ = m.f; return; }
    for (const FormatMarker& m : kVocabMarkers)
        if (in_vocab(m.a) && in_vocab(m.b)) { format_ = m.f; return; }
    format_ = ChatFormat::Plain;
}

std::unique_ptr<Tokenizer> Tokenizer::create(const Gguf& g, std::string* err) {
    std::string e;
    std::unique_ptr<Tokenizer> t(new Tokenizer());
    if (!t->load_vocab(g, &e) || !t->load_merges(g, &e)) {
        if (err) *err = e;
        return nullptr;
    }
    t->detect_format(g);
    return t;
}

// ------------------------------------------------------------ specials trie

void Tokenizer::trie_insert(const std::string& s, int32_t id) {
    if (trie_.empty()) trie_.emplace_back();
    int node = 0;
    for (unsigned char ch : s) {
        auto it = trie_[node].next.find(ch);
        if (it == trie_[node].next.end()) {
            trie_.emplace_back();
            const int nn = (int)trie_.size() - 1;
            trie_[node].next.emplace(ch, nn);
            node = nn;
        } else {
            node = it->second;
        }
    }
    if (trie_[node].id < 0) trie_[node].id = id;   // equal texts: the first id
}

// the longest special token starting at byte i: its id and length, or -1
int32_t Tokenizer::special_at(const std::string& s, size_t i, size_t* len) const {
    if (trie_.empty()) return -1;
    int node = 0;
    int32_t best = -1;
    for (size_t k = i; k < s.size(); ++k) {
        auto it = trie_[node].next.find((unsigned char)s[k]);
        if (it == trie_[node].next.end()) break;
        node = it->second;
        if (trie_[node].id >= 0) {
            best = trie_[node].id;
            *len = k + 1 - i;
        }
    }
    return best;
}

// ------------------------------------------------------------ encoding

std::vector<std::string> Tokenizer::pre_split(const std::string& s) const {
    const std::vector<Cp> cps = decode_text(s);
    const SplitCtx x{cps, digits_};
    std::vector<std::string> pieces;
    for (size_t i = 0; i < cps.size();) {
        size_t end = 0;
        for (Rule r : kSplitRules)
            if ((end = r(x, i)) != 0) break;
        const size_t b0 = cps[i].at, b1 = end < cps.size() ? cps[end].at : s.size();
        pieces.emplace_back(s, b0, b1 - b0);
        i = end;
    }
    return pieces;
}

std::vector<int32_t> Tokenizer::encode_bpe_piece(const std::string& piece) const {
    const ByteAlphabet& ab = byte_alphabet();
    // one symbol per byte (its alphabet character); a character the
    // vocabulary lacks falls back to the alphabet tokens of its UTF-8 bytes
    std::vector<Node> sy;
    for (unsigned char b : piece) {
        const std::string& ch = ab.to_text[b];
        const int32_t id = lookup(ch);
        if (id >= 0) {
            sy.push_back({0, 0, id, 0, 0});
            continue;
        }
        for (unsigned char u : ch) {
            const int32_t bt = lookup(ab.to_text[u]);
            if (bt >= 0) sy.push_back({0, 0, bt, 0, 0});
        }
    }
    const int n = (int)sy.size();
    for (int i = 0; i < n; ++i) {
        sy[i].prev = i - 1;
        sy[i].next = i + 1 < n ? i + 1 : -1;
    }
    std::vector<uint32_t> stamp(n, 0);   // bumped when a symbol changes
    std::priority_queue<Candidate> q;
    auto offer = [&](int l, int r) {
        if (l < 0 || r < 0) return;
        auto it = ranks_.find(pair_key(sy[l].id, sy[r].id));
        if (it != ranks_.end()) q.push({(double)it->second.rank, l, r, stamp[l], stamp[r]});
    };
    for (int i = 0; i + 1 < n; ++i) offer(i, i + 1);
    while (!q.empty()) {
        const Candidate c = q.top();
        q.pop();
        if (stamp[c.left] != c.stamp_l || stamp[c.right] != c.stamp_r || sy[c.left].next != c.right) continue;
        Node& L = sy[c.left];
        Node& R = sy[c.right];
        L.id = ranks_.at(pair_key(L.id, R.id)).id;
        L.next = R.next;
        if (R.next >= 0) sy[R.next].prev = c.left;
        ++stamp[c.left];
        ++stamp[c.right];
        R.next = -2;   // removed
        offer(L.prev, c.left);
        offer(c.left, L.next);
    }
    std::vector<int32_t> out;
    for (int i = n > 0 ? 0 : -1; i >= 0; i = sy[i].next) out.push_back(sy[i].id);
    return out;
}

std::vector<int32_t> Tokenizer::encode_spm(const std::string& raw) const {
    // spaces become the word-boundary mark, with one in front when asked
    std::string text;
    text.reserve(raw.size() * 2 + 3);
    if (space_prefix_ && !raw.empty()) text += kSpaceMark;
    for (char ch : raw) {
        if (ch == ' ') text += kSpaceMark;
        else text += ch;
    }
    const std::vector<Cp> cps = decode_text(text);
    const int n = (int)cps.size();
    std::vector<Node> sy(n);
    for (int i = 0; i < n; ++i) {
        const uint32_t end = i + 1 < n ? cps[i + 1].at : (uint32_t)text.size();
        sy[i] = {i - 1, i + 1 < n ? i + 1 : -1, -1, cps[i].at, end - cps[i].at};
    }
    std::priority_queue<Candidate> q;
    auto offer = [&](int l, int r) {
        if (l < 0 || r < 0) return;
        const int32_t id = lookup(text.substr(sy[l].at, sy[l].len + sy[r].len));
        if (id < 0 || (size_t)id >= scores_.size()) return;
        q.push({-(double)scores_[id], l, r, sy[l].len, sy[r].len});   // the highest score first
    };
    for (int i = 0; i + 1 < n; ++i) offer(i, i + 1);
    while (!q.empty()) {
        const Candidate c = q.top();
        q.pop();
        Node& L = sy[c.left];
        Node& R = sy[c.right];
        if (L.len != c.stamp_l || R.len != c.stamp_r || L.next != c.right) continue;
        L.len += R.len;
        R.len = 0;
        L.next = R.next;
        if (R.next >= 0) sy[R.next].prev = c.left;
        offer(L.prev, c.left);
        offer(c.left, L.next);
    }
    std::vector<int32_t> out;
    for (int i = n > 0 ? 0 : -1; i >= 0; i = sy[i].next) {
        const std::string piece = text.substr(sy[i].at, sy[i].len);
        const int32_t id = lookup(piece);
        if (id >= 0) { out.push_back(id); continue; }
        const size_t before = out.size();
        for (unsigned char b : piece)
            if (byte_ids_[b] >= 0) out.push_back(byte_ids_[b]);
        if (out.size() == before) out.push_back(unk_);
    }
    return out;
}

std::vector<int32_t> Tokenizer::encode_plain(const std::string& text) const {
    std::vector<int32_t> ids;
    if (text.empty()) return ids;
    if (spm_) return encode_spm(text);
    for (const std::string& p : pre_split(text)) {
        const std::vector<int32_t> part = encode_bpe_piece(p);
        ids.insert(ids.end(), part.begin(), part.end());
    }
    return ids;
}

std::vector<int32_t> Tokenizer::encode(const std::string& text, bool add_bos, bool parse_special) const {
    std::vector<int32_t> ids;
    if (add_bos && bos_ >= 0) ids.push_back(bos_);
    auto plain = [&](size_t a, size_t b) {
        if (b <= a) return;
        const std::vector<int32_t> part = encode_plain(text.substr(a, b - a));
        ids.insert(ids.end(), part.begin(), part.end());
    };
    if (!parse_special) {
        plain(0, text.size());
        return ids;
    }
    // specials only start at code-point boundaries
    const unsigned char* p = reinterpret_cast<const unsigned char*>(text.data());
    size_t from = 0;
    for (size_t i = 0; i < text.size();) {
        size_t len = 0;
        const int32_t sp = special_at(text, i, &len);
        if (sp >= 0) {
            plain(from, i);
            ids.push_back(sp);
            i += len;
            from = i;
            continue;
        }
        size_t step;
        utf8_at(p + i, text.size() - i, &step);
        i += step;
    }
    plain(from, text.size());
    return ids;
}

std::string Tokenizer::token_text(int32_t id) const {
    return id >= 0 && (size_t)id < texts_.size() ? texts_[id] : std::string();
}

std::string Tokenizer::decode(const std::vector<int32_t>& ids) const {
    std::string o;
    for (int32_t id : ids) o += token_text(id);
    if (spm_ && space_prefix_ && !o.empty() && o[0] == ' ') o.erase(0, 1);
    return o;
}

// ------------------------------------------------------------ chat

std::vector<std::pair<std::string, bool>> Tokenizer::chat_parts(const Messages& msgs, ChatFormat f) const {
    std::vector<std::pair<std::string, bool>> parts;
    const ChatBuilder b{parts};
    const std::string eos_text = eos_ >= 0 ? tokens_[eos_] : std::string();
    if (f == ChatFormat::Llama3) {
        for (const auto& [role, content] : msgs) {
            b.tag("<|start_header_id|>" + (role == "tool" ? std::string("ipython") : role) + "<|end_header_id|>\n\n");
            b.text(content);
            b.tag("<|eot_id|>");
        }
        b.tag("<|start_header_id|>assistant<|end_header_id|>\n\n");
    } else if (f == ChatFormat::ChatML) {
        for (const auto& [role, content] : msgs) {
            const bool tool = role == "tool";
            b.tag("<|im_start|>" + (tool ? std::string("user") : role) + "\n");
            b.text(tool ? "<tool_response>\n" + content + "\n</tool_response>" : content);
            b.tag("<|im_end|>\n");
        }
        b.tag("<|im_start|>assistant\n");
    } else if (f == ChatFormat::Phi3) {
        for (const auto& [role, content] : msgs) {
            b.tag("<|" + (role == "tool" ? std::string("user") : role) + "|>\n");
            b.text(content);
            b.tag("<|end|>\n");
        }
        b.tag("<|assistant|>\n");
    } else if (f == ChatFormat::Gemma) {
        // system text joins the next user turn
        std::string system;
        for (const auto& [role, content] : msgs) {
            if (role == "system") {
                if (!system.empty()) system += "\n";
                system += content;
                continue;
            }
            const bool model = role == "assistant";
            b.tag(model ? "<start_of_turn>model\n" : "<start_of_turn>user\n");
            if (!model && !system.empty()) {
                b.text(system + "\n\n");
                system.clear();
            }
            b.text(content);
            b.tag("<end_of_turn>\n");
        }
        b.tag("<start_of_turn>model\n");
    } else if (f == ChatFormat::Mistral) {
        std::string system;
        for (const auto& [role, content] : msgs) {
            if (role == "system") {
                if (!system.empty()) system += "\n";
                system += content;
            } else if (role == "assistant") {
                b.text(" " + content);
                b.tag(eos_ >= 0 ? eos_text : std::string("</s>"));
            } else {
                b.tag("[INST]");
                b.text(" " + (system.empty() ? std::string() : system + "\n\n") + content + " ");
                system.clear();
                b.tag("[/INST]");
            }
        }
    } else if (f == ChatFormat::DeepSeek) {
        const std::string user = "<\xEF\xBD\x9C" "User\xEF\xBD\x9C>", assistant = "<\xEF\xBD\x9C" "Assistant\xEF\xBD\x9C>";
        for (const auto& [role, content] : msgs) {
            if (role == "system") {
                b.text(content);
            } else if (role == "assistant") {
                b.tag(assistant);
                b.text(content);
                b.tag(eos_text);
            } else {
                b.tag(user);
                b.text(content);
            }
        }
        b.tag(assistant);
    } else {
        // plain: "Role: text" paragraphs, then the assistant's cue
        for (const auto& [role, content] : msgs) {
            std::string r = role;
            if (!r.empty() && r[0] >= 'a' && r[0] <= 'z') r[0] = (char)(r[0] - 'a' + 'A');
            b.text(r + ": " + content + "\n\n");
        }
        b.text("Assistant:");
    }
    return parts;
}

std::vector<int32_t> Tokenizer::encode_chat(const Messages& msgs) const {
    std::vector<int32_t> ids;
    if (add_bos_ && bos_ >= 0) ids.push_back(bos_);
    for (const auto& [text, special] : chat_parts(msgs, format_)) {
        const std::vector<int32_t> part = encode(text, false, special);
        ids.insert(ids.end(), part.begin(), part.end());
    }
    return ids;
}

std::string Tokenizer::apply_chat(const Messages& msgs, ChatFormat f) const {
    std::string o;
    if (add_bos_ && bos_ >= 0 && f != ChatFormat::Plain) o += tokens_[bos_];
    for (const auto& part : chat_parts(msgs, f)) o += part.first;
    return o;
}

}  // namespace fb
