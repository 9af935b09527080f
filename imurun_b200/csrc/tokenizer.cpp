// tokenizer.cpp — see tokenizer.h. The algorithms (and the character classes
// they depend on) restate the reference's so the ids are identical:
// create (tokenizer.cpp:156-292), pre-split (294-415), BPE merges (419-465),
// SentencePiece (469-563), encode with specials (567-613), token_text /
// decode (617-665), chat segments (669-792).
#include "tokenizer.h"

#include <algorithm>
#include <climits>
#include <cstring>
#include <queue>

namespace fb {

namespace {

const char* kSpace = "\xE2\x96\x81";   // U+2581

// Next code point of s at i (advances i); malformed bytes count as one unit.
uint32_t cp_at(const std::string& s, size_t& i) {
    if (i >= s.size()) return 0;
    const unsigned char c = static_cast<unsigned char>(s[i]);
    int len = c < 0x80 ? 1 : (c & 0xE0) == 0xC0 ? 2 : (c & 0xF0) == 0xE0 ? 3 : (c & 0xF8) == 0xF0 ? 4 : 1;
    if (len == 1) { ++i; return c; }
    if (i + (size_t)len > s.size()) { ++i; return c; }
    uint32_t v = c & (0xFFu >> (len + 1));
    for (int k = 1; k < len; ++k) v = (v << 6) | (static_cast<unsigned char>(s[i + k]) & 0x3Fu);
    i += (size_t)len;
    return v;
}

void put_utf8(std::string& o, uint32_t cp) {
    if (cp < 0x80) o += (char)cp;
    else if (cp < 0x800) { o += (char)(0xC0 | (cp >> 6)); o += (char)(0x80 | (cp & 0x3F)); }
    else if (cp < 0x10000) { o += (char)(0xE0 | (cp >> 12)); o += (char)(0x80 | ((cp >> 6) & 0x3F)); o += (char)(0x80 | (cp & 0x3F)); }
    else { o += (char)(0xF0 | (cp >> 18)); o += (char)(0x80 | ((cp >> 12) & 0x3F)); o += (char)(0x80 | ((cp >> 6) & 0x3F)); o += (char)(0x80 | (cp & 0x3F)); }
}

// GPT-2 byte <-> printable code point alphabet.
struct Alphabet {
    std::string enc[256];
    std::unordered_map<uint32_t, uint8_t> dec;
    Alphabet() {
        int extra = 0;
        for (int b = 0; b < 256; ++b) {
            const bool printable = (b >= '!' && b <= '~') || (b >= 0xA1 && b <= 0xAC) || (b >= 0xAE && b <= 0xFF);
            const uint32_t cp = printable ? (uint32_t)b : (uint32_t)(256 + extra++);
            put_utf8(enc[b], cp);
            dec[cp] = (uint8_t)b;
        }
    }
};
const Alphabet& alphabet() { static const Alphabet a; return a; }

bool is_space(uint32_t c) {
    return c == ' ' || c == '\t' || c == '\n' || c == '\r' || c == '\f' || c == '\v' || c == 0x85 || c == 0xA0 ||
           c == 0x1680 || (c >= 0x2000 && c <= 0x200A) || c == 0x2028 || c == 0x2029 || c == 0x202F ||
           c == 0x205F || c == 0x3000;
}

bool is_digit(uint32_t c) {
    return (c >= '0' && c <= '9') || (c >= 0x0660 && c <= 0x0669) || (c >= 0x06F0 && c <= 0x06F9) ||
           (c >= 0x0966 && c <= 0x096F) || (c >= 0x09E6 && c <= 0x09EF) || (c >= 0xFF10 && c <= 0xFF19) ||
           c == 0xB2 || c == 0xB3 || c == 0xB9 || (c >= 0xBC && c <= 0xBE);
}

bool is_letter(uint32_t c) {
    if ((c >= 'a' && c <= 'z') || (c >= 'A' && c <= 'Z')) return true;
    if (c < 0x80) return false;
    if (c < 0xC0) return c == 0xAA || c == 0xB5 || c == 0xBA;
    if (c == 0xD7 || c == 0xF7) return false;
    if (is_digit(c)) return false;
    if (c >= 0x2000 && c <= 0x2BFF) return false;
    if (c >= 0x3000 && c <= 0x303F) return false;
    if (c >= 0xFE00 && c <= 0xFE0F) return false;
    if (c >= 0xFF00 && c <= 0xFF20) return false;
    if (c >= 0x1F000 && c <= 0x1FAFF) return false;
    if (c >= 0xE000 && c <= 0xF8FF) return false;
    return true;
}

char lower(char c) { return (c >= 'A' && c <= 'Z') ? (char)(c + 32) : c; }

}  // namespace

const char* chat_format_name(ChatFormat f) {
    switch (f) {
        case ChatFormat::Llama3: return "llama3";
        case ChatFormat::ChatML: return "chatml";
        case ChatFormat::Phi3: return "phi3";
        case ChatFormat::Gemma: return "gemma";
        case ChatFormat::Mistral: return "mistral";
        case ChatFormat::DeepSeek: return "deepseek";
        default: return "plain";
    }
}

std::unique_ptr<Tokenizer> Tokenizer::create(const Gguf& g, std::string* err) {
    auto fail = [&](const std::string& w) -> std::unique_ptr<Tokenizer> { if (err) *err = w; return nullptr; };
    const MetaValue* toks = g.meta("tokenizer.ggml.tokens");
    if (!toks || toks->sarr.empty()) return fail("tokenizer.ggml.tokens missing");
    std::unique_ptr<Tokenizer> t(new Tokenizer());
    t->tokens_ = toks->sarr;
    t->index_.reserve(t->tokens_.size() * 2);
    for (size_t i = 0; i < t->tokens_.size(); ++i) t->index_.emplace(t->tokens_[i], (int32_t)i);
    const std::string model = g.str("tokenizer.ggml.model", "gpt2");
    if (model == "llama") t->spm_ = true;
    else if (model != "gpt2" && model != "bpe") return fail("unsupported tokenizer model: " + model);
    const int64_t nv = (int64_t)t->tokens_.size();
    auto id_key = [&](const char* key, int32_t def) {
        const int64_t v = g.i64(key, def);
        return (v >= 0 && v < nv) ? (int32_t)v : def;
    };
    t->bos_ = id_key("tokenizer.ggml.bos_token_id", t->spm_ ? 1 : -1);
    t->eos_ = id_key("tokenizer.ggml.eos_token_id", t->spm_ ? 2 : -1);
    t->unk_ = id_key("tokenizer.ggml.unknown_token_id", 0);
    t->add_bos_ = g.flag("tokenizer.ggml.add_bos_token", t->bos_ >= 0);
    if (t->bos_ < 0) t->add_bos_ = false;
    t->space_prefix_ = g.flag("tokenizer.ggml.add_space_prefix", true);
    if (t->eos_ >= 0) t->eog_.insert(t->eos_);
    for (const char* key : {"tokenizer.ggml.eot_token_id", "tokenizer.ggml.eom_token_id"}) {
        const int32_t id = id_key(key, -1);
        if (id >= 0) t->eog_.insert(id);
    }
    for (const char* s : {"<|eot_id|>", "<|end_of_text|>", "<|im_end|>", "<|end|>", "<|endoftext|>", "<end_of_turn>",
                          "<|eom_id|>", "<\xEF\xBD\x9C" "end\xE2\x96\x81" "of\xE2\x96\x81" "sentence\xEF\xBD\x9C>"}) {
        const int32_t id = t->id_of(s);
        if (id >= 0) t->eog_.insert(id);
    }
    const std::string pre = g.str("tokenizer.ggml.pre", "");
    if (pre == "qwen2" || pre == "qwen35" || pre == "deepseek-llm" || pre == "deepseek-coder" || pre == "deepseek-v3" ||
        pre == "stablelm2" || pre == "command-r" || pre == "olmo" || pre == "dbrx" || pre == "chatglm-bpe" || pre == "glm4")
        t->digits_ = 1;
    else if (pre == "gpt-2" || pre == "starcoder" || pre == "refact" || pre == "jina-v2-en")
        t->digits_ = 0;
    else
        t->digits_ = 3;
    if (const MetaValue* m = g.meta("tokenizer.ggml.merges")) {
        t->merges_.reserve(m->sarr.size() * 2);
        for (size_t rank = 0; rank < m->sarr.size(); ++rank) {
            const std::string& line = m->sarr[rank];
            const size_t sp = line.find(' ');
            if (sp == std::string::npos) continue;
            const std::string a = line.substr(0, sp), b = line.substr(sp + 1);
            const int32_t ia = t->id_of(a), ib = t->id_of(b), iab = t->id_of(a + b);
            if (ia < 0 || ib < 0 || iab < 0) continue;
            const uint64_t key = ((uint64_t)(uint32_t)ia << 32) | (uint32_t)ib;
            t->merges_.emplace(key, std::make_pair((int)rank, iab));
        }
    }
    if (!t->spm_ && t->merges_.empty()) return fail("tokenizer.ggml.merges missing for a BPE vocabulary");
    if (const MetaValue* s = g.meta("tokenizer.ggml.scores")) t->scores_ = s->farr;
    if (t->spm_ && t->scores_.size() != t->tokens_.size()) t->scores_.assign(t->tokens_.size(), 0.0f);
    const MetaValue* types = g.meta("tokenizer.ggml.token_type");
    t->types_.assign(t->tokens_.size(), 1);
    if (types)
        for (size_t i = 0; i < t->tokens_.size() && i < types->iarr.size(); ++i) t->types_[i] = types->iarr[i];
    for (size_t i = 0; i < t->tokens_.size(); ++i) {
        bool special = t->types_[i] == 3 || t->types_[i] == 4;
        const std::string& s = t->tokens_[i];
        if (!special && !types && s.size() >= 4 && s[0] == '<' && s[1] == '|' && s.back() == '>' && s[s.size() - 2] == '|')
            special = true;
        if (special && !s.empty()) t->specials_.emplace_back(s, (int32_t)i);
    }
    std::stable_sort(t->specials_.begin(), t->specials_.end(),
                     [](const auto& a, const auto& b) { return a.first.size() > b.first.size(); });
    if (t->spm_) {
        t->byte_ids_.assign(256, -1);
        char name[8];
        for (int b = 0; b < 256; ++b) {
            std::snprintf(name, sizeof(name), "<0x%02X>", b);
            t->byte_ids_[b] = t->id_of(name);
        }
    }
    const std::string tmpl = g.str("tokenizer.chat_template", "");
    auto in = [&](const char* s) { return tmpl.find(s) != std::string::npos; };
    auto has = [&](const char* s) { return t->id_of(s) >= 0; };
    if (in("<|start_header_id|>")) t->format_ = ChatFormat::Llama3;
    else if (in("<|im_start|>")) t->format_ = ChatFormat::ChatML;
    else if (in("<start_of_turn>")) t->format_ = ChatFormat::Gemma;
    else if (in("<|user|>") && in("<|end|>")) t->format_ = ChatFormat::Phi3;
    else if (in("User\xEF\xBD\x9C>")) t->format_ = ChatFormat::DeepSeek;
    else if (in("[INST]")) t->format_ = ChatFormat::Mistral;
    else if (has("<|start_header_id|>") && has("<|end_header_id|>")) t->format_ = ChatFormat::Llama3;
    else if (has("<|im_start|>")) t->format_ = ChatFormat::ChatML;
    else if (has("<|user|>") && has("<|end|>")) t->format_ = ChatFormat::Phi3;
    else if (has("<start_of_turn>")) t->format_ = ChatFormat::Gemma;
    else if (has("<\xEF\xBD\x9C" "User\xEF\xBD\x9C>")) t->format_ = ChatFormat::DeepSeek;
    else if (has("[INST]")) t->format_ = ChatFormat::Mistral;
    else t->format_ = ChatFormat::Plain;
    return t;
}

// Pieces of `text` under the byte-level BPE pre-tokenizer: contractions,
// optional non-letter + letters, digit groups, optional space + punctuation
// run + newlines, whitespace runs (newline-terminated, or leaving the last
// space for the next word), else one code point.
std::vector<std::string> Tokenizer::pre_split(const std::string& s) const {
    std::vector<std::string> out;
    const size_t n = s.size();
    size_t i = 0;
    auto emit = [&](size_t a, size_t b) { if (b > a) out.push_back(s.substr(a, b - a)); };
    auto run_while = [&](size_t from, bool (*pred)(uint32_t)) {
        size_t e = from;
        while (e < n) {
            size_t r = e;
            if (!pred(cp_at(s, r))) break;
            e = r;
        }
        return e;
    };
    while (i < n) {
        size_t nx = i;
        const uint32_t c = cp_at(s, nx);
        if (c == '\'') {
            static const char* kc[] = {"'s", "'t", "'re", "'ve", "'m", "'ll", "'d"};
            bool hit = false;
            for (const char* w : kc) {
                const size_t L = std::strlen(w);
                if (i + L > n) continue;
                bool eq = true;
                for (size_t k = 0; k < L; ++k) if (lower(s[i + k]) != lower(w[k])) { eq = false; break; }
                if (eq) { emit(i, i + L); i += L; hit = true; break; }
            }
            if (hit) continue;
        }
        if (is_letter(c)) {
            const size_t e = run_while(i, is_letter);
            emit(i, e);
            i = e;
            continue;
        }
        if (c != '\r' && c != '\n' && !is_digit(c) && nx < n) {
            size_t r = nx;
            if (is_letter(cp_at(s, r))) {
                const size_t e = run_while(nx, is_letter);
                emit(i, e);
                i = e;
                continue;
            }
        }
        if (is_digit(c)) {
            size_t e = i;
            int cnt = 0;
            while (e < n && (digits_ == 0 || cnt < digits_)) {
                size_t r = e;
                if (!is_digit(cp_at(s, r))) break;
                e = r;
                ++cnt;
            }
            emit(i, e);
            i = e;
            continue;
        }
        {
            size_t st = i;
            if (c == ' ') st = nx;
            if (st < n) {
                size_t r = st;
                const uint32_t cc = cp_at(s, r);
                if (!is_space(cc) && !is_letter(cc) && !is_digit(cc)) {
                    size_t e = st;
                    while (e < n) {
                        size_t q = e;
                        const uint32_t x = cp_at(s, q);
                        if (is_space(x) || is_letter(x) || is_digit(x)) break;
                        e = q;
                    }
                    while (e < n) {
                        size_t q = e;
                        const uint32_t x = cp_at(s, q);
                        if (x != '\r' && x != '\n') break;
                        e = q;
                    }
                    emit(i, e);
                    i = e;
                    continue;
                }
            }
        }
        if (is_space(c)) {
            size_t e = i, last_ws = i, last_nl = 0;
            while (e < n) {
                size_t q = e;
                const uint32_t x = cp_at(s, q);
                if (!is_space(x)) break;
                if (x == '\n' || x == '\r') last_nl = q;
                last_ws = e;
                e = q;
            }
            if (last_nl > 0) { emit(i, last_nl); i = last_nl; }
            else if (e < n && last_ws > i) { emit(i, last_ws); i = last_ws; }
            else { emit(i, e); i = e; }
            continue;
        }
        emit(i, nx);
        i = nx;
    }
    return out;
}

std::vector<int32_t> Tokenizer::encode_bpe_piece(const std::string& pre) const {
    const Alphabet& ab = alphabet();
    std::string enc;
    for (unsigned char b : pre) enc += ab.enc[b];
    std::vector<int32_t> sym;
    size_t i = 0;
    while (i < enc.size()) {
        size_t j = i;
        cp_at(enc, j);
        const int32_t id = id_of(enc.substr(i, j - i));
        if (id >= 0) sym.push_back(id);
        else
            for (size_t k = i; k < j; ++k) {
                const int32_t bt = id_of(ab.enc[(unsigned char)enc[k]]);
                if (bt >= 0) sym.push_back(bt);
            }
        i = j;
    }
    while (sym.size() > 1) {
        int best = INT_MAX;
        size_t at = sym.size();
        int32_t mid = -1;
        for (size_t k = 0; k + 1 < sym.size(); ++k) {
            auto it = merges_.find(((uint64_t)(uint32_t)sym[k] << 32) | (uint32_t)sym[k + 1]);
            if (it != merges_.end() && it->second.first < best) { best = it->second.first; at = k; mid = it->second.second; }
        }
        if (at == sym.size()) break;
        sym[at] = mid;
        sym.erase(sym.begin() + (long)at + 1);
    }
    return sym;
}

std::vector<int32_t> Tokenizer::encode_spm(const std::string& raw) const {
    std::string text;
    if (space_prefix_ && !raw.empty()) text += kSpace;
    for (char ch : raw) {
        if (ch == ' ') text += kSpace;
        else text += ch;
    }
    struct Sym { int prev, next; size_t off, len; };
    std::vector<Sym> sy;
    for (size_t i = 0; i < text.size();) {
        size_t j = i;
        cp_at(text, j);
        sy.push_back({(int)sy.size() - 1, j < text.size() ? (int)sy.size() + 1 : -1, i, j - i});
        i = j;
    }
    std::vector<int32_t> out;
    if (sy.empty()) return out;
    struct Bi { int l, r; float score; size_t size; };
    auto lower_prio = [](const Bi& a, const Bi& b) {
        if (a.score != b.score) return a.score < b.score;
        return a.l > b.l;
    };
    std::priority_queue<Bi, std::vector<Bi>, decltype(lower_prio)> heap(lower_prio);
    auto push = [&](int l, int r) {
        if (l < 0 || r < 0) return;
        const int32_t id = id_of(text.substr(sy[l].off, sy[l].len + sy[r].len));
        if (id < 0 || (size_t)id >= scores_.size()) return;
        heap.push({l, r, scores_[id], sy[l].len + sy[r].len});
    };
    for (size_t i = 1; i < sy.size(); ++i) push((int)i - 1, (int)i);
    while (!heap.empty()) {
        const Bi b = heap.top();
        heap.pop();
        Sym& L = sy[b.l];
        Sym& R = sy[b.r];
        if (L.len == 0 || R.len == 0 || L.len + R.len != b.size) continue;
        L.len += R.len;
        R.len = 0;
        L.next = R.next;
        if (R.next >= 0) sy[R.next].prev = b.l;
        push(L.prev, b.l);
        push(b.l, L.next);
    }
    for (int i = 0; i >= 0; i = sy[i].next) {
        const Sym& s = sy[i];
        if (s.len == 0) continue;
        const std::string piece = text.substr(s.off, s.len);
        const int32_t id = id_of(piece);
        if (id >= 0) { out.push_back(id); continue; }
        bool any = false;
        for (unsigned char b : piece) {
            const int32_t bt = byte_ids_[b];
            if (bt >= 0) { out.push_back(bt); any = true; }
        }
        if (!any) out.push_back(unk_);
    }
    return out;
}

std::vector<int32_t> Tokenizer::encode_plain(const std::string& text) const {
    if (text.empty()) return {};
    if (spm_) return encode_spm(text);
    std::vector<int32_t> ids;
    for (const std::string& p : pre_split(text)) {
        const auto part = encode_bpe_piece(p);
        ids.insert(ids.end(), part.begin(), part.end());
    }
    return ids;
}

std::vector<int32_t> Tokenizer::encode(const std::string& text, bool add_bos, bool parse_special) const {
    std::vector<int32_t> ids;
    if (add_bos && bos_ >= 0) ids.push_back(bos_);
    if (!parse_special) {
        const auto part = encode_plain(text);
        ids.insert(ids.end(), part.begin(), part.end());
        return ids;
    }
    size_t i = 0, from = 0;
    while (i < text.size()) {
        bool hit = false;
        for (const auto& sp : specials_) {
            if (i + sp.first.size() > text.size() || text.compare(i, sp.first.size(), sp.first) != 0) continue;
            if (i > from) {
                const auto part = encode_plain(text.substr(from, i - from));
                ids.insert(ids.end(), part.begin(), part.end());
            }
            ids.push_back(sp.second);
            i += sp.first.size();
            from = i;
            hit = true;
            break;
        }
        if (!hit) cp_at(text, i);
    }
    if (from < text.size()) {
        const auto part = encode_plain(text.substr(from));
        ids.insert(ids.end(), part.begin(), part.end());
    }
    return ids;
}

std::string Tokenizer::token_text(int32_t id) const {
    if (id < 0 || (size_t)id >= tokens_.size()) return {};
    const std::string& tok = tokens_[id];
    const int ty = types_[id];
    if (spm_) {
        if (ty == 6 && tok.size() == 6 && tok[0] == '<' && tok[1] == '0' && tok[2] == 'x')
            return std::string(1, (char)std::strtol(tok.c_str() + 3, nullptr, 16));
        if (ty == 3 || ty == 4) return tok;
        std::string o;
        for (size_t i = 0; i < tok.size();) {
            if (tok.compare(i, 3, kSpace) == 0) { o += ' '; i += 3; }
            else o += tok[i++];
        }
        return o;
    }
    if (ty == 3 || ty == 4) return tok;
    const Alphabet& ab = alphabet();
    std::string o;
    for (size_t i = 0; i < tok.size();) {
        const size_t st = i;
        const uint32_t cp = cp_at(tok, i);
        auto it = ab.dec.find(cp);
        if (it != ab.dec.end()) o += (char)it->second;
        else o.append(tok, st, i - st);
    }
    return o;
}

std::string Tokenizer::decode(const std::vector<int32_t>& ids) const {
    std::string o;
    for (int32_t id : ids) o += token_text(id);
    if (spm_ && space_prefix_ && !o.empty() && o[0] == ' ') o.erase(0, 1);
    return o;
}

std::vector<Tokenizer::Seg> Tokenizer::chat_segments(const Messages& msgs, ChatFormat f) const {
    std::vector<Seg> sg;
    auto T = [&](const std::string& s) { if (!s.empty()) sg.push_back({s, true}); };
    auto C = [&](const std::string& s) { if (!s.empty()) sg.push_back({s, false}); };
    const std::string eos_text = eos_ >= 0 ? tokens_[eos_] : std::string();
    switch (f) {
        case ChatFormat::Llama3:
            for (const auto& m : msgs) {
                T("<|start_header_id|>" + (m.first == "tool" ? std::string("ipython") : m.first) + "<|end_header_id|>\n\n");
                C(m.second);
                T("<|eot_id|>");
            }
            T("<|start_header_id|>assistant<|end_header_id|>\n\n");
            break;
        case ChatFormat::ChatML:
            for (const auto& m : msgs) {
                if (m.first == "tool") {
                    T("<|im_start|>user\n");
                    C("<tool_response>\n" + m.second + "\n</tool_response>");
                    T("<|im_end|>\n");
                    continue;
                }
                T("<|im_start|>" + m.first + "\n");
                C(m.second);
                T("<|im_end|>\n");
            }
            T("<|im_start|>assistant\n");
            break;
        case ChatFormat::Phi3:
            for (const auto& m : msgs) {
                T("<|" + (m.first == "tool" ? std::string("user") : m.first) + "|>\n");
                C(m.second);
                T("<|end|>\n");
            }
            T("<|assistant|>\n");
            break;
        case ChatFormat::Gemma: {
            std::string sys;
            for (const auto& m : msgs) {
                if (m.first == "system") { sys += (sys.empty() ? "" : "\n") + m.second; continue; }
                const std::string role = m.first == "assistant" ? "model" : "user";
                T("<start_of_turn>" + role + "\n");
                if (!sys.empty() && role == "user") { C(sys + "\n\n"); sys.clear(); }
                C(m.second);
                T("<end_of_turn>\n");
            }
            T("<start_of_turn>model\n");
            break;
        }
        case ChatFormat::Mistral: {
            std::string sys;
            for (const auto& m : msgs) {
                if (m.first == "system") sys += (sys.empty() ? "" : "\n") + m.second;
                else if (m.first == "assistant") { C(" " + m.second); T(eos_ >= 0 ? eos_text : "</s>"); }
                else {
                    T("[INST]");
                    C(" " + (sys.empty() ? "" : sys + "\n\n") + m.second + " ");
                    sys.clear();
                    T("[/INST]");
                }
            }
            break;
        }
        case ChatFormat::DeepSeek: {
            const std::string ut = "<\xEF\xBD\x9C" "User\xEF\xBD\x9C>", at = "<\xEF\xBD\x9C" "Assistant\xEF\xBD\x9C>";
            for (const auto& m : msgs) {
                if (m.first == "system") { C(m.second); continue; }
                if (m.first == "assistant") { T(at); C(m.second); T(eos_text); }
                else { T(ut); C(m.second); }
            }
            T(at);
            break;
        }
        default:
            for (const auto& m : msgs) {
                std::string role = m.first;
                if (!role.empty() && role[0] >= 'a' && role[0] <= 'z') role[0] = (char)(role[0] - 32);
                C(role + ": " + m.second + "\n\n");
            }
            C("Assistant:");
            break;
    }
    return sg;
}

std::vector<int32_t> Tokenizer::encode_chat(const Messages& msgs) const {
    std::vector<int32_t> ids;
    if (add_bos_ && bos_ >= 0) ids.push_back(bos_);
    for (const Seg& s : chat_segments(msgs, format_)) {
        const auto part = encode(s.text, false, s.special);
        ids.insert(ids.end(), part.begin(), part.end());
    }
    return ids;
}

std::string Tokenizer::apply_chat(const Messages& msgs, ChatFormat f) const {
    std::string o;
    if (add_bos_ && bos_ >= 0 && f != ChatFormat::Plain) o += tokens_[bos_];
    for (const Seg& s : chat_segments(msgs, f)) o += s.text;
    return o;
}

}  // namespace fb
