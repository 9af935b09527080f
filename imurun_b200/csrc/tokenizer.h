// tokenizer.h — GGUF-vocabulary tokenizer and chat templates (host code).
//
// Produces the same ids as the reference tokenizer (model/fish/src/
// tokenizer.cpp) so the FISH ABI's tokenise / chat / prefix-cache behaviour is
// unchanged: SentencePiece score merges with <0xNN> byte fallback, byte-level
// BPE with rank merges after the llama3 / qwen2 / gpt2 pre-split, special
// tokens matched longest-first only when allowed, structural chat templates.
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <utility>
#include <vector>

#include "gguf.h"

namespace fb {

enum class ChatFormat { Llama3, ChatML, Phi3, Gemma, Mistral, DeepSeek, Plain };
const char* chat_format_name(ChatFormat f);

using Messages = std::vector<std::pair<std::string, std::string>>;

class Tokenizer {
public:
    static std::unique_ptr<Tokenizer> create(const Gguf& g, std::string* err);
    std::vector<int32_t> encode(const std::string& text, bool add_bos, bool parse_special = true) const;
    std::vector<int32_t> encode_chat(const Messages& msgs) const;
    std::string apply_chat(const Messages& msgs, ChatFormat f) const;
    std::string token_text(int32_t id) const;
    std::string decode(const std::vector<int32_t>& ids) const;
    bool is_eog(int32_t id) const { return eog_.count(id) != 0; }
    ChatFormat format() const { return format_; }
    bool spm() const { return spm_; }
    int32_t bos() const { return bos_; }
    int32_t eos() const { return eos_; }
    size_t size() const { return tokens_.size(); }

private:
    struct Seg { std::string text; bool special; };
    std::vector<Seg> chat_segments(const Messages& msgs, ChatFormat f) const;
    std::vector<int32_t> encode_plain(const std::string& text) const;
    std::vector<int32_t> encode_spm(const std::string& text) const;
    std::vector<int32_t> encode_bpe_piece(const std::string& piece) const;
    std::vector<std::string> pre_split(const std::string& text) const;
    int32_t id_of(const std::string& s) const {
        auto it = index_.find(s);
        return it == index_.end() ? -1 : it->second;
    }

    bool spm_ = false;
    std::vector<std::string> tokens_;
    std::vector<int32_t> types_;
    std::vector<float> scores_;
    std::unordered_map<std::string, int32_t> index_;
    std::unordered_map<uint64_t, std::pair<int, int32_t>> merges_;   // (a<<32|b) -> (rank, id)
    std::vector<std::pair<std::string, int32_t>> specials_;          // longest first
    std::unordered_set<int32_t> eog_;
    std::vector<int32_t> byte_ids_;
    int32_t bos_ = 1, eos_ = 2, unk_ = 0;
    bool add_bos_ = true, space_prefix_ = true;
    int digits_ = 3;
    ChatFormat format_ = ChatFormat::Plain;
};

}  // namespace fb
