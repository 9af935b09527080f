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
    struct MergeTo {
        int rank;
        int32_t id;
    };
    struct TrieNode {
        std::unordered_map<unsigned char, int> next;
        int32_t id = -1;
    };
    static uint64_t pair_key(int32_t a, int32_t b) { return ((uint64_t)(uint32_t)a << 32) | (uint32_t)b; }
    int32_t lookup(const std::string& s) const {
        auto it = index_.find(s);
        return it == index_.end() ? -1 : it->second;
    }
    bool load_vocab(const Gguf& g, std::string* err);
    bool load_merges(const Gguf& g, std::string* err);
    void detect_format(const Gguf& g);
    void trie_insert(const std::string& s, int32_t id);
    int32_t special_at(const std::string& s, size_t i, size_t* len) const;
    std::vector<std::pair<std::string, bool>> chat_parts(const Messages& msgs, ChatFormat f) const;
    std::vector<int32_t> encode_plain(const std::string& text) const;
    std::vector<int32_t> encode_spm(const std::string& text) const;
    std::vector<int32_t> encode_bpe_piece(const std::string& piece) const;
    std::vector<std::string> pre_split(const std::string& text) const;

    bool spm_ = false;
    std::vector<std::string> tokens_;
    std::vector<std::string> texts_;       // decoded text of every token
    std::vector<int32_t> types_;
    std::vector<float> scores_;
    std::unordered_map<std::string, int32_t> index_;
    std::unordered_map<uint64_t, MergeTo> ranks_;   // (left id, right id) -> merge rank and result
    std::vector<TrieNode> trie_;                    // special tokens
    std::unordered_set<int32_t> eog_;
    std::vector<int32_t> byte_ids_;                 // SPM <0xNN> tokens
    int32_t bos_ = 1, eos_ = 2, unk_ = 0;
    bool add_bos_ = true, space_prefix_ = true;
    int digits_ = 3;
    ChatFormat format_ = ChatFormat::Plain;
};

}  // namespace fb
