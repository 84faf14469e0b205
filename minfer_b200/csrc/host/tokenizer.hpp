// Qwen3 byte-level BPE tokenizer and chat template for the host runtime, with
// the reference's behaviour (include/minfer/models/qwen3/tokenizer.hpp,
// src/models/qwen3/tokenizer.cpp):
// * vocabulary strings are raw bytes (the byte form the reference's GGUF
//   converter writes); token types 3 (control) and 4 (user defined) are
//   special tokens, matched in the text before any other splitting;
// * the text between special tokens is pre-split by the reference's PCRE2
//   pattern (tokenizer.cpp:142), here a hand-written scanner with the same
//   alternatives, possessive quantifiers and end-of-segment anchor;
// * each piece is BPE-encoded by applying the merge rules in rank order, every
//   rule once, left to right (tokenizer.cpp:228-289);
// * decode concatenates the vocabulary strings; unused tokens (type 5) decode
//   as "<UNK>" (tokenizer.cpp:64-87);
// * apply_chat_template renders the GGUF's Jinja chat template
//   (tokenizer.cpp:291-335) with the template engine in chat_template.hpp.
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

namespace minfer {

class GGUFFile;
class ChatTemplate;

class Qwen3Tokenizer {
public:
    // BaseTokenizer::Message / Tool (include/minfer/base/tokenizer.hpp:13-27)
    struct Message {
        std::string role;
        std::string content;
        std::string reasoning_content;
        std::vector<std::pair<std::string, std::string>> tool_calls;  // name, arguments (JSON text)
    };
    struct Tool {
        std::string name;
        std::string description;
        std::string parameters;  // JSON text
    };

    static constexpr uint32_t CONTROL_TOKEN = 3;
    static constexpr uint32_t USER_DEFINED_TOKEN = 4;
    static constexpr uint32_t UNUSED_TOKEN = 5;

    // Throws std::invalid_argument when tokens and token_types differ in
    // length, or a merge rule has no space (tokenizer.cpp:28-30,124-128).
    Qwen3Tokenizer(const std::vector<std::string>& tokens, const std::vector<std::string>& merges,
                   const std::vector<uint32_t>& token_types, const std::string& chat_template, uint32_t eos_id,
                   uint32_t pad_id);
    ~Qwen3Tokenizer();
    // From the tokenizer.ggml.{tokens, merges, token_type, eos_token_id,
    // padding_token_id} and tokenizer.chat_template keys of a GGUF file.
    static std::unique_ptr<Qwen3Tokenizer> from_gguf(const GGUFFile& f);

    // Throws std::runtime_error when a piece needs a byte or merged string
    // that is not in the vocabulary (tokenizer.cpp:243-245,282-284).
    std::vector<uint32_t> encode(const std::string& text) const;
    std::string decode(const std::vector<uint32_t>& ids) const;
    std::string decode_token(uint32_t id) const;  // std::out_of_range past the vocabulary
    std::string apply_chat_template(const std::vector<Message>& messages, const std::vector<Tool>& tools = {},
                                    bool add_generation_prompt = true) const;
    // The same, with messages and tools given as JSON arrays (the shape
    // apply_chat_template builds from Message/Tool, tokenizer.cpp:296-326).
    std::string apply_chat_template_json(const std::string& messages_json, const std::string& tools_json,
                                         bool add_generation_prompt) const;

    // The pieces encode turns into ids, as [begin, end) byte offsets
    // (regex_split, tokenizer.cpp:176-226).
    std::vector<std::pair<size_t, size_t>> pre_split(const std::string& text) const;

    size_t vocab_size() const { return vocab_.size(); }
    uint32_t eos_id() const { return eos_id_; }
    uint32_t pad_id() const { return pad_id_; }

private:
    struct Rule {
        int32_t left, right, merged;  // symbol ids
    };
    int32_t intern(const std::string& s);
    std::vector<uint32_t> bpe(const char* p, size_t n) const;
    // earliest special token at or after `from`: (position, length), or (n, 0)
    std::pair<size_t, size_t> next_special(const std::string& text, size_t from) const;

    std::vector<std::string> vocab_;
    std::vector<uint32_t> types_;
    uint32_t eos_id_ = 0, pad_id_ = 0;
    std::unordered_map<std::string, uint32_t> vocab_to_id_;
    // special tokens by first byte, longest first (index into vocab_)
    std::vector<uint32_t> specials_[256];
    // merge rules over interned symbols; pair -> ranks of the rules merging it
    std::unordered_map<std::string, int32_t> sym_id_;
    std::vector<std::string> syms_;
    std::vector<int64_t> sym_vocab_;  // symbol -> vocabulary id, -1 when absent
    std::vector<Rule> rules_;
    std::unordered_map<uint64_t, std::vector<int32_t>> pair_ranks_;
    std::unique_ptr<ChatTemplate> chat_;
    // encoded pieces (the split and the merges are pure functions of the piece)
    mutable std::mutex cache_mu_;
    mutable std::unordered_map<std::string, std::vector<uint32_t>> cache_;
};

}  // namespace minfer
