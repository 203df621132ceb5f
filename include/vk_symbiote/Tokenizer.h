// Text <-> token ids.
//
// From a GGUF file with a SentencePiece vocabulary (tokenizer.ggml.model "llama", tokens,
// scores and token types) the tokenizer is the SentencePiece BPE of that vocabulary: spaces
// become U+2581, a dummy prefix space is added, UTF-8 characters are merged pairwise in order
// of the merged piece's score (ties: the leftmost pair), pieces missing from the vocabulary
// fall back to <0xXX> byte tokens, and BOS is prepended (tokenizer.ggml.add_bos_token,
// default true). decode() reverses it (control tokens render as nothing, byte tokens as their
// byte, U+2581 as a space, the dummy prefix removed).
//
// From a GGUF file with a byte-level BPE vocabulary (tokenizer.ggml.model "gpt2": tokens,
// token types, merges, tokenizer.ggml.pre) it is GPT-2-style byte-level BPE: the text is split
// by the pre-tokenizer pattern of tokenizer.ggml.pre ("llama-bpe" / "llama3": the Llama 3
// pattern; "qwen2": the same with one digit per number piece; anything else: GPT-2's), each piece's bytes become the printable characters of
// GPT-2's byte map, and adjacent symbols are merged in order of merge rank (ties: leftmost);
// with the Llama 3 pattern a piece that is itself a token is not merged (ignore_merges). BOS
// is prepended when tokenizer.ggml.add_bos_token is true (default false). decode() maps the
// characters back to bytes (control tokens render as nothing).
//
// Without such a vocabulary it keeps the behaviour the reference actually exhibits
// (vk_symbiote/src/Tokenizer.cpp): its GGUF reader reads key, type and length in the wrong
// order (:41-46), so it always falls back to the 256-entry byte vocabulary (:113-129):
// encode() maps every non-whitespace byte of the text to its value (words are split on
// whitespace, :131-178) and returns {0} for empty text; decode() maps each id to the byte
// id % 256 and joins them with single spaces (:180-198).
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "Common.h"
#include "ConfigManager.h"

namespace vk_symbiote {

class VSL_CPP_API Tokenizer {
public:
    static std::unique_ptr<Tokenizer> from_gguf(const Path& gguf_path);
    static std::unique_ptr<Tokenizer> byte_level();
    // SentencePiece BPE over an explicit vocabulary (token types: 1 normal, 2 unknown,
    // 3 control, 6 byte; GGUF's tokenizer.ggml.token_type)
    static std::unique_ptr<Tokenizer> sentencepiece(const std::vector<std::string>& tokens,
                                                    const std::vector<float>& scores,
                                                    const std::vector<int32_t>& types, uint32_t bos_id,
                                                    uint32_t eos_id, uint32_t unk_id, bool add_bos,
                                                    bool add_space_prefix);
    // GPT-2-style byte-level BPE: tokens in byte-map form, token types (3 = control, never
    // produced by encode), merges "left right" in rank order, pre-tokenizer name
    static std::unique_ptr<Tokenizer> byte_bpe(const std::vector<std::string>& tokens, const std::vector<int32_t>& types,
                                               const std::vector<std::string>& merges, const std::string& pre,
                                               uint32_t bos_id, uint32_t eos_id, bool add_bos);
    ~Tokenizer();

    std::vector<uint32_t> encode(const std::string& text) const;
    std::string decode(const std::vector<uint32_t>& tokens) const;
    // Text of `tokens` generated after `context`: for a vocabulary, decode(context + tokens)
    // with decode(context) taken off the front, so each piece keeps its own spaces (decoding a
    // piece alone would drop its leading space as the dummy prefix); for the byte-level
    // contract, the tokens decoded one by one and concatenated, as the reference's generate does.
    std::string decode_continuation(const std::vector<uint32_t>& context, const std::vector<uint32_t>& tokens) const;
    uint32_t vocab_size() const;
    bool is_subword() const { return spm_ != nullptr || bpe_ != nullptr; }
    bool is_byte_bpe() const { return bpe_ != nullptr; }  // a GPT-2-style ("gpt2") vocabulary
    uint32_t bos_id() const;
    uint32_t eos_id() const;

private:
    struct Spm;
    struct Bpe;
    Spm* spm_ = nullptr;  // SentencePiece vocabulary
    Bpe* bpe_ = nullptr;  // byte-level BPE vocabulary (both null: the byte-level contract)
    std::vector<uint32_t> bpe_encode(const std::string& text) const;
    std::string bpe_decode(const std::vector<uint32_t>& tokens) const;
};

}  // namespace vk_symbiote
