// Byte-level BPE vocabulary of vk_symbiote::Tokenizer (tokenizer_bpe.cpp), shared with
// tokenizer.cpp, which owns the object.
#pragma once

#include <string>
#include <unordered_map>
#include <vector>

#include "../../../include/vk_symbiote/Tokenizer.h"

namespace vk_symbiote {

struct Tokenizer::Bpe {
    std::vector<std::string> tokens;
    std::vector<int32_t> types;
    std::unordered_map<std::string, uint32_t> index;  // byte-map form -> id (non-control)
    std::unordered_map<std::string, int> ranks;       // "left right" -> merge rank
    std::string byte_char[256];                       // byte -> its printable character (UTF-8)
    std::unordered_map<unsigned, unsigned char> char_byte;
    bool llama3 = false;      // the Llama 3 pattern family (with ignore_merges), else GPT-2's
    size_t max_digits = 3;    // digits per number piece in that family (Qwen 2: 1)
    uint32_t bos = 0, eos = 0;
    bool add_bos = false;
};

}  // namespace vk_symbiote
