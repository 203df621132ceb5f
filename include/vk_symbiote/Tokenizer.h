// Text <-> token id conversion with the behaviour the reference actually exhibits
// (vk_symbiote/src/Tokenizer.cpp). Its GGUF vocabulary reader reads key, type and
// length in the wrong order (:41-46), so on standard GGUF files it always falls back to the
// 256-entry byte vocabulary (:113-129): encode() maps every non-whitespace byte of the text
// to its value (words are split on whitespace, :131-178) and returns {0} for empty text;
// decode() maps each id to the byte id % 256 and joins them with single spaces (:180-198).
// This class reproduces that contract; a real subword tokenizer is outside the decode path.
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

    std::vector<uint32_t> encode(const std::string& text) const;
    std::string decode(const std::vector<uint32_t>& tokens) const;
    uint32_t vocab_size() const { return 256; }
};

}  // namespace vk_symbiote
