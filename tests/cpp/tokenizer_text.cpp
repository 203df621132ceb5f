// Text of generated tokens (Tokenizer::decode_continuation), built by tests/test_tokenizer_text.py
// (no GPU): pieces keep their spaces after a prompt, byte-level BPE text is the plain byte
// concatenation, and the byte-level contract stays the reference's token-by-token text.
// Prints one line per case: "<case> <ok|got ...>".
#include <cstdio>
#include <string>
#include <vector>

#include "vk_symbiote/Tokenizer.h"

using namespace vk_symbiote;

static void report(const char* name, const std::string& got, const std::string& want) {
    if (got == want) printf("%s ok\n", name);
    else printf("%s got [%s] want [%s]\n", name, got.c_str(), want.c_str());
}

int main() {
    // SentencePiece: <unk> <s> </s>, 256 byte pieces, then words with the U+2581 space mark
    std::vector<std::string> pieces = {"<unk>", "<s>", "</s>"};
    std::vector<int32_t> types = {2, 3, 3};
    char buf[8];
    for (int b = 0; b < 256; b++) {
        snprintf(buf, sizeof buf, "<0x%02X>", b);
        pieces.push_back(buf);
        types.push_back(6);
    }
    const std::string sp = "\xE2\x96\x81";
    for (const char* w : {"the", "quick", "fox"}) {
        pieces.push_back(sp + w);
        types.push_back(1);
    }
    const uint32_t the = 259, quick = 260, fox = 261;
    std::vector<float> scores(pieces.size(), 0.0f);
    auto spm = Tokenizer::sentencepiece(pieces, scores, types, 1, 2, 0, true, true);
    const std::vector<uint32_t> ctx = {1, the, quick};  // <s> "the quick"
    report("spm_prompt", spm->decode(ctx), "the quick");
    report("spm_continuation", spm->decode_continuation(ctx, {fox, the}), " fox the");
    report("spm_no_context", spm->decode_continuation({}, {fox, the}), "fox the");
    // the prompt ends with the first two byte tokens of a U+2581 mark (E2 96); the continuation
    // brings its last byte (81) and 'x': the new text is the space and the x
    report("spm_split_mark", spm->decode_continuation({1, the, 3 + 0xE2, 3 + 0x96}, {3 + 0x81, 3 + 'x'}), " x");
    // the prompt ends inside a two-byte character (C3 of U+00E9): the prompt's text keeps the
    // lead byte, so the continuation starts with the trailing byte (their concatenation is the
    // full text)
    report("spm_split_char", spm->decode_continuation({1, the, 3 + 0xC3}, {3 + 0xA9, fox}), "\xA9 fox");
    // byte-level BPE: the continuation is the bytes of its tokens
    std::vector<std::string> toks;
    std::vector<int32_t> btypes;
    for (int v = 0; v < 256; v++) {  // GPT-2's byte map, restated for the test's few bytes
        std::string s;
        if ((v >= '!' && v <= '~')) s = std::string(1, (char)v);
        else s = "?" + std::to_string(v);  // placeholders: only printable bytes are used below
        toks.push_back(s);
        btypes.push_back(1);
    }
    toks.push_back("\xC4\xA0" "fox");  // U+0120 (the space byte's character) + "fox"
    btypes.push_back(1);
    auto bpe = Tokenizer::byte_bpe(toks, btypes, {}, "llama-bpe", 0, 0, false);
    report("bpe_continuation", bpe->decode_continuation({'a', 'b'}, {256, '!'}), " fox!");
    // no vocabulary: the reference's generate appends each token's text (ids as bytes)
    auto raw = Tokenizer::byte_level();
    report("byte_contract", raw->decode_continuation({104}, {105, 33}), "i!");
    return 0;
}
