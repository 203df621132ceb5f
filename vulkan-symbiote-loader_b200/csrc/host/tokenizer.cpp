// Tokenizer: SentencePiece BPE or GPT-2-style byte-level BPE (tokenizer_bpe.cpp) from a GGUF
// vocabulary, or the reference's byte-level contract (vk_symbiote/src/Tokenizer.cpp:113-198)
// when the file has none. Host code, off the decode path: the engine consumes ids.
#include "../../../include/vk_symbiote/Tokenizer.h"

#include <algorithm>
#include <cstring>
#include <queue>
#include <sstream>
#include <unordered_map>

#include "../../../include/vk_symbiote/GGUFLoader.h"
#include "../../../include/vsl.h"
#include "status.h"
#include "tokenizer_bpe.h"

namespace vk_symbiote {

static const std::string SPACE_MARK = "\xE2\x96\x81";  // U+2581, SentencePiece's space

struct Tokenizer::Spm {
    std::vector<std::string> pieces;
    std::vector<float> scores;
    std::vector<int32_t> types;
    std::unordered_map<std::string, uint32_t> index;
    uint32_t byte_id[256];
    bool has_byte[256];
    uint32_t bos = 1, eos = 2, unk = 0;
    bool add_bos = true, add_space_prefix = true;
};

// The byte of a byte piece "<0xXX>" (exactly two hex digits), or -1 for any other piece.
static int byte_piece(const std::string& p) {
    if (p.size() != 6 || p.compare(0, 3, "<0x") != 0 || p[5] != '>') return -1;
    auto hex = [](char c) {
        return c >= '0' && c <= '9' ? c - '0' : c >= 'A' && c <= 'F' ? c - 'A' + 10 : c >= 'a' && c <= 'f' ? c - 'a' + 10 : -1;
    };
    const int hi = hex(p[3]), lo = hex(p[4]);
    return hi < 0 || lo < 0 ? -1 : hi * 16 + lo;
}

Tokenizer::~Tokenizer() {
    delete spm_;
    delete bpe_;
}

std::unique_ptr<Tokenizer> Tokenizer::byte_level() { return std::unique_ptr<Tokenizer>(new Tokenizer()); }

std::unique_ptr<Tokenizer> Tokenizer::sentencepiece(const std::vector<std::string>& tokens,
                                                    const std::vector<float>& scores,
                                                    const std::vector<int32_t>& types, uint32_t bos_id,
                                                    uint32_t eos_id, uint32_t unk_id, bool add_bos,
                                                    bool add_space_prefix) {
    std::unique_ptr<Tokenizer> t(new Tokenizer());
    Spm* s = new Spm();
    t->spm_ = s;
    s->pieces = tokens;
    s->scores = scores;
    s->scores.resize(tokens.size(), 0.0f);
    s->types = types;
    s->types.resize(tokens.size(), 1);
    s->bos = bos_id;
    s->eos = eos_id;
    s->unk = unk_id;
    s->add_bos = add_bos;
    s->add_space_prefix = add_space_prefix;
    for (int b = 0; b < 256; b++) s->has_byte[b] = false;
    for (uint32_t i = 0; i < (uint32_t)tokens.size(); i++) {
        const std::string& p = tokens[i];
        // byte pieces "<0xXX>" (type 6 in GGUF) are the fallback for characters without a piece
        const int b = byte_piece(p);
        if (b >= 0) {
            if (!s->has_byte[b]) {
                s->has_byte[b] = true;
                s->byte_id[b] = i;
            }
            continue;
        }
        if (s->types[i] == 3) continue;  // control tokens (<s>, </s>) are never produced by merges
        s->index.emplace(p, i);          // the first id of a duplicated piece wins
    }
    return t;
}

std::unique_ptr<Tokenizer> Tokenizer::from_gguf(const Path& gguf_path) {
    GGUFLoader loader(gguf_path);
    if (!loader.load()) return byte_level();
    const GGUFMetadataKV* model = loader.get_metadata("tokenizer.ggml.model");
    const auto& vocab = loader.get_vocabulary();
    if (!model || vocab.empty()) return byte_level();
    auto u32 = [&](const char* key, uint32_t dflt) {
        const GGUFMetadataKV* kv = loader.get_metadata(key);
        return kv ? (uint32_t)kv->get_number() : dflt;
    };
    auto flag = [&](const char* key, bool dflt) {
        const GGUFMetadataKV* kv = loader.get_metadata(key);
        return kv ? kv->get_bool() : dflt;
    };
    if (model->get_string() == "gpt2") {  // byte-level BPE: tokens, types, merges, pre-tokenizer
        const GGUFMetadataKV* merges = loader.get_metadata("tokenizer.ggml.merges");
        if (!merges) return byte_level();
        const GGUFMetadataKV* pre = loader.get_metadata("tokenizer.ggml.pre");
        std::vector<std::string> toks;
        std::vector<int32_t> types;
        toks.reserve(vocab.size());
        for (const auto& e : vocab) {
            toks.push_back(e.token);
            types.push_back((int32_t)e.token_type);
        }
        return byte_bpe(toks, types, merges->array_strings, pre ? pre->get_string() : std::string(),
                        u32("tokenizer.ggml.bos_token_id", 0), u32("tokenizer.ggml.eos_token_id", 0),
                        flag("tokenizer.ggml.add_bos_token", false));
    }
    if (model->get_string() != "llama") return byte_level();
    std::vector<std::string> toks;
    std::vector<float> scores;
    std::vector<int32_t> types;
    toks.reserve(vocab.size());
    for (const auto& e : vocab) {
        toks.push_back(e.token);
        scores.push_back(e.score);
        types.push_back(e.token_type);
    }
    return sentencepiece(toks, scores, types, u32("tokenizer.ggml.bos_token_id", 1), u32("tokenizer.ggml.eos_token_id", 2),
                         u32("tokenizer.ggml.unknown_token_id", 0), flag("tokenizer.ggml.add_bos_token", true),
                         flag("tokenizer.ggml.add_space_prefix", true));
}

uint32_t Tokenizer::vocab_size() const {
    return spm_ ? (uint32_t)spm_->pieces.size() : bpe_ ? (uint32_t)bpe_->tokens.size() : 256u;
}
uint32_t Tokenizer::bos_id() const { return spm_ ? spm_->bos : bpe_ ? bpe_->bos : 0u; }
uint32_t Tokenizer::eos_id() const { return spm_ ? spm_->eos : bpe_ ? bpe_->eos : 0u; }

static size_t utf8_len(unsigned char c) {
    if (c < 0x80) return 1;
    if ((c >> 5) == 0x6) return 2;
    if ((c >> 4) == 0xE) return 3;
    if ((c >> 3) == 0x1E) return 4;
    return 1;  // stray continuation byte: its own symbol
}

// bytes of the character at t[i]: its UTF-8 length when all continuation bytes are present,
// else 1 (a malformed lead byte is a symbol of its own and does not swallow what follows)
static size_t char_len(const std::string& t, size_t i) {
    const size_t n = utf8_len((unsigned char)t[i]);
    if (i + n > t.size()) return 1;
    for (size_t k = 1; k < n; k++)
        if (((unsigned char)t[i + k] & 0xC0) != 0x80) return 1;
    return n;
}

std::vector<uint32_t> Tokenizer::encode(const std::string& text) const {
    if (bpe_) return bpe_encode(text);
    if (!spm_) {  // byte-level contract of the reference
        std::vector<uint32_t> ids;
        std::istringstream in(text);
        std::string word;
        while (in >> word)
            for (unsigned char c : word) ids.push_back(c);
        if (ids.empty()) ids.push_back(0);
        return ids;
    }
    const Spm& s = *spm_;
    std::vector<uint32_t> out;
    if (s.add_bos) out.push_back(s.bos);
    if (text.empty()) return out;
    // normalise: spaces -> U+2581, dummy prefix
    std::string t = s.add_space_prefix ? SPACE_MARK : std::string();
    for (char c : text) {
        if (c == ' ') t += SPACE_MARK;
        else t += c;
    }
    // symbols: UTF-8 characters in a linked list
    struct Sym {
        int prev, next;
        size_t pos, len;
    };
    std::vector<Sym> sym;
    for (size_t i = 0; i < t.size();) {
        const size_t n = char_len(t, i);
        sym.push_back({(int)sym.size() - 1, (int)sym.size() + 1, i, n});
        i += n;
    }
    sym.back().next = -1;
    struct Pair {
        float score;
        int left, right;
        size_t len;  // merged length, to discard stale pairs
    };
    auto worse = [](const Pair& a, const Pair& b) {
        return a.score < b.score || (a.score == b.score && a.left > b.left);  // best: high score, then leftmost
    };
    std::priority_queue<Pair, std::vector<Pair>, decltype(worse)> q(worse);
    auto try_pair = [&](int l, int r) {
        if (l < 0 || r < 0) return;
        const size_t len = sym[l].len + sym[r].len;
        auto it = s.index.find(t.substr(sym[l].pos, len));
        if (it == s.index.end()) return;
        q.push({s.scores[it->second], l, r, len});
    };
    for (int i = 0; i + 1 < (int)sym.size(); i++) try_pair(i, i + 1);
    while (!q.empty()) {
        const Pair p = q.top();
        q.pop();
        Sym& L = sym[p.left];
        Sym& R = sym[p.right];
        if (L.len == 0 || R.len == 0 || L.len + R.len != p.len || L.next != p.right) continue;  // stale
        L.len += R.len;
        R.len = 0;
        L.next = R.next;
        if (R.next >= 0) sym[R.next].prev = p.left;
        try_pair(L.prev, p.left);
        try_pair(p.left, L.next);
    }
    for (int i = 0; i >= 0 && i < (int)sym.size(); i = sym[i].next) {
        if (sym[i].len == 0) continue;
        const std::string piece = t.substr(sym[i].pos, sym[i].len);
        auto it = s.index.find(piece);
        if (it != s.index.end()) {
            out.push_back(it->second);
            continue;
        }
        for (unsigned char c : piece) out.push_back(s.has_byte[c] ? s.byte_id[c] : s.unk);
    }
    return out;
}

std::string Tokenizer::decode(const std::vector<uint32_t>& tokens) const {
    if (bpe_) return bpe_decode(tokens);
    if (!spm_) {
        std::string out;
        for (size_t i = 0; i < tokens.size(); i++) {
            out += (char)(unsigned char)(tokens[i] % 256u);
            if (i + 1 < tokens.size()) out += ' ';
        }
        return out;
    }
    const Spm& s = *spm_;
    // pieces and byte tokens first, then every U+2581 of the result is a space (also when the
    // mark itself came as byte tokens), then the dummy prefix goes
    std::string raw;
    for (uint32_t id : tokens) {
        if (id >= s.pieces.size()) continue;
        if (s.types[id] == 3) continue;  // control
        const std::string& p = s.pieces[id];
        const int b = byte_piece(p);
        if (b >= 0) raw += (char)b;
        else raw += p;
    }
    std::string out;
    for (size_t i = 0; i < raw.size();) {
        if (raw.compare(i, SPACE_MARK.size(), SPACE_MARK) == 0) {
            out += ' ';
            i += SPACE_MARK.size();
        } else {
            out += raw[i++];
        }
    }
    if (s.add_space_prefix && !out.empty() && out[0] == ' ') out.erase(0, 1);
    return out;
}

std::string Tokenizer::decode_continuation(const std::vector<uint32_t>& context,
                                           const std::vector<uint32_t>& tokens) const {
    std::string per_token;
    if (!is_subword()) {
        for (uint32_t t : tokens) per_token += decode({t});
        return per_token;
    }
    std::vector<uint32_t> all(context);
    all.insert(all.end(), tokens.begin(), tokens.end());
    const std::string head = decode(context), full = decode(all);
    if (full.size() >= head.size() && full.compare(0, head.size(), head) == 0) return full.substr(head.size());
    // The context ends inside a character or a U+2581 space mark that arrived as byte tokens:
    // its raw bytes are not a prefix of the full text. The continuation is the full text after
    // the longest common byte prefix, started on a character boundary.
    size_t n = 0;
    const size_t m = std::min(head.size(), full.size());
    while (n < m && head[n] == full[n]) n++;
    while (n > 0 && n < full.size() && (static_cast<unsigned char>(full[n]) & 0xC0) == 0x80) n--;
    return full.substr(n);
}

}  // namespace vk_symbiote

// ---------------------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------------------
struct vsl_tokenizer {
    std::unique_ptr<vk_symbiote::Tokenizer> t;
};

extern "C" int vsl_tokenizer_create_gguf(const char* path, vsl_tokenizer** out) {
    if (!path || !out) return vsl::set_error(VSL_ERR_INVALID, "tokenizer: null argument");
    try {
        *out = new vsl_tokenizer{vk_symbiote::Tokenizer::from_gguf(path)};
    } catch (const std::exception& e) {
        return vsl::set_error(VSL_ERR_IO, "tokenizer: %s", e.what());
    }
    return VSL_OK;
}

extern "C" void vsl_tokenizer_destroy(vsl_tokenizer* t) { delete t; }

extern "C" int vsl_tokenizer_info(vsl_tokenizer* t, int* vocab_size, int* is_subword, int32_t* bos_id, int32_t* eos_id) {
    if (!t) return vsl::set_error(VSL_ERR_INVALID, "tokenizer: null handle");
    if (vocab_size) *vocab_size = (int)t->t->vocab_size();
    if (is_subword) *is_subword = t->t->is_subword() ? 1 : 0;
    if (bos_id) *bos_id = (int32_t)t->t->bos_id();
    if (eos_id) *eos_id = (int32_t)t->t->eos_id();
    return VSL_OK;
}

extern "C" int vsl_tokenize(vsl_tokenizer* t, const char* text, size_t len, int32_t* out, int cap, int* n) {
    if (!t || (!text && len) || !n || cap < 0) return vsl::set_error(VSL_ERR_INVALID, "tokenize: bad arguments");
    const std::vector<uint32_t> ids = t->t->encode(std::string(text ? text : "", len));
    *n = (int)ids.size();
    if ((int)ids.size() > cap) return vsl::set_error(VSL_ERR_BOUNDS, "tokenize: %zu ids > capacity %d", ids.size(), cap);
    for (size_t i = 0; i < ids.size(); i++) out[i] = (int32_t)ids[i];
    return VSL_OK;
}

extern "C" int vsl_detokenize(vsl_tokenizer* t, const int32_t* ids, int n, char* out, size_t cap, size_t* len) {
    if (!t || (!ids && n) || n < 0 || !len) return vsl::set_error(VSL_ERR_INVALID, "detokenize: bad arguments");
    std::vector<uint32_t> v(ids, ids + n);
    const std::string s = t->t->decode(v);
    *len = s.size();
    if (s.size() > cap || (!out && s.size()))
        return vsl::set_error(VSL_ERR_BOUNDS, "detokenize: %zu bytes > capacity %zu", s.size(), cap);
    if (!s.empty()) memcpy(out, s.data(), s.size());
    return VSL_OK;
}
