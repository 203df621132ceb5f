// GPT-2-style byte-level BPE for GGUF vocabularies with tokenizer.ggml.model "gpt2" (Llama 3
// and other byte-level models). The reference has no such tokenizer (its Tokenizer.cpp falls
// back to bytes for every file); this is the published GPT-2 algorithm:
//   1. pre-tokenize the text with the model's pattern (GPT-2's, or Llama 3's), evaluated here
//      by hand over code points classified with the Unicode tables of unicode_classes.h;
//   2. map every byte of a piece to a printable character (GPT-2's byte map: the bytes
//      '!'..'~', 0xA1..0xAC and 0xAE..0xFF stand for themselves, the other 68 take the code
//      points 256, 257, ... in byte order);
//   3. merge adjacent symbols, always the pair of lowest merge rank first (leftmost on ties),
//      until no adjacent pair is a merge; emit the token id of every symbol.
// Host code, off the decode path.
#include <cstring>
#include <queue>
#include <unordered_map>

#include "../../../include/vk_symbiote/Tokenizer.h"
#include "tokenizer_bpe.h"
#include "unicode_classes.h"

namespace vk_symbiote {

namespace {

enum CpClass { C_LETTER, C_NUMBER, C_SPACE, C_OTHER };

bool in_ranges(const CpRange* r, int n, unsigned cp) {
    int lo = 0, hi = n - 1;
    while (lo <= hi) {
        const int mid = (lo + hi) / 2;
        if (cp < r[mid].lo) hi = mid - 1;
        else if (cp > r[mid].hi) lo = mid + 1;
        else return true;
    }
    return false;
}

CpClass classify(unsigned cp) {
    if (in_ranges(kLetter, kLetter_N, cp)) return C_LETTER;
    if (in_ranges(kNumber, kNumber_N, cp)) return C_NUMBER;
    if (in_ranges(kSpace, kSpace_N, cp)) return C_SPACE;
    return C_OTHER;
}

void append_utf8(std::string& s, unsigned cp) {
    if (cp < 0x80) {
        s += (char)cp;
    } else if (cp < 0x800) {
        s += (char)(0xC0 | (cp >> 6));
        s += (char)(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
        s += (char)(0xE0 | (cp >> 12));
        s += (char)(0x80 | ((cp >> 6) & 0x3F));
        s += (char)(0x80 | (cp & 0x3F));
    } else {
        s += (char)(0xF0 | (cp >> 18));
        s += (char)(0x80 | ((cp >> 12) & 0x3F));
        s += (char)(0x80 | ((cp >> 6) & 0x3F));
        s += (char)(0x80 | (cp & 0x3F));
    }
}

// One decoded character: its code point and its byte span in the text. A byte that does not
// start a valid UTF-8 sequence is a character of its own (class "other").
struct Cp {
    unsigned cp;
    size_t pos, len;
    CpClass cls;
};

std::vector<Cp> decode_utf8(const std::string& t) {
    std::vector<Cp> out;
    const unsigned char* s = reinterpret_cast<const unsigned char*>(t.data());
    const size_t n = t.size();
    for (size_t i = 0; i < n;) {
        const unsigned c = s[i];
        size_t len = 1;
        unsigned cp = c;
        bool ok = true;
        if (c >= 0x80) {
            len = (c >> 5) == 0x6 ? 2 : (c >> 4) == 0xE ? 3 : (c >> 3) == 0x1E ? 4 : 0;
            ok = len > 0 && i + len <= n;
            if (ok) {
                cp = c & (0x7F >> len);
                for (size_t k = 1; k < len && ok; k++) {
                    ok = (s[i + k] & 0xC0) == 0x80;
                    cp = (cp << 6) | (s[i + k] & 0x3F);
                }
            }
            if (!ok) len = 1;
        }
        out.push_back({cp, i, len, ok ? classify(cp) : C_OTHER});
        i += len;
    }
    return out;
}

bool is_crlf(unsigned cp) { return cp == '\r' || cp == '\n'; }

// lower-case match of a contraction letter under the pattern's case folding ("s" also folds
// U+017F, LATIN SMALL LETTER LONG S)
bool fold_eq(unsigned cp, char lower, bool icase) {
    if (cp == (unsigned)lower) return true;
    if (!icase) return false;
    if (cp == (unsigned)(lower - 32)) return true;
    return lower == 's' && cp == 0x17F;
}

// length (in characters) of the contraction at i, 0 if none: 's 't 're 've 'm 'll 'd
size_t contraction(const std::vector<Cp>& c, size_t i, bool icase) {
    const size_t n = c.size();
    if (c[i].cp != '\'' || i + 1 >= n) return 0;
    const unsigned a = c[i + 1].cp;
    if (fold_eq(a, 's', icase) || fold_eq(a, 't', icase) || fold_eq(a, 'm', icase) || fold_eq(a, 'd', icase)) return 2;
    if (i + 2 < n) {
        const unsigned b = c[i + 2].cp;
        if ((fold_eq(a, 'r', icase) || fold_eq(a, 'v', icase)) && fold_eq(b, 'e', icase)) return 3;
        if (fold_eq(a, 'l', icase) && fold_eq(b, 'l', icase)) return 3;
    }
    return 0;
}

size_t run(const std::vector<Cp>& c, size_t i, CpClass k) {
    size_t j = i;
    while (j < c.size() && c[j].cls == k) j++;
    return j - i;
}

// \s+(?!\S) and \s+ at i (c[i] is whitespace): the first keeps the run's last character for
// the next piece when a non-space follows
size_t space_run(const std::vector<Cp>& c, size_t i) {
    const size_t r = run(c, i, C_SPACE);
    if (i + r == c.size() || r < 2) return r;
    return r - 1;
}

// GPT-2: 's|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+
size_t match_gpt2(const std::vector<Cp>& c, size_t i) {
    const size_t n = c.size();
    if (size_t k = contraction(c, i, false)) return k;
    const bool sp = c[i].cp == ' ' && i + 1 < n;
    for (CpClass k : {C_LETTER, C_NUMBER, C_OTHER}) {
        if (sp && c[i + 1].cls == k) return 1 + run(c, i + 1, k);
        if (c[i].cls == k) return run(c, i, k);
    }
    return space_run(c, i);
}

// Llama 3: (?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,3}|
//          ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+
// Qwen 2: the same with \p{N} (one digit per piece): max_digits 1.
size_t match_llama3(const std::vector<Cp>& c, size_t i, size_t max_digits) {
    const size_t n = c.size();
    if (size_t k = contraction(c, i, true)) return k;
    const CpClass ci = c[i].cls;
    if (ci != C_LETTER && ci != C_NUMBER && !is_crlf(c[i].cp) && i + 1 < n && c[i + 1].cls == C_LETTER)
        return 1 + run(c, i + 1, C_LETTER);
    if (ci == C_LETTER) return run(c, i, C_LETTER);
    if (ci == C_NUMBER) {
        const size_t r = run(c, i, C_NUMBER);
        return r < max_digits ? r : max_digits;
    }
    size_t j = 0;
    if (c[i].cp == ' ' && i + 1 < n && c[i + 1].cls == C_OTHER) j = i + 1 + run(c, i + 1, C_OTHER);
    else if (ci == C_OTHER) j = i + run(c, i, C_OTHER);
    if (j) {
        while (j < n && is_crlf(c[j].cp)) j++;
        return j - i;
    }
    // c[i] is whitespace: \s*[\r\n]+ up to the run's last CR/LF, else \s+(?!\S) / \s+
    const size_t r = run(c, i, C_SPACE);
    for (size_t k = r; k > 0; k--)
        if (is_crlf(c[i + k - 1].cp)) return k;
    return space_run(c, i);
}

}  // namespace


std::unique_ptr<Tokenizer> Tokenizer::byte_bpe(const std::vector<std::string>& tokens, const std::vector<int32_t>& types,
                                               const std::vector<std::string>& merges, const std::string& pre,
                                               uint32_t bos_id, uint32_t eos_id, bool add_bos) {
    std::unique_ptr<Tokenizer> t(new Tokenizer());
    Bpe* b = new Bpe();
    t->bpe_ = b;
    b->tokens = tokens;
    b->types = types;
    b->types.resize(tokens.size(), 1);
    b->bos = bos_id;
    b->eos = eos_id;
    b->add_bos = add_bos;
    b->llama3 = pre == "llama-bpe" || pre == "llama3" || pre == "llama-v3" || pre == "qwen2";
    b->max_digits = pre == "qwen2" ? 1 : 3;
    for (uint32_t i = 0; i < (uint32_t)tokens.size(); i++)
        if (b->types[i] != 3) b->index.emplace(tokens[i], i);  // the first id of a duplicate wins
    for (int r = 0; r < (int)merges.size(); r++) b->ranks.emplace(merges[r], r);
    unsigned next = 256;
    for (int v = 0; v < 256; v++) {
        const bool self = (v >= '!' && v <= '~') || (v >= 0xA1 && v <= 0xAC) || (v >= 0xAE && v <= 0xFF);
        const unsigned cp = self ? (unsigned)v : next++;
        append_utf8(b->byte_char[v], cp);
        b->char_byte[cp] = (unsigned char)v;
    }
    return t;
}

std::vector<uint32_t> Tokenizer::bpe_encode(const std::string& text) const {
    const Bpe& b = *bpe_;
    std::vector<uint32_t> out;
    if (b.add_bos) out.push_back(b.bos);
    const std::vector<Cp> c = decode_utf8(text);
    struct Sym {
        int prev, next;
        std::string s;
    };
    struct Pair {
        int rank, left, right;
        size_t len;  // merged length, to discard stale pairs
    };
    auto worse = [](const Pair& x, const Pair& y) { return x.rank > y.rank || (x.rank == y.rank && x.left > y.left); };
    for (size_t i = 0; i < c.size();) {
        const size_t k = b.llama3 ? match_llama3(c, i, b.max_digits) : match_gpt2(c, i);
        const size_t p0 = c[i].pos, p1 = c[i + k - 1].pos + c[i + k - 1].len;
        i += k;
        std::vector<Sym> sym;
        std::string word;
        for (size_t p = p0; p < p1; p++) {
            const std::string& ch = b.byte_char[(unsigned char)text[p]];
            sym.push_back({(int)sym.size() - 1, (int)sym.size() + 1, ch});
            word += ch;
        }
        sym.back().next = -1;
        if (b.llama3) {  // ignore_merges: a piece that is a token stays whole
            auto it = b.index.find(word);
            if (it != b.index.end()) {
                out.push_back(it->second);
                continue;
            }
        }
        std::priority_queue<Pair, std::vector<Pair>, decltype(worse)> q(worse);
        auto try_pair = [&](int l, int r) {
            if (l < 0 || r < 0) return;
            auto it = b.ranks.find(sym[l].s + " " + sym[r].s);
            if (it != b.ranks.end()) q.push({it->second, l, r, sym[l].s.size() + sym[r].s.size()});
        };
        for (int s = 0; s + 1 < (int)sym.size(); s++) try_pair(s, s + 1);
        while (!q.empty()) {
            const Pair pr = q.top();
            q.pop();
            Sym& L = sym[pr.left];
            Sym& R = sym[pr.right];
            if (L.s.empty() || R.s.empty() || L.next != pr.right || L.s.size() + R.s.size() != pr.len) continue;
            L.s += R.s;
            R.s.clear();
            L.next = R.next;
            if (R.next >= 0) sym[R.next].prev = pr.left;
            try_pair(L.prev, pr.left);
            try_pair(pr.left, L.next);
        }
        for (int s = 0; s >= 0; s = sym[s].next) {
            auto it = b.index.find(sym[s].s);
            if (it != b.index.end()) {
                out.push_back(it->second);
                continue;
            }
            // a symbol missing from the vocabulary: its bytes one by one (each byte's
            // character is a token in every complete byte-level vocabulary)
            for (const Cp& x : decode_utf8(sym[s].s)) {
                auto cb = b.char_byte.find(x.cp);
                if (cb == b.char_byte.end()) continue;
                auto bt = b.index.find(b.byte_char[cb->second]);
                if (bt != b.index.end()) out.push_back(bt->second);
            }
        }
    }
    return out;
}

std::string Tokenizer::bpe_decode(const std::vector<uint32_t>& tokens) const {
    const Bpe& b = *bpe_;
    std::string out;
    for (uint32_t id : tokens) {
        if (id >= b.tokens.size() || b.types[id] == 3) continue;  // control tokens render as nothing
        for (const Cp& x : decode_utf8(b.tokens[id])) {
            auto cb = b.char_byte.find(x.cp);
            if (cb != b.char_byte.end()) out += (char)cb->second;
            else out.append(b.tokens[id], x.pos, x.len);  // not a byte-map character: kept as text
        }
    }
    return out;
}

}  // namespace vk_symbiote
