"""Byte-level BPE (GGUF tokenizer.ggml.model "gpt2") without a GPU: the C++ tokenizer against an
independent restatement — the pre-tokenizer patterns evaluated by the `regex` module, GPT-2's
byte map, and the textbook BPE loop (merge every occurrence of the lowest-ranked adjacent pair,
repeat) — on vocabularies trained by BPE on a mixed-script corpus, for the GPT-2 and the Llama 3
pre-tokenizers; hand-computed known answers; and decode(encode(text)) == text."""
import random
from collections import Counter

import pytest

import vsl
from vsl import gguf

regex = pytest.importorskip("regex")

GPT2_PAT = r"""'s|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+"""
LLAMA3_PAT = (r"""(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,3}| ?[^\s\p{L}\p{N}]+[\r\n]*|"""
              r"""\s*[\r\n]+|\s+(?!\S)|\s+""")
QWEN2_PAT = LLAMA3_PAT.replace(r"\p{N}{1,3}", r"\p{N}")
PATTERNS = {"gpt-2": GPT2_PAT, "llama-bpe": LLAMA3_PAT, "qwen2": QWEN2_PAT}
SPECIAL = ["<|begin_of_text|>", "<|end_of_text|>"]


def byte_map():
    """GPT-2's printable character for every byte."""
    bs = list(range(ord("!"), ord("~") + 1)) + list(range(0xA1, 0xAD)) + list(range(0xAE, 0x100))
    cs = bs[:]
    n = 0
    for b in range(256):
        if b not in bs:
            bs.append(b)
            cs.append(256 + n)
            n += 1
    return {b: chr(c) for b, c in zip(bs, cs)}


BYTE_CHAR = byte_map()
CHAR_BYTE = {c: b for b, c in BYTE_CHAR.items()}


def pieces(text, pre):
    return [p for p in regex.findall(PATTERNS[pre], text)]


def to_chars(piece):
    return [BYTE_CHAR[b] for b in piece.encode("utf-8")]


def train(corpus, pre, n_merges):
    """BPE training: repeatedly merge the most frequent adjacent pair (ties: smallest pair)."""
    words = Counter(tuple(to_chars(p)) for t in corpus for p in pieces(t, pre))
    merges = []
    for _ in range(n_merges):
        pairs = Counter()
        for w, f in words.items():
            for a, b in zip(w, w[1:]):
                pairs[(a, b)] += f
        if not pairs:
            break
        best = min(pairs.items(), key=lambda kv: (-kv[1], kv[0]))[0]
        merges.append(best)
        nw = Counter()
        for w, f in words.items():
            out, i = [], 0
            while i < len(w):
                if i + 1 < len(w) and (w[i], w[i + 1]) == best:
                    out.append(w[i] + w[i + 1])
                    i += 2
                else:
                    out.append(w[i])
                    i += 1
            nw[tuple(out)] += f
        words = nw
    return merges


def ref_bpe(chars, ranks):
    """GPT-2 encoder.py's loop: the lowest-ranked pair, every occurrence left to right."""
    word = list(chars)
    while len(word) > 1:
        pairs = {(a, b) for a, b in zip(word, word[1:])}
        best = min(pairs, key=lambda p: ranks.get(p, float("inf")))
        if best not in ranks:
            break
        out, i = [], 0
        while i < len(word):
            if i + 1 < len(word) and (word[i], word[i + 1]) == best:
                out.append(word[i] + word[i + 1])
                i += 2
            else:
                out.append(word[i])
                i += 1
        word = out
    return word


def ref_encode(text, voc, pre, add_bos=True):
    index, ranks, bos = voc["index"], voc["ranks"], voc["bos"]
    out = [bos] if add_bos else []
    for p in pieces(text, pre):
        chars = to_chars(p)
        if pre in ("llama-bpe", "qwen2") and "".join(chars) in index:  # ignore_merges
            out.append(index["".join(chars)])
            continue
        out += [index[s] for s in ref_bpe(chars, ranks)]
    return out


WORDS = ["the", "and", "token", "decode", "Hello", "WORLD", "naïve", "café", "Straße", "über",
         "γειά", "σου", "привет", "мир", "日本語", "東京", "한국어", "שלום", "مرحبا", "ſtraße",
         "don't", "I'LL", "we're", "they've", "it's", "O'Neil", "x2", "3.14159", "2024", "١٢٣", "⅓", "²"]
PUNCT = ["!", "?", "...", "$", "(", ")", "--", "/", "#", "@", "🙂", "€", "—", "'", "\"", "«", "»"]
SPACES = [" ", " ", " ", "  ", "\n", "\n\n", "\t", " \n", "\r\n", "　", " ", "   "]


def random_text(rng, n):
    parts = []
    for _ in range(n):
        r = rng.random()
        if r < 0.55:
            parts.append(rng.choice(WORDS))
        elif r < 0.7:
            parts.append(str(rng.randrange(0, 10 ** rng.randrange(1, 7))))
        elif r < 0.85:
            parts.append(rng.choice(PUNCT))
        else:
            parts.append(chr(rng.choice([rng.randrange(0x20, 0x7F), rng.randrange(0xA0, 0x2FF),
                                         rng.randrange(0x370, 0x52F), rng.randrange(0x4E00, 0x4F00),
                                         rng.randrange(0x1F300, 0x1F650)])))
        parts.append(rng.choice(SPACES))
    return "".join(parts)


def build_vocab(pre, n_merges=300, seed=1):
    rng = random.Random(seed)
    corpus = [random_text(rng, 40) for _ in range(120)]
    merges = train(corpus, pre, n_merges)
    tokens = [BYTE_CHAR[b] for b in range(256)]
    for a, b in merges:
        if a + b not in tokens:
            tokens.append(a + b)
    types = [1] * len(tokens)
    bos = len(tokens)
    tokens += SPECIAL
    types += [3, 3]
    index = {}
    for i, t in enumerate(tokens):
        if types[i] != 3:
            index.setdefault(t, i)
    ranks = {m: r for r, m in enumerate(merges)}
    return dict(tokens=tokens, types=types, merges=[f"{a} {b}" for a, b in merges], index=index, ranks=ranks,
                bos=bos, eos=bos + 1)


def write_bpe_gguf(path, voc, pre, add_bos=True):
    meta = [("general.architecture", gguf.T_STR, "llama"),
            ("tokenizer.ggml.model", gguf.T_STR, "gpt2"),
            ("tokenizer.ggml.pre", gguf.T_STR, pre),
            ("tokenizer.ggml.tokens", gguf.T_ARR, (gguf.T_STR, voc["tokens"])),
            ("tokenizer.ggml.token_type", gguf.T_ARR, (gguf.T_I32, voc["types"])),
            ("tokenizer.ggml.merges", gguf.T_ARR, (gguf.T_STR, voc["merges"])),
            ("tokenizer.ggml.bos_token_id", gguf.T_U32, voc["bos"]),
            ("tokenizer.ggml.eos_token_id", gguf.T_U32, voc["eos"]),
            ("tokenizer.ggml.add_bos_token", gguf.T_BOOL, add_bos)]
    gguf.write_gguf(str(path), meta, [])


@pytest.fixture(scope="module", params=["gpt-2", "llama-bpe", "qwen2"])
def bpe_case(request, tmp_path_factory):
    pre = request.param
    voc = build_vocab(pre)
    path = tmp_path_factory.mktemp("bpe") / f"{pre}.gguf"
    write_bpe_gguf(path, voc, pre)
    tok = vsl.Tokenizer(str(path))
    yield pre, voc, tok
    tok.close()


def test_bpe_matches_reference_on_random_text(bpe_case):
    pre, voc, tok = bpe_case
    assert tok.is_subword and tok.vocab_size == len(voc["tokens"]) and tok.bos_id == voc["bos"]
    rng = random.Random(7)
    n_multi = 0
    for _ in range(150):
        text = random_text(rng, rng.randrange(0, 30))
        want = ref_encode(text, voc, pre)
        got = tok.encode(text)
        assert got == want, (pre, text)
        n_multi += sum(1 for i in got if len(voc["tokens"][i]) > 1)
    assert n_multi > 500  # the merges are exercised, not only single bytes


def test_bpe_round_trip(bpe_case):
    pre, voc, tok = bpe_case
    rng = random.Random(11)
    for _ in range(60):
        text = random_text(rng, 25)
        ids = tok.encode(text)
        assert ids[0] == voc["bos"]
        assert tok.decode(ids) == text  # BOS (a control token) renders as nothing


def test_pretokenizer_edge_cases(bpe_case):
    pre, voc, tok = bpe_case
    for text in ["", " ", "  ", "\n", " \n\n ", "a  b", "a\t\tb", "x\r\n\r\ny", "'s 'S 'll 'LL 'ſ 're",
                 "12345678 ١٢٣٤٥ ²³", "$hello  world!!\n\n", "...\n", "  🙂🙂 🙂", "ab　　cd",
                 " x", "é", "'", "''", "a'"]:
        assert tok.encode(text) == ref_encode(text, voc, pre), (pre, repr(text))


def test_known_answers(tmp_path):
    # vocabulary: the 256 byte characters, then "he", "Ġt", "Ġthe" (Ġ = the space byte's character)
    G = BYTE_CHAR[ord(" ")]
    tokens = [BYTE_CHAR[b] for b in range(256)] + ["he", G + "t", G + "the", "<|begin_of_text|>"]
    types = [1] * 259 + [3]
    voc = dict(tokens=tokens, types=types, merges=["h e", f"{G} t", f"{G}t he"], bos=259, eos=259)
    path = tmp_path / "kat.gguf"
    write_bpe_gguf(path, voc, "gpt-2", add_bos=False)
    tok = vsl.Tokenizer(str(path))
    # " the" -> Ġ t h e -> (h e: rank 0) Ġ t he -> (Ġ t: rank 1) Ġt he -> (Ġt he: rank 2) Ġthe
    assert tok.encode(" the") == [258]
    # "the": t h e -> t he (no "t he" merge)
    assert tok.encode("the") == [ord("t"), 256]
    # bytes outside the printable range map to characters 256+ (byte 0x0A is the 11th such byte)
    assert tokens[ord("\n")] == chr(256 + 10) and tok.encode("\n") == [ord("\n")]
    assert tok.decode([258, 256, 259]) == " thehe"
    tok.close()


def test_arbitrary_bytes_round_trip(bpe_case):
    """Byte-level BPE loses nothing: any byte string, invalid UTF-8 included, comes back
    byte for byte (through the C ABI, without a text decode in between)."""
    import ctypes as C

    import numpy as np
    _, voc, tok = bpe_case
    L = vsl.lib()
    rng = random.Random(5)
    for n in list(range(0, 8)) + [rng.randrange(8, 200) for _ in range(150)]:
        raw = bytes(rng.randrange(256) for _ in range(n))
        ids = np.empty(2 * n + 8, np.int32)
        cnt = C.c_int()
        vsl.check(L.vsl_tokenize(tok.h, raw, len(raw), ids.ctypes.data, ids.size, C.byref(cnt)))
        assert cnt.value >= 1 and ids[0] == voc["bos"]
        buf = C.create_string_buffer(n + 1)
        out_len = C.c_size_t()
        vsl.check(L.vsl_detokenize(tok.h, ids.ctypes.data, cnt.value, buf, n + 1, C.byref(out_len)))
        assert buf.raw[:out_len.value] == raw
