"""Tokenizer without a GPU: SentencePiece BPE from a GGUF vocabulary against an independent
restatement of the algorithm (repeatedly merge the adjacent pair whose concatenation is a
piece with the highest score, leftmost on ties; byte fallback), hand-computed known answers,
round trips, and the byte-level behaviour of files without a vocabulary."""
import random

import pytest

import vsl
from vsl import gguf

SP = "▁"


def write_vocab_gguf(path, pieces, scores, types, add_bos=True, add_space_prefix=True):
    meta = [("general.architecture", gguf.T_STR, "llama"),
            ("tokenizer.ggml.model", gguf.T_STR, "llama"),
            ("tokenizer.ggml.tokens", gguf.T_ARR, (gguf.T_STR, pieces)),
            ("tokenizer.ggml.scores", gguf.T_ARR, (gguf.T_F32, scores)),
            ("tokenizer.ggml.token_type", gguf.T_ARR, (gguf.T_I32, types)),
            ("tokenizer.ggml.bos_token_id", gguf.T_U32, 1),
            ("tokenizer.ggml.eos_token_id", gguf.T_U32, 2),
            ("tokenizer.ggml.unknown_token_id", gguf.T_U32, 0),
            ("tokenizer.ggml.add_bos_token", gguf.T_BOOL, add_bos),
            ("tokenizer.ggml.add_space_prefix", gguf.T_BOOL, add_space_prefix)]
    gguf.write_gguf(str(path), meta, [])


def base_vocab():
    pieces = ["<unk>", "<s>", "</s>"] + [f"<0x{b:02X}>" for b in range(256)]
    types = [2, 3, 3] + [6] * 256
    return pieces, [0.0] * len(pieces), types


def ref_encode(text, pieces, scores, types, add_bos=True, add_space_prefix=True):
    """Textbook SentencePiece BPE (O(n^2) rescans)."""
    index = {}
    for i, p in enumerate(pieces):
        if types[i] in (3, 6):
            continue
        index.setdefault(p, i)
    byte_id = {int(p[3:5], 16): i for i, p in enumerate(pieces) if types[i] == 6}
    out = [1] if add_bos else []
    if not text:
        return out
    t = (SP if add_space_prefix else "") + text.replace(" ", SP)
    syms = list(t)  # code points
    while True:
        best = None
        for i in range(len(syms) - 1):
            m = syms[i] + syms[i + 1]
            if m in index:
                s = scores[index[m]]
                if best is None or s > best[0]:
                    best = (s, i)
        if best is None:
            break
        i = best[1]
        syms[i:i + 2] = [syms[i] + syms[i + 1]]
    for s in syms:
        if s in index:
            out.append(index[s])
        else:
            out += [byte_id.get(b, 0) for b in s.encode("utf-8")]
    return out


def test_known_answers(tmp_path):
    pieces, scores, types = base_vocab()
    extra = [(SP, -1.0), ("h", -2.0), ("e", -2.0), ("l", -2.0), ("o", -2.0), ("w", -2.0), ("r", -2.0),
             ("d", -2.0), (SP + "h", -3.0), ("ll", -3.5), ("llo", -4.0), (SP + "he", -4.5), (SP + "hello", -5.0),
             ("wo", -5.6), ("wor", -6.0), (SP + "w", -6.5), (SP + "wor", -7.0), ("ld", -7.5), (SP + "world", -8.0)]
    # merge paths: ▁h, ll, llo, ▁he, ▁hello; wo, wor, ▁wor, ld, ▁world (▁w loses to wo)
    for p, s in extra:
        pieces.append(p)
        scores.append(s)
        types.append(1)
    path = tmp_path / "v.gguf"
    write_vocab_gguf(path, pieces, scores, types)
    tok = vsl.Tokenizer(str(path))
    assert tok.is_subword and tok.vocab_size == len(pieces) and tok.bos_id == 1 and tok.eos_id == 2
    idx = {p: i for i, p in enumerate(pieces)}
    assert tok.encode("hello world") == [1, idx[SP + "hello"], idx[SP + "world"]]
    assert tok.encode("hello") == [1, idx[SP + "hello"]]
    # 'z' and the euro sign have no piece: UTF-8 byte fallback
    assert tok.encode("hez€") == [1, idx[SP + "he"], 3 + ord("z"), 3 + 0xE2, 3 + 0x82, 3 + 0xAC]
    assert tok.encode("") == [1]
    assert tok.decode(tok.encode("hello world")) == "hello world"
    assert tok.decode([1, idx[SP + "he"], 3 + ord("z"), 3 + 0xE2, 3 + 0x82, 3 + 0xAC, 2]) == "hez€"


@pytest.mark.parametrize("seed", range(4))
def test_matches_reference_restatement_on_random_vocabularies(tmp_path, seed):
    rng = random.Random(seed)
    alphabet = ["a", "b", "c", "d", SP, "é", "中"]
    pieces, scores, types = base_vocab()
    seen = set(pieces)
    for ch in alphabet[:-1]:  # every character but one has a piece
        pieces.append(ch)
        scores.append(-rng.random())
        types.append(1)
        seen.add(ch)
    while len(pieces) < 259 + 120:
        p = "".join(rng.choice(alphabet) for _ in range(rng.randint(2, 5)))
        if p in seen:
            continue
        seen.add(p)
        pieces.append(p)
        scores.append(-rng.uniform(0, 20) if rng.random() > 0.2 else -5.0)  # some score ties
        types.append(1)
    path = tmp_path / f"r{seed}.gguf"
    add_prefix = seed % 2 == 0
    write_vocab_gguf(path, pieces, scores, types, add_space_prefix=add_prefix)
    tok = vsl.Tokenizer(str(path))
    for _ in range(60):
        text = "".join(rng.choice(["a", "b", "c", "d", " ", "é", "中", "x"]) for _ in range(rng.randint(0, 40)))
        want = ref_encode(text, pieces, scores, types, add_space_prefix=add_prefix)
        got = tok.encode(text)
        assert got == want, text
        dec = tok.decode(got)
        assert dec == (text if add_prefix or not text.startswith(" ") else text), (text, dec)


def test_files_without_vocabulary_keep_the_byte_level_contract(tmp_path):
    path = tmp_path / "novocab.gguf"
    gguf.write_gguf(str(path), [("general.architecture", gguf.T_STR, "llama")], [])
    tok = vsl.Tokenizer(str(path))
    assert not tok.is_subword and tok.vocab_size == 256
    assert tok.encode("ab c") == [97, 98, 99]
    assert tok.encode("   ") == [0]
    assert tok.decode([97, 98, 99]) == "a b c"


def test_arbitrary_bytes_round_trip(tmp_path):
    """Byte fallback covers every byte: any byte string (invalid UTF-8 included, without the
    bytes of U+2581 itself) comes back byte for byte through the C ABI."""
    import ctypes as C

    import numpy as np
    pieces, scores, types = base_vocab()
    for p in ("a", "b", SP, SP + "a", "ab", "é"):
        pieces.append(p)
        scores.append(-1.0)
        types.append(1)
    path = tmp_path / "bytes.gguf"
    write_vocab_gguf(path, pieces, scores, types)
    tok = vsl.Tokenizer(str(path))
    L = vsl.lib()
    rng = random.Random(3)
    for n in list(range(0, 6)) + [rng.randrange(6, 120) for _ in range(150)]:
        raw = bytes(rng.choice([rng.randrange(256), ord("a"), ord("b"), ord(" ")]) for _ in range(n))
        if "▁".encode() in raw:
            continue
        ids = np.empty(4 * n + 8, np.int32)
        cnt = C.c_int()
        vsl.check(L.vsl_tokenize(tok.h, raw, len(raw), ids.ctypes.data, ids.size, C.byref(cnt)))
        buf = C.create_string_buffer(n + 8)
        out_len = C.c_size_t()
        vsl.check(L.vsl_detokenize(tok.h, ids.ctypes.data, cnt.value, buf, n + 8, C.byref(out_len)))
        assert buf.raw[:out_len.value] == raw, raw
    tok.close()


def test_encode_grows_its_buffer(tmp_path):
    """Without a U+2581 piece every space costs three byte tokens: more ids than bytes."""
    pieces, scores, types = base_vocab()
    path = tmp_path / "nospace.gguf"
    write_vocab_gguf(path, pieces, scores, types)
    tok = vsl.Tokenizer(str(path))
    ids = tok.encode(" " * 40)
    assert len(ids) == 1 + 3 * 41  # BOS, then the dummy prefix and 40 spaces as 3 bytes each
    assert tok.decode(ids) == " " * 40
    tok.close()
