"""GGUF v3 writer and reader (standard ggml tensor type ids, `general.alignment` honoured).

The writer produces the seeded Llama-architecture models that the parity tests and the
benchmark load through the C++ `GGUFLoader`. Layout follows the public GGUF spec:
header (magic "GGUF", version, tensor count, kv count), metadata key/values, tensor infos
(name, n_dims, ne[] innermost first, ggml type, offset), then the data section aligned to
`general.alignment`. Metadata keys are the ones the reference engine reads
(vk_symbiote/src/GGUFLoader.cpp:673-728).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np

from . import synth

# metadata value types (GGUF spec; the reference's GGUFValueType 0..12 uses the same ids,
# vk_symbiote/include/vk_symbiote/GGUFLoader.h:18-31)
T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64 = range(13)

_SCALAR_FMT = {T_U8: "<B", T_I8: "<b", T_U16: "<H", T_I16: "<h", T_U32: "<I", T_I32: "<i",
               T_F32: "<f", T_BOOL: "<?", T_U64: "<Q", T_I64: "<q", T_F64: "<d"}


@dataclass
class LlamaShape:
    n_layers: int
    d_model: int
    n_heads: int
    n_kv_heads: int
    ffn: int
    vocab: int
    rope_theta: float = 10000.0
    rms_eps: float = 1e-5
    context_length: int = 4096
    head_dim: int = field(init=False)

    def __post_init__(self):
        self.head_dim = self.d_model // self.n_heads


def _s(b: bytearray, text: str):
    raw = text.encode()
    b += struct.pack("<Q", len(raw)) + raw


def _kv(b: bytearray, key: str, vtype: int, value):
    _s(b, key)
    b += struct.pack("<I", vtype)
    if vtype == T_STR:
        _s(b, value)
    elif vtype == T_ARR:
        etype, items = value
        b += struct.pack("<IQ", etype, len(items))
        for it in items:
            if etype == T_STR:
                _s(b, it)
            else:
                b += struct.pack(_SCALAR_FMT[etype], it)
    else:
        b += struct.pack(_SCALAR_FMT[vtype], value)


def _align(n: int, a: int) -> int:
    return (n + a - 1) // a * a


def write_gguf(path: str, metadata: list[tuple[str, int, object]], tensors: list[tuple[str, np.ndarray, int]],
               alignment: int = 32):
    """tensors: (name, array in storage form with shape [rows, cols] or [n], ggml type[, ne]);
    block-quantized tensors pass their GGUF block bytes and the element dimensions ne."""
    head = bytearray()
    head += b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(metadata) + 1)
    _kv(head, "general.alignment", T_U32, alignment)
    for key, vtype, value in metadata:
        _kv(head, key, vtype, value)
    offset = 0
    infos = []
    for name, arr, gtype, *dims in tensors:
        ne = list(dims[0]) if dims else list(reversed(arr.shape))  # ne[0]: the contiguous dimension
        _s(head, name)
        head += struct.pack("<I", len(ne))
        for n in ne:
            head += struct.pack("<Q", n)
        head += struct.pack("<IQ", gtype, offset)
        infos.append((offset, arr))
        offset = _align(offset + arr.nbytes, alignment)
    data0 = _align(len(head), alignment)
    with open(path, "wb") as f:
        f.write(head)
        f.write(b"\0" * (data0 - len(head)))
        pos = 0
        for off, arr in infos:
            if off > pos:
                f.write(b"\0" * (off - pos))
                pos = off
            f.write(np.ascontiguousarray(arr).tobytes())
            pos += arr.nbytes


def llama_metadata(shape: LlamaShape, name: str = "vsl-synthetic") -> list[tuple[str, int, object]]:
    return [
        ("general.architecture", T_STR, "llama"),
        ("general.name", T_STR, name),
        ("llama.context_length", T_U32, shape.context_length),
        ("llama.embedding_length", T_U32, shape.d_model),
        ("llama.block_count", T_U32, shape.n_layers),
        ("llama.feed_forward_length", T_U32, shape.ffn),
        ("llama.attention.head_count", T_U32, shape.n_heads),
        ("llama.attention.head_count_kv", T_U32, shape.n_kv_heads),
        ("llama.rope.freq_base", T_F32, shape.rope_theta),
        ("llama.attention.layer_norm_rms_epsilon", T_F32, shape.rms_eps),
        ("llama.vocab_size", T_U32, shape.vocab),
    ]


def write_synthetic_llama(path: str, shape: LlamaShape, dtype: int, seed: int, sigma: float = 0.02):
    """Seeded Llama model: matrices from vsl.synth (norms 1.0, stored F32)."""
    d, hd, F, V = shape.d_model, shape.head_dim, shape.ffn, shape.vocab
    qd, kvd = shape.n_heads * hd, shape.n_kv_heads * hd
    ones = np.ones(d, dtype=np.float32)

    def mat(tid, rows, cols):
        if dtype in synth.Q_STD:  # block-quantized: GGUF blocks + element dims
            return (synth.synth_q_blocks(seed, tid, rows, cols, dtype, sigma), dtype, (cols, rows))
        return (synth.synth_tensor(seed, tid, (rows, cols), dtype, sigma), dtype)

    t = [("token_embd.weight", *mat(synth.TID_TOK_EMBD, V, d)),
         ("output_norm.weight", ones, synth.GGML_F32),
         ("output.weight", *mat(synth.TID_OUTPUT, V, d))]
    for l in range(shape.n_layers):
        def m(kind, rows, cols):
            return mat(synth.tid_layer(l, kind), rows, cols)
        t += [(f"blk.{l}.attn_norm.weight", ones, synth.GGML_F32),
              (f"blk.{l}.attn_q.weight", *m(synth.K_Q, qd, d)),
              (f"blk.{l}.attn_k.weight", *m(synth.K_K, kvd, d)),
              (f"blk.{l}.attn_v.weight", *m(synth.K_V, kvd, d)),
              (f"blk.{l}.attn_output.weight", *m(synth.K_O, d, qd)),
              (f"blk.{l}.ffn_norm.weight", ones, synth.GGML_F32),
              (f"blk.{l}.ffn_gate.weight", *m(synth.K_GATE, F, d)),
              (f"blk.{l}.ffn_up.weight", *m(synth.K_UP, F, d)),
              (f"blk.{l}.ffn_down.weight", *m(synth.K_DOWN, d, F))]
    write_gguf(path, llama_metadata(shape), t)


# ---------------------------------------------------------------------------------------
# reader (used by tests to inspect files the writer produced)
# ---------------------------------------------------------------------------------------

class _R:
    def __init__(self, buf: bytes):
        self.b, self.p = buf, 0

    def take(self, fmt: str):
        v = struct.unpack_from(fmt, self.b, self.p)
        self.p += struct.calcsize(fmt)
        return v[0]

    def s(self) -> str:
        n = self.take("<Q")
        v = self.b[self.p:self.p + n].decode()
        self.p += n
        return v

    def value(self, t: int):
        if t == T_STR:
            return self.s()
        if t == T_ARR:
            et, n = self.take("<I"), self.take("<Q")
            return [self.value(et) for _ in range(n)]
        return self.take(_SCALAR_FMT[t])


def read_gguf(path: str):
    """Returns (metadata dict, {name: (ggml type, ne list, absolute offset)})."""
    with open(path, "rb") as f:
        buf = f.read()
    r = _R(buf)
    if buf[:4] != b"GGUF":
        raise ValueError("bad magic")
    r.p = 4
    _version, nt, nkv = r.take("<I"), r.take("<Q"), r.take("<Q")
    meta = {}
    for _ in range(nkv):
        k = r.s()
        t = r.take("<I")
        meta[k] = r.value(t)
    infos = {}
    for _ in range(nt):
        name = r.s()
        nd = r.take("<I")
        ne = [r.take("<Q") for _ in range(nd)]
        gt = r.take("<I")
        off = r.take("<Q")
        infos[name] = (gt, ne, off)
    data0 = _align(r.p, int(meta.get("general.alignment", 32)))
    return meta, {k: (gt, ne, data0 + off) for k, (gt, ne, off) in infos.items()}
