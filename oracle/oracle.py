"""ctypes front end of the CPU oracle (oracle/vsl_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline / reference legs as the checker or the timed CPU baseline. The product
library never imports it. Parity status: unpinned by reference outputs (the reference has
no golden vectors and cannot be built without a Vulkan stack); pinned instead against the
float64 NumPy restatement in tests/golden/make_golden.py and source-derived known answers.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

F32, F16, BF16 = 0, 1, 30
Q4_0, Q4_1, Q8_0 = 2, 3, 8


class OrcConfig(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("d", C.c_int), ("n_heads", C.c_int), ("n_kv", C.c_int),
                ("head_dim", C.c_int), ("ffn", C.c_int), ("vocab", C.c_int),
                ("rope_theta", C.c_float), ("eps", C.c_float),
                ("wdtype", C.c_int), ("kvdtype", C.c_int), ("max_seq", C.c_int), ("max_batch", C.c_int)]


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        vp, i32, f32p = C.c_void_p, C.c_int, C.POINTER(C.c_float)
        L.orc_h2f.restype = C.c_float
        L.orc_h2f.argtypes = [C.c_uint16]
        L.orc_f2h.restype = C.c_uint16
        L.orc_f2h.argtypes = [C.c_float]
        L.orc_bf2f.restype = C.c_float
        L.orc_bf2f.argtypes = [C.c_uint16]
        L.orc_f2bf.restype = C.c_uint16
        L.orc_f2bf.argtypes = [C.c_float]
        L.orc_synth_fill.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64, C.c_double, i32, vp]
        L.orc_synth_ids.argtypes = [C.c_uint64, C.c_uint64, i32, i32, vp]
        L.orc_gemv.argtypes = [i32, vp, i32, i32, vp, i32, vp]
        L.orc_rmsnorm.argtypes = [vp, vp, i32, i32, i32, C.c_float, vp]
        L.orc_rope_table.argtypes = [i32, i32, C.c_float, vp, vp]
        L.orc_rope_apply.argtypes = [vp, i32, i32, vp, vp]
        L.orc_swiglu.argtypes = [vp, vp, i32, vp]
        L.orc_argmax.restype = C.c_int32
        L.orc_argmax.argtypes = [vp, i32]
        L.orc_attention.argtypes = [vp, vp, vp, i32, i32, i32, i32, i32, i32, vp, vp]
        L.orc_attention_from.argtypes = [vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, vp, vp]
        L.orc_sparse_first.argtypes = [i32, i32, i32, i32, i32]
        L.orc_sparse_first.restype = i32
        L.orc_model_set_sparse.argtypes = [vp, i32, i32, i32, i32]
        L.orc_model_load_gguf.argtypes = [C.c_char_p, i32, i32, i32, C.POINTER(vp)]
        L.orc_model_load_gguf_ex.argtypes = [C.c_char_p, i32, i32, i32, i32, C.POINTER(vp)]
        L.orc_dequant_blocks.argtypes = [i32, vp, C.c_size_t, i32, vp]
        L.orc_synthq_dequant.argtypes = [C.c_uint64, C.c_uint64, C.c_size_t, C.c_size_t, C.c_double, i32, vp]
        L.orc_model_synthetic.argtypes = [C.POINTER(OrcConfig), C.c_uint64, C.c_double, C.POINTER(vp)]
        L.orc_model_free.argtypes = [vp]
        L.orc_model_get_config.argtypes = [vp, C.POINTER(OrcConfig)]
        L.orc_model_clear_kv.argtypes = [vp]
        L.orc_model_fill_kv_synthetic.argtypes = [vp, C.c_uint64, C.c_double, i32, i32]
        L.orc_model_step.argtypes = [vp, i32, vp, vp, vp, vp]
        L.orc_num_threads.restype = i32
        L.orc_set_num_threads.argtypes = [i32]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def dequant_blocks(dtype, blocks: np.ndarray, n_elems: int, legacy_q4: int = 0) -> np.ndarray:
    """GGUF Q8_0 / Q4_0 / Q4_1 block bytes -> fp32 values (the reference loader's dequantisation)."""
    out = np.empty(n_elems, np.float32)
    b = np.ascontiguousarray(blocks, np.uint8)
    lib().orc_dequant_blocks(dtype, _p(b), n_elems, legacy_q4, _p(out))
    return out


def synthq_dequant(seed, tid, rows, cols, dtype, sigma=0.02) -> np.ndarray:
    """Seeded block-quantized tensor, dequantized to fp32 [rows][cols]."""
    out = np.empty((rows, cols), np.float32)
    lib().orc_synthq_dequant(seed, tid, rows, cols, sigma, dtype, _p(out))
    return out


def synth_fill(seed, tid, n, sigma=0.02, dtype=F32, start=0):
    dt = {F32: np.float32, F16: np.uint16, BF16: np.uint16}[dtype]
    out = np.empty(n, dtype=dt)
    lib().orc_synth_fill(seed, tid, start, n, sigma, dtype, _p(out))
    return out


def synth_ids(seed, stream, n, vocab):
    out = np.empty(n, dtype=np.int32)
    lib().orc_synth_ids(seed, stream, n, vocab, _p(out))
    return out


def gemv(W: np.ndarray, dtype: int, x: np.ndarray) -> np.ndarray:
    N, K = W.shape
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, K)
    y = np.empty((x.shape[0], N), dtype=np.float32)
    lib().orc_gemv(dtype, _p(np.ascontiguousarray(W)), N, K, _p(x), x.shape[0], _p(y))
    return y


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float, wdtype: int = F32) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    B, d = x.reshape(-1, x.shape[-1]).shape
    y = np.empty_like(x)
    lib().orc_rmsnorm(_p(x), _p(np.ascontiguousarray(w)), wdtype, B, d, eps, _p(y))
    return y


def rope_table(n_pos, head_dim, theta):
    c = np.empty((n_pos, head_dim // 2), dtype=np.float32)
    s = np.empty_like(c)
    lib().orc_rope_table(n_pos, head_dim, theta, _p(c), _p(s))
    return c, s


def rope_apply(v: np.ndarray, n_heads, head_dim, cos_row, sin_row):
    v = np.ascontiguousarray(v, dtype=np.float32).copy()
    lib().orc_rope_apply(_p(v), n_heads, head_dim, _p(np.ascontiguousarray(cos_row, np.float32)),
                         _p(np.ascontiguousarray(sin_row, np.float32)))
    return v


def swiglu(g, u):
    g = np.ascontiguousarray(g, np.float32)
    a = np.empty_like(g)
    lib().orc_swiglu(_p(g), _p(np.ascontiguousarray(u, np.float32)), g.size, _p(a))
    return a


def argmax(v):
    v = np.ascontiguousarray(v, np.float32)
    return int(lib().orc_argmax(_p(v), v.size))


def attention(q, Kc, Vc, kvdtype, n_heads, n_kv, head_dim, max_seq, length, first=0):
    """q [n_heads*hd] fp32; Kc/Vc [n_kv][max_seq][hd] in kvdtype storage; positions [first, length)
    -> o [n_heads*hd]."""
    q = np.ascontiguousarray(q, np.float32)
    o = np.empty(n_heads * head_dim, np.float32)
    scratch = np.empty(max(length, 1), np.float32)
    lib().orc_attention_from(_p(q), _p(np.ascontiguousarray(Kc)), _p(np.ascontiguousarray(Vc)), kvdtype, n_heads,
                             n_kv, head_dim, max_seq, first, length, _p(o), _p(scratch))
    return o


def sparse_first(min_len, window, global_tokens, block, pos):
    """First position a query at `pos` attends to under the reference's sparse mask (0: dense)."""
    return int(lib().orc_sparse_first(min_len, window, global_tokens, block, pos))


class Model:
    """Oracle Llama model (weights from a GGUF file or the seeded generator)."""

    def __init__(self, handle):
        self.h = handle
        cfg = OrcConfig()
        lib().orc_model_get_config(self.h, C.byref(cfg))
        self.cfg = cfg

    @classmethod
    def from_gguf(cls, path, kvdtype=F32, max_seq=512, max_batch=1, legacy_q4=0):
        h = C.c_void_p()
        rc = lib().orc_model_load_gguf_ex(path.encode(), kvdtype, max_seq, max_batch, legacy_q4, C.byref(h))
        if rc != 0:
            raise RuntimeError(f"oracle GGUF load failed: {rc}")
        return cls(h)

    @classmethod
    def synthetic(cls, *, n_layers, d, n_heads, n_kv, ffn, vocab, rope_theta=10000.0, eps=1e-5,
                  wdtype=F16, kvdtype=F16, max_seq=512, max_batch=1, seed=0, sigma=0.02):
        cfg = OrcConfig(n_layers, d, n_heads, n_kv, d // n_heads, ffn, vocab, rope_theta, eps, wdtype, kvdtype,
                        max_seq, max_batch)
        h = C.c_void_p()
        rc = lib().orc_model_synthetic(C.byref(cfg), seed, sigma, C.byref(h))
        if rc != 0:
            raise RuntimeError(f"oracle synthetic model failed: {rc}")
        return cls(h)

    def close(self):
        if self.h:
            lib().orc_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def clear_kv(self):
        lib().orc_model_clear_kv(self.h)

    def set_sparse(self, min_len=8192, window=512, global_tokens=16, block=1024):
        """Sparse long-context attention for later steps (min_len 0: dense)."""
        if lib().orc_model_set_sparse(self.h, min_len, window, global_tokens, block) != 0:
            raise RuntimeError("bad sparse mask")

    def fill_kv_synthetic(self, seed, sigma, n_pos, batch):
        rc = lib().orc_model_fill_kv_synthetic(self.h, seed, sigma, n_pos, batch)
        if rc != 0:
            raise RuntimeError(f"fill_kv failed {rc}")

    def step(self, ids, pos, want_logits=True):
        ids = np.ascontiguousarray(ids, np.int32).reshape(-1)
        pos = np.ascontiguousarray(pos, np.int32).reshape(-1)
        B = ids.size
        logits = np.empty((B, self.cfg.vocab), np.float32) if want_logits else None
        out = np.empty(B, np.int32)
        rc = lib().orc_model_step(self.h, B, _p(ids), _p(pos), _p(logits) if want_logits else None, _p(out))
        if rc != 0:
            raise RuntimeError(f"oracle step failed: {rc}")
        return out, logits

    def greedy(self, prompt, n_new, want_logits=False):
        """Token-by-token prompt then greedy decode (B = 1). Returns (ids, logits per step)."""
        self.clear_kv()
        pos = 0
        out_ids, all_logits = [], []
        nxt = None
        for t in prompt:
            nxt, lg = self.step([t], [pos], want_logits)
            pos += 1
        for _ in range(n_new):
            tok = int(nxt[0])
            out_ids.append(tok)
            if want_logits:
                all_logits.append(lg[0].copy())
            nxt, lg = self.step([tok], [pos], want_logits)
            pos += 1
        return out_ids, all_logits
