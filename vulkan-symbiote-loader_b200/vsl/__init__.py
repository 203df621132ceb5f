"""Python binding of libvsl.so (include/vsl.h) through ctypes.

The product is the C ABI; this module only marshals arguments for tests, the benchmark and
Python users. There is no fallback: if lib/libvsl.so is missing or a call fails, a
VslError is raised. Device buffers are passed as raw pointers (e.g. torch `data_ptr()`),
streams as `cudaStream_t` integers.
"""
from __future__ import annotations

import ctypes as C
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
# VSL_LIBRARY=trace selects the trace build (lib/libvsl_trace.so, `make trace`): the same kernels
# stamping a per-CTA timeline, read with trace_records()
LIB_PATH = os.path.join(PKG, "lib", "libvsl_trace.so" if os.environ.get("VSL_LIBRARY") == "trace" else "libvsl.so")
HEADER = os.path.join(os.path.dirname(PKG), "include", "vsl.h")

F32, F16, BF16 = 0, 1, 30
Q4_0, Q4_1, Q8_0 = 2, 3, 8  # weights only (block-quantized device layout)
EPI_STORE, EPI_ADD, EPI_SWIGLU = 0, 1, 2
ERR = {0: "OK", -1: "INVALID", -2: "CUDA", -3: "NCCL", -4: "TIMEOUT", -5: "BOUNDS", -6: "IO", -7: "FORMAT",
       -8: "OOM", -9: "UNSUPPORTED", -10: "STATE"}


class VslError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"VSL_ERR_{ERR.get(code, code)} ({code}): {msg}")
        self.code = code


class ModelConfig(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("d_model", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int),
                ("head_dim", C.c_int), ("ffn", C.c_int), ("vocab", C.c_int), ("rope_theta", C.c_float),
                ("rms_eps", C.c_float), ("wdtype", C.c_int)]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_}


class SparseMask(C.Structure):
    """vsl_sparse_mask: the reference's long-context window (min_len 0: dense)."""
    _fields_ = [("min_len", C.c_int), ("window", C.c_int), ("global_tokens", C.c_int), ("block", C.c_int)]


class EngineOptions(C.Structure):
    _fields_ = [("device", C.c_int), ("max_batch", C.c_int), ("max_seq", C.c_int), ("kv_dtype", C.c_int),
                ("page_size", C.c_int), ("split_len", C.c_int), ("tp_rank", C.c_int), ("tp_size", C.c_int),
                ("nccl_id", C.c_void_p), ("vram_budget_gb", C.c_double), ("use_graph", C.c_int),
                ("use_pdl", C.c_int), ("use_fused", C.c_int),
                ("use_p2p", C.c_int), ("legacy_q4", C.c_int), ("sparse_min_len", C.c_int),
                ("sparse_window", C.c_int), ("sparse_global", C.c_int), ("sparse_block", C.c_int),
                ("attn_route", C.c_int), ("attn_prefetch", C.c_int), ("p2p_chunk_bytes", C.c_int),
                ("nccl_timeout_ms", C.c_int)]


_lib = None


def lib() -> C.CDLL:
    """Load libvsl.so (built by `make -C vulkan-symbiote-loader_b200`). Raises if absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise VslError(-10, f"{LIB_PATH} is missing: build it with `make -C {PKG}` (no CPU fallback exists)")
    L = C.CDLL(LIB_PATH)
    vp, i32, u64, f32, f64, sz = C.c_void_p, C.c_int, C.c_uint64, C.c_float, C.c_double, C.c_size_t
    sig = {
        "vsl_last_error_string": (C.c_char_p, []),
        "vsl_version": (i32, []),
        "vsl_embed_gather": (i32, [i32, vp, i32, i32, vp, i32, vp, vp]),
        "vsl_rmsnorm": (i32, [vp, vp, i32, i32, f32, vp, vp]),
        "vsl_gemv": (i32, [i32, vp, i32, i32, vp, i32, vp, i32, vp, f32, vp]),
        "vsl_skinny_gemm_tc_workspace_size": (i32, [i32, i32, i32, C.POINTER(sz)]),
        "vsl_skinny_gemm_tc": (i32, [i32, vp, i32, i32, vp, i32, vp, i32, vp, f32, vp, sz, vp]),
        "vsl_qkv_rope_append": (i32, [i32, vp, i32, i32, i32, i32, vp, vp, f32, i32, vp, vp, vp, vp, vp, vp, i32, vp,
                                      i32, i32, vp]),
        "vsl_flash_decode_workspace_size": (i32, [i32, i32, i32, i32, i32, i32, C.POINTER(sz)]),
        "vsl_flash_decode": (i32, [vp, vp, vp, i32, vp, i32, i32, vp, i32, i32, i32, i32, i32, i32, vp, vp, sz, vp]),
        "vsl_flash_decode_tc_workspace_size": (i32, [i32, i32, C.POINTER(sz)]),
        "vsl_flash_decode_tc": (i32, [vp, vp, vp, i32, vp, i32, i32, vp, i32, i32, i32, i32, i32, vp, vp, sz, vp]),
        "vsl_lm_head_sample": (i32, [i32, vp, i32, i32, vp, vp, f32, i32, vp, vp, i32, f32, u64, vp, vp]),
        "vsl_argmax": (i32, [vp, i32, i32, vp, vp]),
        "vsl_synth_fill": (i32, [vp, i32, u64, u64, u64, u64, f64, vp]),
        "vsl_engine_default_options": (None, [C.POINTER(EngineOptions)]),
        "vsl_nccl_unique_id": (i32, [vp]),
        "vsl_gguf_model_config": (i32, [C.c_char_p, C.POINTER(ModelConfig)]),
        "vsl_weight_row_bytes": (i32, [i32, i32, C.POINTER(sz)]),
        "vsl_tokenizer_create_gguf": (i32, [C.c_char_p, C.POINTER(vp)]),
        "vsl_tokenizer_destroy": (None, [vp]),
        "vsl_tokenizer_info": (i32, [vp, C.POINTER(i32), C.POINTER(i32), C.POINTER(i32), C.POINTER(i32)]),
        "vsl_tokenize": (i32, [vp, C.c_char_p, sz, vp, i32, C.POINTER(i32)]),
        "vsl_detokenize": (i32, [vp, vp, i32, C.c_char_p, sz, C.POINTER(sz)]),
        "vsl_synth_fill_q": (i32, [vp, i32, sz, u64, u64, sz, sz, f64, vp]),
        "vsl_repack_gguf_rows": (i32, [i32, vp, sz, sz, sz, sz, sz, vp, sz, i32]),
        "vsl_gguf_tensor_info": (i32, [C.c_char_p, C.c_char_p, C.POINTER(i32), C.POINTER(u64), C.POINTER(u64)]),
        "vsl_engine_create_gguf": (i32, [C.c_char_p, C.POINTER(EngineOptions), C.POINTER(vp)]),
        "vsl_engine_create_synthetic": (i32, [C.POINTER(ModelConfig), u64, f64, C.POINTER(EngineOptions),
                                              C.POINTER(vp)]),
        "vsl_engine_destroy": (i32, [vp]),
        "vsl_engine_get_config": (i32, [vp, C.POINTER(ModelConfig)]),
        "vsl_engine_reset": (i32, [vp]),
        "vsl_engine_fill_kv_synthetic": (i32, [vp, u64, f64, i32, i32]),
        "vsl_engine_set_forced": (i32, [vp, vp, i32, i32]),
        "vsl_engine_run": (i32, [vp, i32, i32, f32, u64]),
        "vsl_engine_step_host": (i32, [vp, vp, i32, vp, vp]),
        "vsl_engine_read_tokens": (i32, [vp, i32, i32, vp]),
        "vsl_engine_positions": (i32, [vp, i32, vp]),
        "vsl_engine_generate": (i32, [vp, vp, i32, i32, f32, u64, vp, i32, vp, C.POINTER(i32)]),
        "vsl_engine_stream": (vp, [vp]),
        "vsl_engine_step_stats": (i32, [vp, i32, C.POINTER(i32), C.POINTER(f64)]),
        "vsl_engine_device_status": (i32, [vp, C.POINTER(i32)]),
        "vsl_engine_memory_stats": (i32, [vp, C.POINTER(sz), C.POINTER(sz), C.POINTER(sz)]),
        "vsl_engine_prefill": (i32, [vp, vp, i32, i32, C.POINTER(i32), vp]),
        "vsl_engine_reset_seq": (i32, [vp, i32]),
        "vsl_engine_generate_batch": (i32, [vp, vp, vp, i32, i32, C.c_float, C.c_uint64, vp, i32, vp, vp]),
        "vsl_engine_residency": (i32, [vp, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32), C.POINTER(u64),
                                       C.POINTER(u64)]),
        "vsl_pack_plan": (i32, [u64, C.c_uint32, u64, f64, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32)]),
        "vsl_p2p_buffer_size": (i32, [i32, sz, C.POINTER(sz)]),
        "vsl_p2p_allreduce": (i32, [C.POINTER(vp), i32, i32, sz, vp, i32, i32, vp, vp, u64, vp]),
        "vsl_engine_inject_status": (i32, [vp, i32]),
        "vsl_flash_decode_sparse": (i32, [vp, vp, vp, i32, vp, i32, i32, vp, i32, i32, i32, i32, i32, i32, vp, vp, sz,
                                          C.POINTER(SparseMask), vp]),
        "vsl_flash_decode_short": (i32, [vp, vp, vp, i32, vp, i32, i32, vp, i32, i32, i32, i32, i32, vp,
                                         C.POINTER(SparseMask), vp, vp]),
        "vsl_flash_prefill": (i32, [vp, vp, vp, i32, vp, i32, i32, vp, i32, i32, i32, i32, i32, vp,
                                    C.POINTER(SparseMask), vp, vp]),
        "vsl_flash_decode_tc_sparse": (i32, [vp, vp, vp, i32, vp, i32, i32, vp, i32, i32, i32, i32, i32, vp, vp, sz,
                                             C.POINTER(SparseMask), vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


TRACE_UNITS = ("gemv", "attention", "p2p", "tc", "prefill", "attention_tc")


def trace_records(reset: bool = True):
    """Per-CTA records of the trace build (id, blk, tag, smid, t0, t1, t2 ns), all units."""
    import numpy as np
    rec = np.dtype([("id", "<u4"), ("blk", "<u4"), ("tag", "<u4"), ("smid", "<u4"), ("t0", "<u8"), ("t1", "<u8"),
                    ("t2", "<u8"), ("pad", "<u8")])
    L = lib()
    out = []
    for unit in TRACE_UNITS:
        fn = getattr(L, "vsl_trace_read_" + unit, None)
        if fn is None:
            raise VslError(-10, "trace_records needs the trace build (VSL_LIBRARY=trace, make trace)")
        fn.restype = C.c_int
        fn.argtypes = [C.c_void_p, C.c_uint, C.c_int]
        buf = np.zeros(1 << 20, rec)
        n = fn(buf.ctypes.data, buf.size, 1 if reset else 0)
        if n < 0:
            raise VslError(-2, f"trace read of {unit} failed ({n})")
        out.append(buf[:n])
    return np.concatenate(out)


def header_functions() -> list[str]:
    """Names of every function include/vsl.h declares."""
    with open(HEADER) as f:
        text = f.read()
    return sorted(set(re.findall(r"^VSL_API\s+[\w\s\*]+?\b(vsl_\w+)\s*\(", text, flags=re.M)))


def check(rc: int):
    if rc != 0:
        raise VslError(rc, lib().vsl_last_error_string().decode(errors="replace"))


def _ptr(x):
    """Device/host pointer of a torch tensor, numpy array, int or None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if hasattr(x, "ctypes"):
        return x.ctypes.data
    raise TypeError(f"cannot take a pointer of {type(x)}")


# ---------------------------------------------------------------------------------------
# kernel wrappers (pointers in, status checked)
# ---------------------------------------------------------------------------------------

def embed_gather(dtype, table, V, d, ids, B, x, stream=0):
    check(lib().vsl_embed_gather(dtype, _ptr(table), V, d, _ptr(ids), B, _ptr(x), stream))


def rmsnorm(x, w, B, d, eps, y, stream=0):
    check(lib().vsl_rmsnorm(_ptr(x), _ptr(w), B, d, eps, _ptr(y), stream))


def gemv(wdtype, W, N, K, x, B, y, epilogue=EPI_STORE, norm_w=None, eps=0.0, stream=0):
    check(lib().vsl_gemv(wdtype, _ptr(W), N, K, _ptr(x), B, _ptr(y), epilogue, _ptr(norm_w), eps, stream))


class Tokenizer:
    """SentencePiece BPE of a GGUF vocabulary (tokenizer.ggml.model "llama"), else the
    reference's byte-level behaviour."""

    def __init__(self, path: str):
        self.h = C.c_void_p()
        check(lib().vsl_tokenizer_create_gguf(path.encode(), C.byref(self.h)))
        v, sw, bos, eos = C.c_int(), C.c_int(), C.c_int(), C.c_int()
        check(lib().vsl_tokenizer_info(self.h, C.byref(v), C.byref(sw), C.byref(bos), C.byref(eos)))
        self.vocab_size, self.is_subword, self.bos_id, self.eos_id = v.value, bool(sw.value), bos.value, eos.value

    def encode(self, text: str) -> list[int]:
        import numpy as np
        b = text.encode("utf-8")
        n = C.c_int()
        cap = 2 * len(b) + 8
        out = np.empty(cap, np.int32)
        rc = lib().vsl_tokenize(self.h, b, len(b), out.ctypes.data, cap, C.byref(n))
        if rc == -5 and n.value > cap:  # VSL_ERR_BOUNDS: n holds the count needed
            out = np.empty(n.value, np.int32)
            rc = lib().vsl_tokenize(self.h, b, len(b), out.ctypes.data, n.value, C.byref(n))
        check(rc)
        return out[:n.value].tolist()

    def decode(self, ids) -> str:
        import numpy as np
        a = np.ascontiguousarray(ids, np.int32)
        n = C.c_size_t()
        lib().vsl_detokenize(self.h, a.ctypes.data, a.size, None, 0, C.byref(n))  # size query
        buf = C.create_string_buffer(max(n.value, 1))
        check(lib().vsl_detokenize(self.h, a.ctypes.data, a.size, buf, n.value, C.byref(n)))
        return buf.raw[:n.value].decode("utf-8", errors="replace")

    def close(self):
        if self.h:
            lib().vsl_tokenizer_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def weight_row_bytes(dtype: int, K: int) -> int:
    """Bytes of one weight row of K elements in device layout (quantized rows include scales)."""
    out = C.c_size_t()
    check(lib().vsl_weight_row_bytes(dtype, K, C.byref(out)))
    return out.value


def synth_fill_q(dst, dtype: int, seed: int, tid: int, rows: int, cols: int, sigma: float = 0.02, stream=0):
    """Seeded Q8_0 / Q4_0 / Q4_1 tensor [rows][cols] into device memory in the device row layout."""
    check(lib().vsl_synth_fill_q(_ptr(dst), dtype, weight_row_bytes(dtype, cols), seed, tid, rows, cols, sigma,
                                 stream))


def repack_gguf_rows(dtype: int, blocks, rows: int, cols: int, legacy_q4: bool = False, row0: int = 0,
                     nrows: int | None = None, col0: int = 0, ncols: int | None = None):
    """GGUF Q8_0 / Q4_0 / Q4_1 block bytes ([rows][cols / 32 blocks], host) -> device row layout (uint8
    numpy array [nrows][weight_row_bytes(dtype, ncols)])."""
    import numpy as np
    nrows = rows - row0 if nrows is None else nrows
    ncols = cols - col0 if ncols is None else ncols
    b = np.ascontiguousarray(blocks, np.uint8)
    pitch = weight_row_bytes(dtype, ncols)
    out = np.zeros((nrows, pitch), np.uint8)
    check(lib().vsl_repack_gguf_rows(dtype, b.ctypes.data, cols, row0, nrows, col0, ncols, out.ctypes.data, pitch,
                                     1 if legacy_q4 else 0))
    return out


def skinny_gemm_tc_workspace_size(N, K, B) -> int:
    out = C.c_size_t()
    check(lib().vsl_skinny_gemm_tc_workspace_size(N, K, B, C.byref(out)))
    return out.value


def skinny_gemm_tc(wdtype, W, N, K, x, B, y, epilogue=EPI_STORE, norm_w=None, eps=0.0, workspace=None,
                   workspace_bytes=0, stream=0):
    check(lib().vsl_skinny_gemm_tc(wdtype, _ptr(W), N, K, _ptr(x), B, _ptr(y), epilogue, _ptr(norm_w), eps,
                                   _ptr(workspace), workspace_bytes, stream))


def qkv_rope_append(wdtype, Wqkv, n_heads, n_kv, head_dim, K, x, norm_w, eps, B, pos, rope_cos, rope_sin, q_out,
                    k_cache, v_cache, kvdtype, page_table, max_pages, page_size, stream=0):
    check(lib().vsl_qkv_rope_append(wdtype, _ptr(Wqkv), n_heads, n_kv, head_dim, K, _ptr(x), _ptr(norm_w), eps, B,
                                    _ptr(pos), _ptr(rope_cos), _ptr(rope_sin), _ptr(q_out), _ptr(k_cache),
                                    _ptr(v_cache), kvdtype, _ptr(page_table), max_pages, page_size, stream))


def flash_decode_workspace_size(B, n_heads, n_kv, head_dim, max_len, split_len) -> int:
    out = C.c_size_t()
    check(lib().vsl_flash_decode_workspace_size(B, n_heads, n_kv, head_dim, max_len, split_len, C.byref(out)))
    return out.value


def flash_decode(q, k_cache, v_cache, kvdtype, page_table, max_pages, page_size, pos, B, n_heads, n_kv, head_dim,
                 max_len, split_len, out, workspace, workspace_bytes, stream=0, sparse=None):
    """sparse: None (dense) or (min_len, window, global_tokens, block) -> vsl_flash_decode_sparse."""
    if sparse is None:
        check(lib().vsl_flash_decode(_ptr(q), _ptr(k_cache), _ptr(v_cache), kvdtype, _ptr(page_table), max_pages,
                                     page_size, _ptr(pos), B, n_heads, n_kv, head_dim, max_len, split_len, _ptr(out),
                                     _ptr(workspace), workspace_bytes, stream))
        return
    m = SparseMask(*sparse)
    check(lib().vsl_flash_decode_sparse(_ptr(q), _ptr(k_cache), _ptr(v_cache), kvdtype, _ptr(page_table), max_pages,
                                        page_size, _ptr(pos), B, n_heads, n_kv, head_dim, max_len, split_len, _ptr(out),
                                        _ptr(workspace), workspace_bytes, C.byref(m), stream))


def flash_decode_tc_workspace_size(B, n_kv) -> int:
    out = C.c_size_t()
    check(lib().vsl_flash_decode_tc_workspace_size(B, n_kv, C.byref(out)))
    return out.value


def flash_decode_tc(q, k_cache, v_cache, n_pages, page_table, max_pages, page_size, pos, B, n_heads, n_kv, head_dim,
                    max_len, out, workspace, workspace_bytes, stream=0, sparse=None):
    """sparse: None (dense) or (min_len, window, global_tokens, block) -> vsl_flash_decode_tc_sparse."""
    if sparse is None:
        check(lib().vsl_flash_decode_tc(_ptr(q), _ptr(k_cache), _ptr(v_cache), n_pages, _ptr(page_table), max_pages,
                                        page_size, _ptr(pos), B, n_heads, n_kv, head_dim, max_len, _ptr(out),
                                        _ptr(workspace), workspace_bytes, stream))
        return
    m = SparseMask(*sparse)
    check(lib().vsl_flash_decode_tc_sparse(_ptr(q), _ptr(k_cache), _ptr(v_cache), n_pages, _ptr(page_table),
                                           max_pages, page_size, _ptr(pos), B, n_heads, n_kv, head_dim, max_len,
                                           _ptr(out), _ptr(workspace), workspace_bytes, C.byref(m), stream))


def flash_decode_short(q, k_cache, v_cache, kvdtype, page_table, max_pages, page_size, pos, B, n_heads, n_kv,
                       head_dim, max_len, out, sparse=None, status=None, stream=0):
    """Short-cache decode attention (one CTA per sequence and KV group; no workspace).
    sparse: None (dense) or (min_len, window, global_tokens, block)."""
    m = C.byref(SparseMask(*sparse)) if sparse is not None else None
    check(lib().vsl_flash_decode_short(_ptr(q), _ptr(k_cache), _ptr(v_cache), kvdtype, _ptr(page_table), max_pages,
                                       page_size, _ptr(pos), B, n_heads, n_kv, head_dim, max_len, _ptr(out), m,
                                       _ptr(status), stream))


def flash_prefill(q, k_cache, v_cache, n_pages, page_row, max_pages, page_size, pos, n_rows, n_heads, n_kv, head_dim,
                  max_len, out, sparse=None, status=None, stream=0):
    """Prompt attention of n_rows rows of one sequence (page_row: its page-table row).
    sparse: None (dense) or (min_len, window, global_tokens, block)."""
    m = C.byref(SparseMask(*sparse)) if sparse is not None else None
    check(lib().vsl_flash_prefill(_ptr(q), _ptr(k_cache), _ptr(v_cache), n_pages, _ptr(page_row), max_pages,
                                  page_size, _ptr(pos), n_rows, n_heads, n_kv, head_dim, max_len, _ptr(out), m,
                                  _ptr(status), stream))


def lm_head_sample(wdtype, W, V_local, K, x, norm_w, eps, B, logits, slots, vocab_offset=0, temperature=0.0,
                   seed=0, step_counter=None, stream=0):
    check(lib().vsl_lm_head_sample(wdtype, _ptr(W), V_local, K, _ptr(x), _ptr(norm_w), eps, B, _ptr(logits),
                                   _ptr(slots), vocab_offset, temperature, seed, _ptr(step_counter), stream))


def argmax(logits, B, V, out, stream=0):
    check(lib().vsl_argmax(_ptr(logits), B, V, _ptr(out), stream))


def synth_fill(dst, dtype, seed, tid, start, n, sigma, stream=0):
    check(lib().vsl_synth_fill(_ptr(dst), dtype, seed, tid, start, n, sigma, stream))


def gguf_model_config(path: str) -> dict:
    cfg = ModelConfig()
    check(lib().vsl_gguf_model_config(path.encode(), C.byref(cfg)))
    return cfg.as_dict()


def gguf_tensor_info(path: str, name: str):
    t = C.c_int()
    ne = (C.c_uint64 * 4)()
    off = C.c_uint64()
    check(lib().vsl_gguf_tensor_info(path.encode(), name.encode(), C.byref(t), ne, C.byref(off)))
    return t.value, [int(v) for v in ne if v], off.value


def p2p_buffer_size(n_ranks: int, cap_bytes: int) -> int:
    n = C.c_size_t(0)
    check(lib().vsl_p2p_buffer_size(n_ranks, cap_bytes, C.byref(n)))
    return n.value


def p2p_allreduce(bases, rank: int, cap_bytes: int, data, n: int, op: int, epochs, status=None, wait_ns: int = 10**9,
                  stream=0):
    """One-shot peer-memory all-reduce (vsl_p2p_allreduce): bases = the ranks' receive buffers."""
    arr = (C.c_void_p * len(bases))(*[_ptr(b) for b in bases])
    check(lib().vsl_p2p_allreduce(arr, len(bases), rank, cap_bytes, _ptr(data), n, op, _ptr(epochs), _ptr(status),
                                  wait_ns, _ptr(stream)))


def pack_plan(layer_bytes: int, n_layers: int, fixed_bytes: int, budget_gb: float) -> tuple[int, int]:
    """(resident_layers, streamed_layers) the engine would choose under `budget_gb`."""
    r, st = C.c_uint32(), C.c_uint32()
    check(lib().vsl_pack_plan(layer_bytes, n_layers, fixed_bytes, budget_gb, C.byref(r), C.byref(st)))
    return r.value, st.value


def nccl_unique_id() -> bytes:
    buf = (C.c_uint8 * 128)()
    check(lib().vsl_nccl_unique_id(buf))
    return bytes(buf)


def default_options(**kw) -> EngineOptions:
    o = EngineOptions()
    lib().vsl_engine_default_options(C.byref(o))
    for k, v in kw.items():
        if not hasattr(o, k):
            raise KeyError(k)
        setattr(o, k, v)
    return o


class Engine:
    """Decode engine (one GPU / one tensor-parallel rank)."""

    def __init__(self, handle: C.c_void_p, keep=None):
        self.h = handle
        self._keep = keep  # keeps the NCCL id buffer alive for the engine's lifetime
        cfg = ModelConfig()
        check(lib().vsl_engine_get_config(self.h, C.byref(cfg)))
        self.config = cfg.as_dict()

    @staticmethod
    def _opts(nccl_id, **kw):
        keep = None
        if nccl_id is not None:
            keep = (C.c_uint8 * 128).from_buffer_copy(nccl_id)
            kw["nccl_id"] = C.cast(keep, C.c_void_p)
        return default_options(**kw), keep

    @classmethod
    def from_gguf(cls, path: str, nccl_id: bytes | None = None, **opts) -> "Engine":
        o, keep = cls._opts(nccl_id, **opts)
        h = C.c_void_p()
        check(lib().vsl_engine_create_gguf(path.encode(), C.byref(o), C.byref(h)))
        return cls(h, keep)

    @classmethod
    def synthetic(cls, cfg: dict, seed: int = 0, sigma: float = 0.02, nccl_id: bytes | None = None,
                  **opts) -> "Engine":
        mc = ModelConfig(**{k: cfg[k] for k, _ in ModelConfig._fields_})
        o, keep = cls._opts(nccl_id, **opts)
        h = C.c_void_p()
        check(lib().vsl_engine_create_synthetic(C.byref(mc), seed, sigma, C.byref(o), C.byref(h)))
        return cls(h, keep)

    def close(self):
        if self.h:
            check(lib().vsl_engine_destroy(self.h))
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self):
        check(lib().vsl_engine_reset(self.h))

    def fill_kv_synthetic(self, seed: int, sigma: float, n_pos: int, batch: int):
        check(lib().vsl_engine_fill_kv_synthetic(self.h, seed, sigma, n_pos, batch))

    def set_forced(self, ids):
        import numpy as np
        a = np.ascontiguousarray(ids, dtype=np.int32)
        if a.ndim == 1:
            a = a[:, None]
        check(lib().vsl_engine_set_forced(self.h, a.ctypes.data, a.shape[0], a.shape[1]))

    def run(self, n_steps: int, batch: int = 1, temperature: float = 0.0, seed: int = 0):
        check(lib().vsl_engine_run(self.h, n_steps, batch, temperature, seed))

    def step_host(self, ids, want_logits: bool = False):
        import numpy as np
        a = np.ascontiguousarray(ids, dtype=np.int32).reshape(-1)
        out = np.empty(a.size, np.int32)
        lg = np.empty((a.size, self.config["vocab"]), np.float32) if want_logits else None
        check(lib().vsl_engine_step_host(self.h, a.ctypes.data, a.size, out.ctypes.data,
                                         lg.ctypes.data if lg is not None else None))
        return out, lg

    def read_tokens(self, n: int, batch: int = 1):
        import numpy as np
        out = np.empty((n, batch), np.int32)
        check(lib().vsl_engine_read_tokens(self.h, n, batch, out.ctypes.data))
        return out

    def positions(self, batch: int = 1):
        import numpy as np
        out = np.empty(batch, np.int32)
        check(lib().vsl_engine_positions(self.h, batch, out.ctypes.data))
        return out

    def generate(self, prompt, max_new: int, temperature: float = 0.0, seed: int = 0, stop_ids=()):
        import numpy as np
        p = np.ascontiguousarray(prompt, np.int32)
        st = np.ascontiguousarray(list(stop_ids), np.int32) if len(stop_ids) else None
        out = np.empty(max(max_new, 1), np.int32)
        n = C.c_int()
        check(lib().vsl_engine_generate(self.h, p.ctypes.data, p.size, max_new, temperature, seed,
                                        st.ctypes.data if st is not None else None, 0 if st is None else st.size,
                                        out.ctypes.data, C.byref(n)))
        return out[:n.value].tolist()

    @property
    def stream(self) -> int:
        return lib().vsl_engine_stream(self.h) or 0

    def step_stats(self, batch: int = 1):
        k = C.c_int()
        b = C.c_double()
        check(lib().vsl_engine_step_stats(self.h, batch, C.byref(k), C.byref(b)))
        return k.value, b.value

    def memory_stats(self):
        w, kv, o = C.c_size_t(), C.c_size_t(), C.c_size_t()
        check(lib().vsl_engine_memory_stats(self.h, C.byref(w), C.byref(kv), C.byref(o)))
        return dict(weights=w.value, kv=kv.value, other=o.value)

    def prefill(self, ids, seq: int = 0, want_logits: bool = False):
        """Prompt pass for sequence `seq`; returns (next id, logits of the last prompt token or None)."""
        import numpy as np
        a = np.ascontiguousarray(ids, dtype=np.int32).reshape(-1)
        nxt = C.c_int()
        lg = np.empty(self.config["vocab"], np.float32) if want_logits else None
        check(lib().vsl_engine_prefill(self.h, a.ctypes.data, a.size, seq, C.byref(nxt),
                                       lg.ctypes.data if lg is not None else None))
        return nxt.value, lg

    def reset_seq(self, seq: int):
        check(lib().vsl_engine_reset_seq(self.h, seq))

    def generate_batch(self, prompts, max_new: int, temperature: float = 0.0, seed: int = 0, stop_ids=()):
        """One prompt pass per sequence, then batched decode; returns one id list per prompt."""
        import numpy as np
        flat = np.ascontiguousarray(np.concatenate([np.asarray(p, np.int32).reshape(-1) for p in prompts]), np.int32)
        lens = np.ascontiguousarray([len(p) for p in prompts], np.int32)
        st = np.ascontiguousarray(list(stop_ids), np.int32) if len(stop_ids) else None
        out = np.zeros((len(prompts), max(max_new, 1)), np.int32)
        n = np.zeros(len(prompts), np.int32)
        check(lib().vsl_engine_generate_batch(self.h, flat.ctypes.data, lens.ctypes.data, len(prompts), max_new,
                                              temperature, seed, st.ctypes.data if st is not None else None,
                                              0 if st is None else st.size, out.ctypes.data, n.ctypes.data))
        return [out[b, :n[b]].tolist() for b in range(len(prompts))]

    def residency(self) -> dict:
        """Weight residency under the HBM budget (layers kept in HBM / streamed each step)."""
        r, st = C.c_uint32(), C.c_uint32()
        sb, hb = C.c_uint64(), C.c_uint64()
        check(lib().vsl_engine_residency(self.h, C.byref(r), C.byref(st), C.byref(sb), C.byref(hb)))
        return {"resident_layers": r.value, "streamed_layers": st.value, "streamed_bytes_per_step": sb.value,
                "host_bytes": hb.value}

    def device_status(self) -> int:
        s = C.c_int()
        check(lib().vsl_engine_device_status(self.h, C.byref(s)))
        return s.value

    def inject_status(self, code: int):
        """Test hook: set the sticky device status word (host-made failure)."""
        check(lib().vsl_engine_inject_status(self.h, code))
